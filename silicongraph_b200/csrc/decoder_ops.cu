// Glue kernels of the decoder layer around the linear and attention kernels:
//   qkv_rope_append: the fused QKV projection output [T, (H + 2 Hkv) * D] is
//     split, q and k are rotated (rope_apply_neon, matmul_neon.h:262-275),
//     q is written head-major [H, T, D] for attention and k / v are appended to
//     the layer's KV cache rows (kv_cache_layout.cpp:16-53 flat layout
//     [K|V][kv_head][seq][dim], or the paged layout of :65-102, pages
//     [K|V][kv_head][16][dim] found through a page table) at each token's
//     position;
//   head_transpose: attention output [H, T, D] -> [T, H, D] for the output
//     projection.
// Positions come from a device array (so one captured decode step serves
// every position) or from pos0 + t.
#include "sm100.cuh"

namespace {

// Where a token's k / v rows go in a paged cache (pt == nullptr: flat).
struct PageView {
  const int32_t* pt;
  int64_t pt_bs, pt_ps, page_stride;
  int npages;
  int* err;
};

template <typename T>
__global__ void qkv_rope_append_kernel(const T* __restrict__ qkv, int T_, int Ts, int H, int Hkv, int D,
                                       const int32_t* __restrict__ pos, int pos0, float base, T* __restrict__ q_out,
                                       T* __restrict__ k_cache, T* __restrict__ v_cache, int64_t kv_head_stride,
                                       int64_t kv_batch_stride, PageView pv) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  const int half = D / 2;
  const int slots = H + 2 * Hkv;  // head slots per token: q heads, k heads, v heads
  const int64_t total = (int64_t)T_ * slots * half;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(e % half);
    const int64_t ts = e / half;
    const int slot = (int)(ts % slots);
    const int t = (int)(ts / slots);
    const int b = t / Ts, tl = t - b * Ts;  // sequence, token within it
    const int p = pos ? pos[tl] : pos0 + tl;
    const T* src = qkv + ((int64_t)t * slots + slot) * D;
    float x0 = (float)src[i], x1 = (float)src[i + half];
    if (slot < H + Hkv) {  // q and k rotate
      float y0, y1;
      sgd::rope_pair(x0, x1, p, i, D, base, &y0, &y1);
      x0 = y0;
      x1 = y1;
    }
    T* dst;
    if (slot < H) {
      dst = q_out + (((int64_t)b * H + slot) * Ts + tl) * D;
    } else {
      const bool is_k = slot < H + Hkv;
      const int hk = is_k ? slot - H : slot - H - Hkv;
      T* cache = is_k ? k_cache : v_cache;
      if (pv.pt) {
        const int pg = __ldg(pv.pt + (int64_t)b * pv.pt_bs + (int64_t)(p >> 4) * pv.pt_ps);
        if ((unsigned)pg >= (unsigned)pv.npages) {  // no such page: the row is dropped and reported
          if (i == 0) atomicOr(pv.err, 4);
          continue;
        }
        dst = cache + (int64_t)pg * pv.page_stride + ((int64_t)hk * 16 + (p & 15)) * D;
      } else {
        dst = cache + b * kv_batch_stride + hk * kv_head_stride + (int64_t)p * D;
      }
    }
    dst[i] = (T)x0;
    dst[i + half] = (T)x1;
  }
}

template <typename T>
__global__ void head_transpose_kernel(const T* __restrict__ in, T* __restrict__ out, int H, int T_, int D) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  const int64_t total = (int64_t)H * T_ * D;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(e % D);
    const int64_t ht = e / D;
    const int t = (int)(ht % T_);
    const int h = (int)(ht / T_);
    out[((int64_t)t * H + h) * D + d] = in[e];
  }
}

// y[t, j] = round(silu(gu[t, j])) * gu[t, F + j]  (gate and up halves of the fused projection)
template <typename T>
__global__ void swiglu_rows_kernel(const T* __restrict__ gu, T* __restrict__ y, int rows, int F) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  const int64_t total = (int64_t)rows * F;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(e % F);
    const int64_t t = e / F;
    // silu rounded as the reference's silu writes it, then the product
    y[e] = sgd::swiglu_value<T>((float)gu[t * 2 * F + j], (float)gu[t * 2 * F + F + j]);
  }
}

// Greedy token and its log-probability: out = argmax, logprob = x[out] - max - log(sum exp(x - max)).
__global__ void __launch_bounds__(256) argmax_logprob_kernel(const float* __restrict__ logits, int n,
                                                             int32_t* __restrict__ out, float* __restrict__ logprob) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float ss[32];
  const float* row = logits + (int64_t)blockIdx.x * n;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = row[i];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  best = lane < nw ? sv[lane] : -INFINITY;
  bi = lane < nw ? si[lane] : 0x7fffffff;
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  float sum = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) sum += expf(row[i] - best);
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) ss[w] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < nw; ++k) t += ss[k];
    const int idx = bi == 0x7fffffff ? 0 : bi;
    out[blockIdx.x] = idx;
    if (logprob) logprob[blockIdx.x] = row[idx] - best - logf(t);
  }
}

// Parallel form: each block reduces a slice of one row to (max, first index
// of the max, sum of exp(x - max)); one block per row merges the slices in
// order (equal maxima keep the lowest index).
constexpr int kArgSlice = 4096;

__global__ void __launch_bounds__(256) argmax_partial_kernel(const float* __restrict__ logits, int n, int slices,
                                                             float* __restrict__ part) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  __shared__ float sv[8], ssum[8];
  __shared__ int si[8];
  const int row = blockIdx.y, sl = blockIdx.x;
  const float* x = logits + (int64_t)row * n;
  const int i0 = sl * kArgSlice, i1 = min(n, i0 + kArgSlice);
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const float v = x[i];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  best = sv[0];
  bi = si[0];
  for (int k = 1; k < 8; ++k)
    if (sv[k] > best || (sv[k] == best && si[k] < bi)) {
      best = sv[k];
      bi = si[k];
    }
  float sum = 0.f;
  if (best != -INFINITY)
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) sum += expf(x[i] - best);
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) ssum[w] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += ssum[k];
    float* pp = part + ((int64_t)row * slices + sl) * 3;
    pp[0] = best;
    pp[1] = __int_as_float(bi);
    pp[2] = t;
  }
}

__global__ void argmax_merge_kernel(const float* __restrict__ logits, int n, int slices,
                                    const float* __restrict__ part, int32_t* __restrict__ out,
                                    float* __restrict__ logprob) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  if (threadIdx.x != 0) return;
  const int row = blockIdx.x;
  const float* pp = part + (int64_t)row * slices * 3;
  float M = -INFINITY;
  int idx = 0x7fffffff;
  for (int k = 0; k < slices; ++k) {
    const float m = pp[3 * k];
    const int i = __float_as_int(pp[3 * k + 1]);
    if (m > M || (m == M && i < idx)) {
      M = m;
      idx = i;
    }
  }
  float L = 0.f;
  if (M != -INFINITY)
    for (int k = 0; k < slices; ++k)
      if (pp[3 * k] != -INFINITY) L += pp[3 * k + 2] * expf(pp[3 * k] - M);
  const int r = idx == 0x7fffffff ? 0 : idx;
  out[row] = r;
  if (logprob) logprob[row] = logits[(int64_t)row * n + r] - M - logf(L);
}

int grid_of(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (int)(b < 1 ? 1 : (b > 148 * 16 ? 148 * 16 : b));
}

// Tensor-parallel greedy token: per-rank triples, then the pick over ranks (one row per sequence).
__global__ void tp_argmax_pack_kernel(const float* __restrict__ logits, int vocab_local, const int32_t* __restrict__ idx,
                                      const float* __restrict__ logprob, int vocab0, int rows, float* __restrict__ out) {
  sgd::pdl_wait();
  sgd::pdl_launch_dependents();
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const int i = idx[r];
    const float m = logits[(int64_t)r * vocab_local + i];
    out[3 * r] = m;
    out[3 * r + 1] = m - logprob[r];  // log-sum-exp of this rank's shard
    out[3 * r + 2] = (float)(vocab0 + i);
  }
}

__global__ void tp_argmax_pick_kernel(const float* __restrict__ all, int world, int rows, int32_t* __restrict__ next,
                                      float* __restrict__ logprob) {
  sgd::pdl_wait();
  sgd::pdl_launch_dependents();
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    int best = 0;
    float M = all[3 * r], Lmax = all[3 * r + 1];
    for (int w = 1; w < world; ++w) {
      const float* tw = all + 3 * ((int64_t)w * rows + r);
      if (tw[0] > M) {
        M = tw[0];
        best = w;
      }
      Lmax = fmaxf(Lmax, tw[1]);
    }
    float s = 0.f;
    for (int w = 0; w < world; ++w) s += expf(all[3 * ((int64_t)w * rows + r) + 1] - Lmax);
    next[r] = (int32_t)all[3 * ((int64_t)best * rows + r) + 2];
    if (logprob) logprob[r] = M - (Lmax + logf(s));
  }
}

}  // namespace

extern "C" {

static SgStatus qkv_rope_append_run(const void* qkv, int32_t batch, int32_t seq_tokens, int32_t heads, int32_t kv_heads,
                             int32_t head_dim, const int32_t* positions, int32_t pos0, float base, void* q_out,
                             void* k_cache, void* v_cache, int64_t kv_head_stride, int64_t kv_batch_stride,
                             const SgKvPages* pages, int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(batch >= 0 && seq_tokens >= 0 && heads > 0 && kv_heads > 0 && head_dim > 0,
               "sg_qkv_rope_append: bad size");
  const int64_t tokens = (int64_t)batch * seq_tokens;
  if (tokens == 0) return SG_OK;
  SG_CHECK_ARG(tokens <= INT32_MAX, "sg_qkv_rope_append: too many tokens");
  SG_CHECK_ARG(qkv && q_out && k_cache && v_cache, "sg_qkv_rope_append: NULL pointer");
  SG_CHECK_ARG(head_dim % 2 == 0, "sg_qkv_rope_append: head_dim %d is odd", head_dim);
  PageView pv{};
  if (pages) {
    SG_CHECK_ARG(pages->table && pages->num_pages > 0 && pages->page_size == 16,
                 "sg_qkv_rope_append_paged: needs a table, pages and 16 tokens per page");
    SG_CHECK_ARG(pages->page_stride >= (int64_t)kv_heads * 16 * head_dim,
                 "sg_qkv_rope_append_paged: page_stride smaller than a page's kv heads");
    pv.pt = pages->table;
    pv.pt_bs = pages->table_batch_stride;
    pv.pt_ps = pages->table_page_stride;
    pv.page_stride = pages->page_stride;
    pv.npages = pages->num_pages;
    SgStatus es = sg::device_error_word(&pv.err);
    if (es != SG_OK) return es;
  } else {
    SG_CHECK_ARG(kv_head_stride >= head_dim, "sg_qkv_rope_append: kv_head_stride < head_dim");
    SG_CHECK_ARG(batch == 1 || kv_batch_stride >= kv_heads * kv_head_stride,
                 "sg_qkv_rope_append: kv_batch_stride smaller than one sequence's cache");
  }
  const int dt = io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : io_dtype;
  SG_CHECK_ARG(dt == SG_DT_F16 || dt == SG_DT_BF16, "sg_qkv_rope_append: io_dtype %d unsupported", io_dtype);
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const int64_t total = tokens * (heads + 2 * kv_heads) * (head_dim / 2);
  if (dt == SG_DT_F16)
    SG_CUDA_TRY(sgd::launch_pdl(qkv_rope_append_kernel<__half>, dim3(grid_of(total)), dim3(256), 0, cs,
                                static_cast<const __half*>(qkv), (int)tokens, (int)seq_tokens, (int)heads,
                                (int)kv_heads, (int)head_dim, positions, (int)pos0, base, static_cast<__half*>(q_out),
                                static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), kv_head_stride,
                                kv_batch_stride, pv));
  else
    SG_CUDA_TRY(sgd::launch_pdl(qkv_rope_append_kernel<__nv_bfloat16>, dim3(grid_of(total)), dim3(256), 0, cs,
                                static_cast<const __nv_bfloat16*>(qkv), (int)tokens, (int)seq_tokens, (int)heads,
                                (int)kv_heads, (int)head_dim, positions, (int)pos0, base,
                                static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
                                static_cast<__nv_bfloat16*>(v_cache), kv_head_stride, kv_batch_stride, pv));
  return SG_OK;
}

SgStatus sg_qkv_rope_append_batched(const void* qkv, int32_t batch, int32_t seq_tokens, int32_t heads,
                                    int32_t kv_heads, int32_t head_dim, const int32_t* positions, int32_t pos0,
                                    float base, void* q_out, void* k_cache, void* v_cache, int64_t kv_head_stride,
                                    int64_t kv_batch_stride, int32_t io_dtype, void* stream) {
  return qkv_rope_append_run(qkv, batch, seq_tokens, heads, kv_heads, head_dim, positions, pos0, base, q_out, k_cache,
                             v_cache, kv_head_stride, kv_batch_stride, nullptr, io_dtype, stream);
}

SgStatus sg_qkv_rope_append_paged(const void* qkv, int32_t batch, int32_t seq_tokens, int32_t heads,
                                  int32_t kv_heads, int32_t head_dim, const int32_t* positions, int32_t pos0,
                                  float base, void* q_out, void* k_pages, void* v_pages, const SgKvPages* pages,
                                  int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(pages != nullptr, "sg_qkv_rope_append_paged: pages is NULL");
  return qkv_rope_append_run(qkv, batch, seq_tokens, heads, kv_heads, head_dim, positions, pos0, base, q_out,
                             k_pages, v_pages, 0, 0, pages, io_dtype, stream);
}

SgStatus sg_qkv_rope_append(const void* qkv, int32_t tokens, int32_t heads, int32_t kv_heads, int32_t head_dim,
                            const int32_t* positions, int32_t pos0, float base, void* q_out, void* k_cache,
                            void* v_cache, int64_t kv_head_stride, int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(tokens >= 0, "sg_qkv_rope_append: bad size");
  return sg_qkv_rope_append_batched(qkv, 1, tokens, heads, kv_heads, head_dim, positions, pos0, base, q_out, k_cache,
                                    v_cache, kv_head_stride, 0, io_dtype, stream);
}

SgStatus sg_head_transpose(const void* in, void* out, int32_t heads, int32_t tokens, int32_t head_dim,
                           int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(heads >= 0 && tokens >= 0 && head_dim >= 0, "sg_head_transpose: bad size");
  if ((int64_t)heads * tokens * head_dim == 0) return SG_OK;
  SG_CHECK_ARG(in && out, "sg_head_transpose: NULL pointer");
  const int dt = io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : io_dtype;
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const int64_t total = (int64_t)heads * tokens * head_dim;
  if (dt == SG_DT_F32)
    head_transpose_kernel<float><<<grid_of(total), 256, 0, cs>>>(static_cast<const float*>(in),
                                                                 static_cast<float*>(out), heads, tokens, head_dim);
  else
    head_transpose_kernel<uint16_t><<<grid_of(total), 256, 0, cs>>>(
        static_cast<const uint16_t*>(in), static_cast<uint16_t*>(out), heads, tokens, head_dim);
  return sg::check_launch("sg_head_transpose");
}

SgStatus sg_swiglu_rows(const void* gate_up, void* y, int32_t rows, int32_t ffn, int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(rows >= 0 && ffn >= 0, "sg_swiglu_rows: bad size");
  if ((int64_t)rows * ffn == 0) return SG_OK;
  SG_CHECK_ARG(gate_up && y, "sg_swiglu_rows: NULL pointer");
  const int dt = io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : io_dtype;
  SG_CHECK_ARG(dt == SG_DT_F16 || dt == SG_DT_BF16, "sg_swiglu_rows: io_dtype %d unsupported", io_dtype);
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const int64_t total = (int64_t)rows * ffn;
  if (dt == SG_DT_F16)
    SG_CUDA_TRY(sgd::launch_pdl(swiglu_rows_kernel<__half>, dim3(grid_of(total)), dim3(256), 0, cs,
                                static_cast<const __half*>(gate_up), static_cast<__half*>(y), (int)rows, (int)ffn));
  else
    SG_CUDA_TRY(sgd::launch_pdl(swiglu_rows_kernel<__nv_bfloat16>, dim3(grid_of(total)), dim3(256), 0, cs,
                                static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(y),
                                (int)rows, (int)ffn));
  return sg::check_launch("sg_swiglu_rows");
}

SgStatus sg_argmax_logprob(const float* logits, int32_t rows, int32_t n, int32_t* out, float* logprob, void* stream) {
  SG_CHECK_ARG(rows >= 0 && n >= 1, "sg_argmax_logprob: bad size");
  if (rows == 0) return SG_OK;
  SG_CHECK_ARG(logits && out, "sg_argmax_logprob: logits and out must be non-NULL");
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const int slices = (n + kArgSlice - 1) / kArgSlice;
  if (slices <= 1 || rows > 65535) {
    argmax_logprob_kernel<<<rows, 256, 0, cs>>>(logits, n, out, logprob);
    return sg::check_launch("sg_argmax_logprob");
  }
  void* ws = nullptr;
  SgStatus st = sg::library_workspace(stream, (size_t)rows * slices * 3 * sizeof(float), &ws, sg::kWsArgmax);
  if (st != SG_OK) return st;
  SG_CUDA_TRY(sgd::launch_pdl(argmax_partial_kernel, dim3(slices, rows), dim3(256), 0, cs, logits, (int)n, slices,
                              static_cast<float*>(ws)));
  SG_CUDA_TRY(sgd::launch_pdl(argmax_merge_kernel, dim3(rows), dim3(32), 0, cs, logits, (int)n, slices,
                              static_cast<const float*>(ws), out, logprob));
  return SG_OK;
}

SgStatus sg_tp_argmax_pack(const float* logits, int32_t rows, int32_t vocab_local, const int32_t* idx,
                           const float* logprob, int32_t vocab0, float* out3, void* stream) {
  SG_CHECK_ARG(logits && idx && logprob && out3 && rows >= 1 && vocab_local >= 1, "sg_tp_argmax_pack: bad argument");
  SG_CUDA_TRY(sgd::launch_pdl(tp_argmax_pack_kernel, dim3(1), dim3(128), 0, static_cast<cudaStream_t>(stream), logits,
                              (int)vocab_local, idx, logprob, (int)vocab0, (int)rows, out3));
  return SG_OK;
}

SgStatus sg_tp_argmax_pick(const float* all3, int32_t world, int32_t rows, int32_t* next, float* logprob,
                           void* stream) {
  SG_CHECK_ARG(all3 && next && world >= 1 && rows >= 1, "sg_tp_argmax_pick: bad argument");
  SG_CUDA_TRY(sgd::launch_pdl(tp_argmax_pick_kernel, dim3(1), dim3(128), 0, static_cast<cudaStream_t>(stream), all3,
                              (int)world, (int)rows, next, logprob));
  return SG_OK;
}

}  // extern "C"
