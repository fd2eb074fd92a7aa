// Transformer block element-wise ops on the GPU, restating the reference's
// fp16 CPU kernels (compiler/kernels/cpu/matmul_neon.h):
//   rmsnorm   :154-190  y = x * (1 / sqrt(mean(x^2) + eps)) * w
//   silu      :196-225  y = x / (1 + exp(-x))            (+ SwiGLU form silu(g) * u)
//   softmax   :230-256  y = exp(x - max) rounded to the I/O type, summed, scaled
//   rope      :262-275  rotate-half pairs (i, i + D/2), theta = pos / base^(2i/D)
// plus the decoder's embedding gather and greedy argmax.  All are HBM-bound:
// 16-byte loads where the row allows, fp32 arithmetic, one rounding to the
// I/O type at the end (the reference's order of operations).
#include <algorithm>
#include <cfloat>

#include "rownorm.cuh"
#include "sm100.cuh"

namespace {

using sgd::load_as_float;
using sgd::store_from_float;

constexpr int kRowThreads = sgn::kNormThreads;

__device__ __forceinline__ float ld(const void* p, int dt, int64_t i) {
  switch (dt) {
    case SG_DT_F32: return load_as_float<SG_DT_F32>(p, i);
    case SG_DT_BF16: return load_as_float<SG_DT_BF16>(p, i);
    default: return load_as_float<SG_DT_F16>(p, i);
  }
}
__device__ __forceinline__ void st(void* p, int dt, int64_t i, float v) {
  switch (dt) {
    case SG_DT_F32: store_from_float<SG_DT_F32>(p, i, v); break;
    case SG_DT_BF16: store_from_float<SG_DT_BF16>(p, i, v); break;
    default: store_from_float<SG_DT_F16>(p, i, v); break;
  }
}
// value rounded to the I/O type and back (the reference sums rounded values)
__device__ __forceinline__ float round_io(float v, int dt) {
  switch (dt) {
    case SG_DT_F32: return v;
    case SG_DT_BF16: return __bfloat162float(__float2bfloat16_rn(v));
    default: return __half2float(__float2half_rn(v));
  }
}

using sgn::block_sum;

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : -FLT_MAX;
#pragma unroll
  for (int o = 16; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}

// One CTA per row.  With a residual: h = x + residual is written back to the
// residual (I/O type) and normalised; without: h = x.
__global__ void __launch_bounds__(kRowThreads) rmsnorm_kernel(const void* x, void* residual, const void* w, void* y,
                                                              int n, float eps, int dt) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  __shared__ float red[32];
  const int64_t base = (int64_t)blockIdx.x * n;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float h = ld(x, dt, base + i);
    if (residual) {
      h = round_io(h + ld(residual, dt, base + i), dt);  // the residual stream keeps the I/O type
      st(residual, dt, base + i, h);
    }
    ss += h * h;
  }
  ss = block_sum(ss, red);
  const float rms_inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float h = residual ? ld(residual, dt, base + i) : ld(x, dt, base + i);
    st(y, dt, base + i, h * rms_inv * ld(w, dt, i));
  }
}

// Same operation for 16-bit rows with n % 8 == 0 and n <= 8 * kRowThreads * kVecPerThread:
// the row stays in registers between the sum of squares and the scaling,
// loaded and stored 8 values (16 bytes) at a time.
// The sum of squares is formed as in sgn::row_rms_inv (rownorm.cuh), which the
// INT4 GEMV uses when it fuses this norm into its activation staging.
constexpr int kVecPerThread = sgn::kNormVecPerThread;
using sgn::pack8;
using sgn::unpack8;

template <typename T>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_vec_kernel(const T* __restrict__ x, T* __restrict__ residual,
                                                                  const T* __restrict__ w, T* __restrict__ y, int n,
                                                                  float eps) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  __shared__ float red[32];
  const int64_t base = (int64_t)blockIdx.x * n;
  const int nv = n / 8;
  float h[kVecPerThread][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k) {
    const int v = threadIdx.x + k * kRowThreads;
    if (v < nv) {
      unpack8<T>(reinterpret_cast<const uint4*>(x + base)[v], h[k]);
      if (residual) {
        float r[8];
        unpack8<T>(reinterpret_cast<const uint4*>(residual + base)[v], r);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[k][e] = (float)(T)(h[k][e] + r[e]);  // the residual stream keeps T
        reinterpret_cast<uint4*>(residual + base)[v] = pack8<T>(h[k]);
      }
      ss = sgn::sumsq8(h[k], ss);
    }
  }
  ss = block_sum(ss, red);
  const float rms_inv = 1.0f / sqrtf(ss / (float)n + eps);
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k) {
    const int v = threadIdx.x + k * kRowThreads;
    if (v < nv) {
      float wf[8], o[8];
      unpack8<T>(reinterpret_cast<const uint4*>(w)[v], wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = h[k][e] * rms_inv * wf[e];
      reinterpret_cast<uint4*>(y + base)[v] = pack8<T>(o);
    }
  }
}

// y = silu(g) (* u when u != NULL)
__global__ void silu_kernel(const void* g, const void* u, void* y, int64_t n, int dt) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float xi = ld(g, dt, i);
    float v = xi / (1.0f + expf(-xi));
    if (u) v = round_io(v, dt) * ld(u, dt, i);  // silu output rounded as the reference's silu writes it
    st(y, dt, i, v);
  }
}

// One CTA per row (reference order: max; y = round(exp(x - max)); sum of the
// rounded values; y = round(y * (1 / sum))).
__global__ void __launch_bounds__(kRowThreads) softmax_kernel(const void* x, void* y, int n, int dt) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  __shared__ float red[32];
  const int64_t base = (int64_t)blockIdx.x * n;
  float mx = -FLT_MAX;
  for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, ld(x, dt, base + i));
  mx = block_max(mx, red);
  float sum = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float e = round_io(expf(ld(x, dt, base + i) - mx), dt);
    st(y, dt, base + i, e);
    sum += e;
  }
  sum = block_sum(sum, red);
  const float inv = 1.0f / sum;
  for (int i = threadIdx.x; i < n; i += blockDim.x) st(y, dt, base + i, ld(y, dt, base + i) * inv);
}

// In place on x [tokens, heads, D]: token t is at position pos[t] (or pos0 + t).
__global__ void rope_kernel(void* x, int tokens, int heads, int D, const int32_t* pos, int pos0, float base, int dt) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  const int half = D / 2;
  const int64_t total = (int64_t)tokens * heads * half;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(e % half);
    const int64_t th = e / half;  // token * heads + head
    const int t = (int)(th / heads);
    const int p = pos ? pos[t] : pos0 + t;
    const int64_t r = th * D;
    const float x0 = ld(x, dt, r + i), x1 = ld(x, dt, r + i + half);
    float y0, y1;
    sgd::rope_pair(x0, x1, p, i, D, base, &y0, &y1);
    st(x, dt, r + i, y0);
    st(x, dt, r + i + half, y1);
  }
}

// out[t, :] = table[ids[t], :]; ids outside [0, vocab) give zeros and the error word.
__global__ void embedding_kernel(const void* table, const int32_t* ids, void* out, int tokens, int hidden, int vocab,
                                 int esz, int* bad) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  const int t = blockIdx.y;
  if (t >= tokens) return;
  const int id = ids[t];
  const int64_t row_bytes = (int64_t)hidden * esz;
  unsigned char* dst = static_cast<unsigned char*>(out) + t * row_bytes;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && bad) atomicCAS(bad, 0, 1);
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < row_bytes; b += (int64_t)gridDim.x * blockDim.x)
      dst[b] = 0;
    return;
  }
  const unsigned char* src = static_cast<const unsigned char*>(table) + (int64_t)id * row_bytes;
  if (row_bytes % 16 == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0) {
    for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 16; b < row_bytes;
         b += (int64_t)gridDim.x * blockDim.x * 16)
      *reinterpret_cast<uint4*>(dst + b) = *reinterpret_cast<const uint4*>(src + b);
  } else {
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < row_bytes; b += (int64_t)gridDim.x * blockDim.x)
      dst[b] = src[b];
  }
}

// Greedy argmax per row of fp32 logits (first index among equal maxima; NaN never wins).
__global__ void __launch_bounds__(kRowThreads) argmax_kernel(const float* logits, int n, int32_t* out) {
  sgd::pdl_wait();  // inputs come from the previous kernel on the stream
  sgd::pdl_launch_dependents();
  __shared__ float sv[32];
  __shared__ int si[32];
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
#pragma unroll
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
  if (w == 0) {
    best = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

int grid_for(int64_t n, int threads) {
  const int64_t b = (n + threads - 1) / threads;
  return (int)(b < 148 * 32 ? (b < 1 ? 1 : b) : 148 * 32);
}

SgStatus check_dt(const char* name, int32_t dt) {
  const int d = dt == SG_DT_DEFAULT ? SG_DT_F16 : dt;
  SG_CHECK_ARG(d == SG_DT_F16 || d == SG_DT_BF16 || d == SG_DT_F32, "%s: io_dtype %d unsupported", name, dt);
  return SG_OK;
}

}  // namespace

extern "C" {

SgStatus sg_rmsnorm(const void* x, void* residual, const void* w, void* y, int32_t rows, int32_t n, float eps,
                    int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(rows >= 0 && n >= 0, "sg_rmsnorm: negative size");
  if (rows == 0 || n == 0) return SG_OK;
  SG_CHECK_ARG(x && w && y, "sg_rmsnorm: x, w and y must be non-NULL");
  SgStatus s = check_dt("sg_rmsnorm", io_dtype);
  if (s != SG_OK) return s;
  const int dt = io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : io_dtype;
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const bool vec = dt != SG_DT_F32 && n % 8 == 0 && n <= 8 * kRowThreads * kVecPerThread && sg::aligned16(x) &&
                   sg::aligned16(w) && sg::aligned16(y) && (residual == nullptr || sg::aligned16(residual));
  if (vec && dt == SG_DT_F16)
    SG_CUDA_TRY(sgd::launch_pdl(rmsnorm_vec_kernel<__half>, dim3(rows), dim3(kRowThreads), 0, cs,
                                static_cast<const __half*>(x), static_cast<__half*>(residual),
                                static_cast<const __half*>(w), static_cast<__half*>(y), n, eps));
  else if (vec)
    SG_CUDA_TRY(sgd::launch_pdl(rmsnorm_vec_kernel<__nv_bfloat16>, dim3(rows), dim3(kRowThreads), 0, cs,
                                static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(residual),
                                static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y), n, eps));
  else
    rmsnorm_kernel<<<rows, kRowThreads, 0, cs>>>(x, residual, w, y, n, eps, dt);
  return sg::check_launch("sg_rmsnorm");
}

SgStatus sg_silu(const void* x, void* y, int64_t n, int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(n >= 0, "sg_silu: negative size");
  if (n == 0) return SG_OK;
  SG_CHECK_ARG(x && y, "sg_silu: x and y must be non-NULL");
  SgStatus s = check_dt("sg_silu", io_dtype);
  if (s != SG_OK) return s;
  const int dt = io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : io_dtype;
  silu_kernel<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, nullptr, y, n, dt);
  return sg::check_launch("sg_silu");
}

SgStatus sg_silu_mul(const void* gate, const void* up, void* y, int64_t n, int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(n >= 0, "sg_silu_mul: negative size");
  if (n == 0) return SG_OK;
  SG_CHECK_ARG(gate && up && y, "sg_silu_mul: gate, up and y must be non-NULL");
  SgStatus s = check_dt("sg_silu_mul", io_dtype);
  if (s != SG_OK) return s;
  const int dt = io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : io_dtype;
  silu_kernel<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(gate, up, y, n, dt);
  return sg::check_launch("sg_silu_mul");
}

SgStatus sg_softmax(const void* x, void* y, int32_t rows, int32_t n, int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(rows >= 0 && n >= 0, "sg_softmax: negative size");
  if (rows == 0 || n == 0) return SG_OK;
  SG_CHECK_ARG(x && y, "sg_softmax: x and y must be non-NULL");
  SgStatus s = check_dt("sg_softmax", io_dtype);
  if (s != SG_OK) return s;
  const int dt = io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : io_dtype;
  softmax_kernel<<<rows, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n, dt);
  return sg::check_launch("sg_softmax");
}

SgStatus sg_rope(void* x, int32_t tokens, int32_t heads, int32_t head_dim, const int32_t* positions, int32_t pos0,
                 float base, int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(tokens >= 0 && heads >= 0 && head_dim >= 0, "sg_rope: negative size");
  if (tokens == 0 || heads == 0 || head_dim == 0) return SG_OK;
  SG_CHECK_ARG(x != nullptr, "sg_rope: x is NULL");
  SG_CHECK_ARG(head_dim % 2 == 0, "sg_rope: head_dim %d is odd", head_dim);
  SG_CHECK_ARG(base > 0.f, "sg_rope: base must be positive");
  SgStatus s = check_dt("sg_rope", io_dtype);
  if (s != SG_OK) return s;
  const int dt = io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : io_dtype;
  const int64_t total = (int64_t)tokens * heads * (head_dim / 2);
  rope_kernel<<<grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, tokens, heads, head_dim,
                                                                                  positions, pos0, base, dt);
  return sg::check_launch("sg_rope");
}

SgStatus sg_embedding(const void* table, const int32_t* ids, void* out, int32_t tokens, int32_t hidden, int32_t vocab,
                      int32_t io_dtype, void* stream) {
  SG_CHECK_ARG(tokens >= 0 && hidden >= 0 && vocab >= 0, "sg_embedding: negative size");
  if (tokens == 0 || hidden == 0) return SG_OK;
  SG_CHECK_ARG(table && ids && out, "sg_embedding: table, ids and out must be non-NULL");
  SG_CHECK_ARG(tokens <= 65535, "sg_embedding: at most 65535 tokens per call");
  SgStatus s = check_dt("sg_embedding", io_dtype);
  if (s != SG_OK) return s;
  const int dt = io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : io_dtype;
  int* err = nullptr;
  s = sg::device_error_word(&err);
  if (s != SG_OK) return s;
  const int64_t row_bytes = (int64_t)hidden * sg::elem_size(dt);
  const dim3 grid((unsigned)std::max<int64_t>(1, std::min<int64_t>(8, (row_bytes / 16 + 255) / 256)), tokens);
  SG_CUDA_TRY(sgd::launch_pdl(embedding_kernel, grid, dim3(256), 0, static_cast<cudaStream_t>(stream), table, ids,
                              out, tokens, hidden, vocab, (int)sg::elem_size(dt), err));
  return sg::check_launch("sg_embedding");
}

SgStatus sg_argmax(const float* logits, int32_t rows, int32_t n, int32_t* out, void* stream) {
  SG_CHECK_ARG(rows >= 0 && n >= 1, "sg_argmax: bad size");
  if (rows == 0) return SG_OK;
  SG_CHECK_ARG(logits && out, "sg_argmax: logits and out must be non-NULL");
  argmax_kernel<<<rows, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(logits, n, out);
  return sg::check_launch("sg_argmax");
}

}  // extern "C"
