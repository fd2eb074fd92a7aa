// Causal flash attention on CUDA cores, and its split-K decode form (sm_100a).
//
// Replaces flash_attention_fp16 / flash_attn_head
// (compiler/kernels/cpu/flash_attention.h:49-144): layout [B, heads, S, D],
// scale = p.scale > 0 ? p.scale : 1/sqrt(D) (:101), GQA kv_head = h / (H / Hkv)
// (:102,113), causal: key j visible to the query at position p iff j <= p
// (:60), online softmax with running max and normaliser (:55-89).
//
// Work item = (batch, kv head, block of query positions, key split).  The
// query heads that share a kv head (GQA group) are processed together, so a
// K/V tile is read from HBM once per group.  Tiles of 64 keys are staged in
// shared memory as fp32; each warp owns a few (head, position) rows, lanes
// split the head dimension, scores come from a warp reduction.
//   * one split: the normalised output is written directly;
//   * several splits (decode): each writes (m, l, unnormalised o) to scratch
//     and a combine kernel merges the splits in fixed order (deterministic).
// Used for decode (few queries, long KV) and for shapes outside the tensor-core
// prefill kernel.
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <string_view>

#include "sm100.cuh"

namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kKeyTile = 64;
constexpr int kMaxRowsPerWarp = 8;
constexpr int kMaxD = 256;

struct AArgs {
  const void* Q;
  const void* K;
  const void* V;
  void* O;
  int B, H, Hkv, Sq, Skv, D, G;  // G = query heads per kv head
  float scale;
  int causal, q_pos0;
  int64_t kv_bs, kv_hs;         // element strides of K/V (batch, kv head); row stride = D
  int io_dt;
  int qb;                       // query positions per work item
  int nsplit, keys_per_split;
  float* part;                  // [B][H][Sq][nsplit][D + 2]  (o..., m, l)
  const int32_t* q_pos_dev;     // device position of query 0 (Skv is then the capacity)
  // paged KV cache (pt != NULL): key j of sequence b lives in physical page
  // pt[b * pt_bs + (j / 16) * pt_ps] of the pool, row j % 16
  const int32_t* pt;
  int64_t pt_bs, pt_ps, page_stride;
  int npages;
  int* err;                     // device error word (a page id outside the pool)
};

// Element offset of (sequence b, kv head hk, key) in K and in V: the flat
// [B][Hkv][S][D] layout with the caller's strides, or row key % 16 of the
// page that holds it, [page][kv_head][16][D] within the pool (the reference's
// page layout, kv_cache_layout.cpp:65-102).  A page id outside the pool reads
// page 0 instead and sets bit 4 of the device error word.
__device__ __forceinline__ int kv_page(const AArgs& a, int b, int key) {
  int page = __ldg(a.pt + (int64_t)b * a.pt_bs + (int64_t)(key >> 4) * a.pt_ps);
  if ((unsigned)page >= (unsigned)a.npages) {
    if (a.err) atomicOr(a.err, 4);
    page = 0;
  }
  return page;
}

__device__ __forceinline__ int64_t kv_off(const AArgs& a, int b, int hk, int key) {
  if (!a.pt) return (int64_t)b * a.kv_bs + (int64_t)hk * a.kv_hs + (int64_t)key * a.D;
  return (int64_t)kv_page(a, b, key) * a.page_stride + ((int64_t)hk * 16 + (key & 15)) * a.D;
}

__device__ __forceinline__ float ld_io(const void* p, int dt, int64_t i) {
  switch (dt) {
    case SG_DT_F32: return static_cast<const float*>(p)[i];
    case SG_DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default: return __half2float(static_cast<const __half*>(p)[i]);
  }
}

__device__ __forceinline__ void st_io(void* p, int dt, int64_t i, float v) {
  switch (dt) {
    case SG_DT_F32: static_cast<float*>(p)[i] = v; break;
    case SG_DT_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    default: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
  }
}

// Keys per split.  With the position in device memory (a captured decode step
// launched for the cache's capacity) the live keys are spread evenly over the
// splits in whole 64-key tiles, so every split works whatever the position;
// otherwise the host's split.
__device__ __forceinline__ int split_keys(const AArgs& a, int q_pos0, int Skv) {
  if (!a.q_pos_dev) return a.keys_per_split;
  const int live = a.causal ? min(Skv, q_pos0 + a.Sq) : Skv;
  const int per = (live + a.nsplit - 1) / a.nsplit;
  return max(64, (per + 63) / 64 * 64);
}

template <int DPL>  // head-dim elements per lane (D <= 32 * DPL)
__global__ void __launch_bounds__(kThreads) attn_cc_kernel(AArgs a) {
  extern __shared__ float sm[];
  float* ks = sm;                         // [kKeyTile][D]
  float* vs = sm + kKeyTile * a.D;        // [kKeyTile][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, hk = blockIdx.y;
  const int nqb = (a.Sq + a.qb - 1) / a.qb;
  const int qblk = blockIdx.x % nqb, split = blockIdx.x / nqb;
  const int q0 = qblk * a.qb;
  const int nq = min(a.qb, a.Sq - q0);
  const int rows = a.G * nq;  // row r: head hk*G + r / nq, position q0 + r % nq

  // positions from the device (a captured decode step) or from the launch
  const int q_pos0 = a.q_pos_dev ? *a.q_pos_dev : a.q_pos0;
  const int Skv = a.q_pos_dev ? min(a.Skv, q_pos0 + a.Sq) : a.Skv;
  // key range of this split, clipped to what the causal mask lets any row see
  const int kps = split_keys(a, q_pos0, Skv);
  int j0 = split * kps;
  int j1 = min(Skv, j0 + kps);
  if (a.causal) j1 = min(j1, q_pos0 + q0 + nq);  // last visible key + 1

  float q[kMaxRowsPerWarp][DPL], o[kMaxRowsPerWarp][DPL], m[kMaxRowsPerWarp], l[kMaxRowsPerWarp];
  int pos[kMaxRowsPerWarp];
  bool live[kMaxRowsPerWarp];
#pragma unroll
  for (int rr = 0; rr < kMaxRowsPerWarp; ++rr) {
    const int r = warp + rr * kWarps;
    m[rr] = -INFINITY;
    l[rr] = 0.f;
    pos[rr] = 0;
    live[rr] = r < rows;
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
      q[rr][e] = 0.f;
      o[rr][e] = 0.f;
    }
    if (r < rows) {
      const int h = hk * a.G + r / nq, qi = q0 + r % nq;
      pos[rr] = q_pos0 + qi;
      const int64_t qoff = (((int64_t)b * a.H + h) * a.Sq + qi) * a.D;
#pragma unroll
      for (int e = 0; e < DPL; ++e) {
        const int d = lane + 32 * e;
        if (d < a.D) q[rr][e] = ld_io(a.Q, a.io_dt, qoff + d);
      }
    }
  }

  for (int jt = j0; jt < j1; jt += kKeyTile) {
    const int nk = min(kKeyTile, j1 - jt);
    __syncthreads();
    for (int i = threadIdx.x; i < nk * a.D; i += kThreads) {
      const int64_t off = kv_off(a, b, hk, jt + i / a.D) + (i % a.D);
      ks[i] = ld_io(a.K, a.io_dt, off);
      vs[i] = ld_io(a.V, a.io_dt, off);
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < kMaxRowsPerWarp; ++rr) {
      if (!live[rr]) continue;  // warp-uniform
      const int jmax = a.causal ? min(nk, pos[rr] - jt + 1) : nk;
      for (int jj = 0; jj < jmax; ++jj) {
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
          const int d = lane + 32 * e;
          if (d < a.D) s = fmaf(q[rr][e], ks[jj * a.D + d], s);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        s *= a.scale;
        const float m_new = fmaxf(m[rr], s);
        const float e_s = expf(s - m_new);
        const float c_old = expf(m[rr] - m_new);
        l[rr] = l[rr] * c_old + e_s;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
          const int d = lane + 32 * e;
          if (d < a.D) o[rr][e] = fmaf(o[rr][e], c_old, e_s * vs[jj * a.D + d]);
        }
        m[rr] = m_new;
      }
    }
  }

#pragma unroll
  for (int rr = 0; rr < kMaxRowsPerWarp; ++rr) {
    if (!live[rr]) continue;
    const int r = warp + rr * kWarps;
    const int h = hk * a.G + r / nq, qi = q0 + r % nq;
    if (a.nsplit == 1) {
      const float inv = l[rr] > 0.f ? 1.0f / l[rr] : 0.f;
      const int64_t ooff = (((int64_t)b * a.H + h) * a.Sq + qi) * a.D;
#pragma unroll
      for (int e = 0; e < DPL; ++e) {
        const int d = lane + 32 * e;
        if (d < a.D) st_io(a.O, a.io_dt, ooff + d, o[rr][e] * inv);
      }
    } else {
      float* pp = a.part + ((((int64_t)b * a.H + h) * a.Sq + qi) * a.nsplit + split) * (a.D + 2);
#pragma unroll
      for (int e = 0; e < DPL; ++e) {
        const int d = lane + 32 * e;
        if (d < a.D) pp[d] = o[rr][e];
      }
      if (lane == 0) {
        pp[a.D] = m[rr];
        pp[a.D + 1] = l[rr];
      }
    }
  }
}

// Decode form: few query rows per kv head (G * Sq <= 32), head_dim 64 or 128.
// Per 64-key tile: scores with one key per thread (K tile padded in shared
// memory, no shuffles per key), online softmax with one warp per row, then
// O += P V with one (row, dim) per thread.  Scores are prescaled by
// scale * log2(e) and use exp2; the partial max is written back in natural
// units for attn_combine_kernel.
constexpr int kDecRows = 32;

template <int D>
__global__ void __launch_bounds__(kThreads) attn_decode_kernel(AArgs a) {
  constexpr int KT = kKeyTile;   // 64 keys per tile
  constexpr int KS = D + 1;      // padded K row
  constexpr int OPT = (kDecRows * D + kThreads - 1) / kThreads;  // outputs per thread (max)
  extern __shared__ float sm[];
  float* qs = sm;                        // [kDecRows][D]  prescaled queries
  float* ks = qs + kDecRows * D;         // [KT][KS]
  float* vs = ks + KT * KS;              // [KT][D]
  float* ps = vs + KT * D;               // [kDecRows][KT] scores / probabilities
  float* ms = ps + kDecRows * KT;        // [kDecRows] running max (log2 units)
  float* ls = ms + kDecRows;             // [kDecRows] running sum
  float* al = ls + kDecRows;             // [kDecRows] rescale of this tile
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.z, hk = blockIdx.y, split = blockIdx.x;
  const int nq = a.Sq, R = a.G * nq;  // row r: head hk*G + r / nq, query r % nq
  const int q_pos0 = a.q_pos_dev ? *a.q_pos_dev : a.q_pos0;
  const int Skv = a.q_pos_dev ? min(a.Skv, q_pos0 + a.Sq) : a.Skv;
  const int kps = split_keys(a, q_pos0, Skv);
  const int j0 = split * kps;
  int j1 = min(Skv, j0 + kps);
  if (a.causal) j1 = min(j1, q_pos0 + nq);
  const float qscale = a.scale * 1.4426950408889634f;
  for (int i = tid; i < R * D; i += kThreads) {
    const int r = i / D, d = i % D;
    const int h = hk * a.G + r / nq, qi = r % nq;
    qs[i] = ld_io(a.Q, a.io_dt, (((int64_t)b * a.H + h) * a.Sq + qi) * D + d) * qscale;
  }
  for (int r = tid; r < kDecRows; r += kThreads) {
    ms[r] = -INFINITY;
    ls[r] = 0.f;
  }
  float o[OPT];
#pragma unroll
  for (int k = 0; k < OPT; ++k) o[k] = 0.f;
  for (int jt = j0; jt < j1; jt += KT) {
    const int nk = min(KT, j1 - jt);
    __syncthreads();  // previous tile's readers are done
    for (int i = tid; i < KT * D; i += kThreads) {
      const int j = i / D, d = i % D;
      float kv = 0.f, vv = 0.f;
      if (j < nk) {
        const int64_t off = kv_off(a, b, hk, jt + j) + d;
        kv = ld_io(a.K, a.io_dt, off);
        vv = ld_io(a.V, a.io_dt, off);
      }
      ks[j * KS + d] = kv;
      vs[j * D + d] = vv;
    }
    __syncthreads();
    // scores: thread -> key j = tid % KT, rows tid / KT, + kThreads / KT, ...
    {
      const int j = tid % KT;
      for (int r = tid / KT; r < R; r += kThreads / KT) {
        float sdot = 0.f;
#pragma unroll 8
        for (int d = 0; d < D; ++d) sdot = fmaf(qs[r * D + d], ks[j * KS + d], sdot);
        const int key = jt + j;
        const bool vis = j < nk && (!a.causal || key <= q_pos0 + r % nq);
        ps[r * KT + j] = vis ? sdot : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax: one warp per row
    for (int r = warp; r < R; r += kThreads / 32) {
      const float s0 = ps[r * KT + lane], s1 = ps[r * KT + lane + 32];
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = ms[r];
      const float m_new = fmaxf(m_old, mx);
      const float p0 = m_new == -INFINITY ? 0.f : exp2f(s0 - m_new);
      const float p1 = m_new == -INFINITY ? 0.f : exp2f(s1 - m_new);
      ps[r * KT + lane] = p0;
      ps[r * KT + lane + 32] = p1;
      float sum = p0 + p1;
#pragma unroll
      for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      const float alpha = m_old == -INFINITY ? 0.f : exp2f(m_old - m_new);
      __syncwarp();
      if (lane == 0) {
        ms[r] = m_new;
        ls[r] = ls[r] * alpha + sum;
        al[r] = alpha;
      }
    }
    __syncthreads();
    // O += P V: thread -> outputs i = tid + k * kThreads (row i / D, dim i % D)
#pragma unroll
    for (int k = 0; k < OPT; ++k) {
      const int i = tid + k * kThreads;
      if (i < R * D) {
        const int r = i / D, d = i % D;
        float acc = o[k] * al[r];
#pragma unroll 8
        for (int j = 0; j < KT; ++j) acc = fmaf(ps[r * KT + j], vs[j * D + d], acc);
        o[k] = acc;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < OPT; ++k) {
    const int i = tid + k * kThreads;
    if (i >= R * D) continue;
    const int r = i / D, d = i % D;
    const int h = hk * a.G + r / nq, qi = r % nq;
    if (a.nsplit == 1) {
      const float inv = ls[r] > 0.f ? 1.0f / ls[r] : 0.f;
      st_io(a.O, a.io_dt, (((int64_t)b * a.H + h) * a.Sq + qi) * D + d, o[k] * inv);
    } else {
      float* pp = a.part + ((((int64_t)b * a.H + h) * a.Sq + qi) * a.nsplit + split) * (D + 2);
      pp[d] = o[k];
      if (d == 0) {
        pp[D] = ms[r] == -INFINITY ? -INFINITY : ms[r] * 0.6931471805599453f;  // back to natural units
        pp[D + 1] = ls[r];
      }
    }
  }
}

template <int D>
constexpr size_t decode_smem() {
  return sizeof(float) * ((size_t)kDecRows * D + kKeyTile * (D + 1) + kKeyTile * D + kDecRows * kKeyTile +
                          3 * kDecRows);
}

// Merge the splits of one (batch, head, query) row: fixed split order.
__global__ void attn_combine_kernel(AArgs a) {
  const int row = blockIdx.x;  // (b * H + h) * Sq + qi
  const float* pp = a.part + (int64_t)row * a.nsplit * (a.D + 2);
  float M = -INFINITY;
  for (int sp = 0; sp < a.nsplit; ++sp) M = fmaxf(M, pp[sp * (a.D + 2) + a.D]);
  float L = 0.f;
  for (int sp = 0; sp < a.nsplit; ++sp) {
    const float ms = pp[sp * (a.D + 2) + a.D];
    if (ms != -INFINITY) L += pp[sp * (a.D + 2) + a.D + 1] * expf(ms - M);
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
    float acc = 0.f;
    for (int sp = 0; sp < a.nsplit; ++sp) {
      const float ms = pp[sp * (a.D + 2) + a.D];
      if (ms != -INFINITY) acc += pp[sp * (a.D + 2) + d] * expf(ms - M);
    }
    st_io(a.O, a.io_dt, (int64_t)row * a.D + d, acc * inv);
  }
}

// Decode form: few query rows per kv head (R = G * Sq <= 32), head_dim 64 or
// 128.  The key splits of one (batch, kv head) form one thread-block cluster.
// Each block streams its 64-key tiles with 16-byte loads straight into
// registers, one tile ahead: thread t holds half of key t / 2 (K and V).
// Scores come from the K registers (queries prescaled by scale * log2(e),
// shared memory, broadcast reads), the online softmax runs one warp per row,
// and O += P V reads V from shared memory as fp32.  At the end every block
// stores its (max, sum, unnormalised O) into rank 0's shared memory and rank
// 0 merges the splits in rank order (deterministic) and writes O: no global
// scratch and no second kernel.
constexpr int kDecClusterMax = 16;
constexpr int kDecTile = 64;

template <int IO>
struct IoVec;
template <>
struct IoVec<SG_DT_F16> {
  static constexpr int kBytes = 2;
  __device__ static void to_f32(const uint4& v, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __half22float2(h[i]);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
};
template <>
struct IoVec<SG_DT_BF16> {
  static constexpr int kBytes = 2;
  __device__ static void to_f32(const uint4& v, float* f) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __bfloat1622float2(h[i]);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
};
template <>
struct IoVec<SG_DT_F32> {
  static constexpr int kBytes = 4;
  __device__ static void to_f32(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
};

// shared memory of attn_dec_cluster_kernel<D> for R rows and nsplit ranks (floats)
inline size_t dec_cluster_smem(int D, int R, int nsplit) {
  return sizeof(float) * ((size_t)2 * R * (D / 2) + 4 + (size_t)R * kDecTile + (size_t)kDecTile * D + 3 * R +
                          (size_t)nsplit * R * (D + 2));
}

template <int D, int IO>
__global__ void __launch_bounds__(kThreads) attn_dec_cluster_kernel(AArgs a) {
  namespace cg = cooperative_groups;
  constexpr int KT = kDecTile, DH = D / 2;
  constexpr int EPV = 16 / IoVec<IO>::kBytes;  // elements per 16-byte load
  constexpr int NV = DH / EPV;                 // 16-byte loads per thread per tile (K, and V)
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.z, hk = blockIdx.y, split = blockIdx.x;
  const int nq = a.Sq, R = a.G * nq;  // row r: head hk*G + r / nq, query r % nq
  float* qs = sm;                        // [part][R][DH], part 1 offset by 4 floats (banks)
  float* ps = qs + 2 * R * DH + 4;       // [R][KT] scores, then probabilities
  float* vsf = ps + R * KT;              // [KT][D] V tile
  float* ms = vsf + KT * D;              // [R] running max (log2 units)
  float* ls = ms + R;                    // [R] running sum
  float* al = ls + R;                    // [R] rescale of this tile
  float* comb = al + R;                  // rank 0: [rank][R][D + 2]
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  sgd::pdl_wait();  // the newest key and the queries come from the previous kernel
  sgd::pdl_launch_dependents();

  const int q_pos0 = a.q_pos_dev ? *a.q_pos_dev : a.q_pos0;
  const int Skv = a.q_pos_dev ? min(a.Skv, q_pos0 + a.Sq) : a.Skv;
  const int kps = split_keys(a, q_pos0, Skv);
  const int j0 = split * kps;
  int j1 = min(Skv, j0 + kps);
  if (a.causal) j1 = min(j1, q_pos0 + nq);
  const float qscale = a.scale * 1.4426950408889634f;
  const int kk = tid >> 1, part = tid & 1;
  float* qpart = qs + part * (R * DH + 4);
  for (int r = tid; r < R; r += kThreads) {
    ms[r] = -INFINITY;
    ls[r] = 0.f;
  }
  constexpr int kUnits = (kDecRows * D / 4 + kThreads - 1) / kThreads;  // float4 outputs per thread (max)
  float4 o[kUnits];
#pragma unroll
  for (int k = 0; k < kUnits; ++k) o[k] = make_float4(0.f, 0.f, 0.f, 0.f);

  uint4 kr[NV], vr[NV];
  auto load_tile = [&](int jt) {
    const int key = jt + kk;
    const bool live = key < j1;
    const int64_t e0 = kv_off(a, b, hk, live ? key : j0) + part * DH;
    const uint4* kp = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.K) + e0 * IoVec<IO>::kBytes);
    const uint4* vp = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.V) + e0 * IoVec<IO>::kBytes);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      kr[i] = live ? __ldg(kp + i) : make_uint4(0u, 0u, 0u, 0u);
      vr[i] = live ? __ldg(vp + i) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  if (j0 < j1) load_tile(j0);  // in flight together with the query loads
  for (int i = tid; i < R * D; i += kThreads) {
    const int r = i / D, d = i % D;
    const int h = hk * a.G + r / nq, qi = r % nq;
    const float v = ld_io(a.Q, a.io_dt, (((int64_t)b * a.H + h) * a.Sq + qi) * D + d) * qscale;
    qs[(d / DH) * (R * DH + 4) + r * DH + (d % DH)] = v;
  }
  __syncthreads();
  for (int jt = j0; jt < j1; jt += KT) {
    // V tile into shared memory; scores of this thread's key half for every row
    float kf[DH];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float vf[EPV];
      IoVec<IO>::to_f32(vr[i], vf);
#pragma unroll
      for (int e = 0; e < EPV; e += 4)
        *reinterpret_cast<float4*>(vsf + kk * D + part * DH + i * EPV + e) =
            make_float4(vf[e], vf[e + 1], vf[e + 2], vf[e + 3]);
      IoVec<IO>::to_f32(kr[i], kf + i * EPV);
    }
    const int key = jt + kk;
    const bool vis_key = key < j1;
    for (int r = 0; r < R; ++r) {
      const float* qr = qpart + r * DH;
      float sdot = 0.f;
#pragma unroll
      for (int d = 0; d < DH; d += 4) {
        const float4 q4 = *reinterpret_cast<const float4*>(qr + d);
        sdot = fmaf(q4.x, kf[d], sdot);
        sdot = fmaf(q4.y, kf[d + 1], sdot);
        sdot = fmaf(q4.z, kf[d + 2], sdot);
        sdot = fmaf(q4.w, kf[d + 3], sdot);
      }
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
      const bool vis = vis_key && (!a.causal || key <= q_pos0 + r % nq);
      if (part == 0) ps[r * KT + kk] = vis ? sdot : -INFINITY;
    }
    if (jt + KT < j1) load_tile(jt + KT);  // next tile in flight during this one's softmax and P V
    __syncthreads();
    // online softmax: one warp per row
    for (int r = warp; r < R; r += kThreads / 32) {
      const float s0 = ps[r * KT + lane], s1 = ps[r * KT + lane + 32];
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = ms[r];
      const float m_new = fmaxf(m_old, mx);
      const float p0 = m_new == -INFINITY ? 0.f : exp2f(s0 - m_new);
      const float p1 = m_new == -INFINITY ? 0.f : exp2f(s1 - m_new);
      ps[r * KT + lane] = p0;
      ps[r * KT + lane + 32] = p1;
      float sum = p0 + p1;
#pragma unroll
      for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      const float alpha = m_old == -INFINITY ? 0.f : exp2f(m_old - m_new);
      __syncwarp();
      if (lane == 0) {
        ms[r] = m_new;
        ls[r] = ls[r] * alpha + sum;
        al[r] = alpha;
      }
    }
    __syncthreads();
    // O += P V: thread -> float4 units u = tid + k * kThreads (row u / (D/4), dims 4 (u % (D/4)))
#pragma unroll
    for (int k = 0; k < kUnits; ++k) {
      const int u = tid + k * kThreads;
      if (u < R * (D / 4)) {
        const int r = u / (D / 4), d = 4 * (u % (D / 4));
        const float alr = al[r];
        float4 acc = make_float4(o[k].x * alr, o[k].y * alr, o[k].z * alr, o[k].w * alr);
#pragma unroll 8
        for (int j = 0; j < KT; ++j) {
          const float p = ps[r * KT + j];
          const float4 v = *reinterpret_cast<const float4*>(vsf + j * D + d);
          acc.x = fmaf(p, v.x, acc.x);
          acc.y = fmaf(p, v.y, acc.y);
          acc.z = fmaf(p, v.z, acc.z);
          acc.w = fmaf(p, v.w, acc.w);
        }
        o[k] = acc;
      }
    }
    __syncthreads();  // ps, vsf and al are rewritten by the next tile
  }

  // ---- merge the splits in rank 0 (cluster rank == split)
  cg::cluster_group cluster = cg::this_cluster();
  const int nsplit = a.nsplit;
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  float* dst = cluster.map_shared_rank(comb, 0) + (size_t)split * R * (D + 2);
#pragma unroll
  for (int k = 0; k < kUnits; ++k) {
    const int u = tid + k * kThreads;
    if (u < R * (D / 4)) {
      const int r = u / (D / 4), d = 4 * (u % (D / 4));
      float* pr = dst + r * (D + 2) + d;
      pr[0] = o[k].x;
      pr[1] = o[k].y;
      pr[2] = o[k].z;
      pr[3] = o[k].w;
    }
  }
  for (int r = tid; r < R; r += kThreads) {
    dst[r * (D + 2) + D] = ms[r];
    dst[r * (D + 2) + D + 1] = ls[r];
  }
  cluster.sync();
  if (split != 0) return;
  for (int i = tid; i < R * D; i += kThreads) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, comb[((size_t)sp * R + r) * (D + 2) + D]);
    float L = 0.f, acc = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float* pr = comb + ((size_t)sp * R + r) * (D + 2);
      if (pr[D] == -INFINITY) continue;
      const float w = exp2f(pr[D] - M);
      L = fmaf(pr[D + 1], w, L);
      acc = fmaf(pr[d], w, acc);
    }
    const int h = hk * a.G + r / nq, qi = r % nq;
    st_io(a.O, a.io_dt, (((int64_t)b * a.H + h) * a.Sq + qi) * D + d, L > 0.f ? acc / L : 0.f);
  }
}

// Decode form on tensor cores: up to 16 query rows per kv head (R = G * Sq),
// head_dim 64 or 128, fp16 or bf16 I/O (bf16 values go to fp16 for the MMAs,
// so that P keeps 11 significant bits).  Same cluster-of-splits structure as
// attn_dec_cluster_kernel; per 64-key tile:
//   * S = Q K^T with mma.sync m16n8k16 (queries = the 16 A rows, kept in
//     registers as fragments; warp w of 8 takes keys 8w .. 8w+7, K row-major in
//     shared memory with 16 bytes of padding per row, so the B fragments are
//     conflict-free 32-bit loads);
//   * online softmax on the scores in shared memory, one warp per row;
//   * O += P V with mma.sync (P rebuilt as fp16 A fragments, V fragments by
//     ldmatrix.trans from row-major V; warp w owns an eighth of the head dims).
// K and V tiles stream through a 3-stage cp.async ring (two tiles in flight
// while one is computed; bf16 tiles are converted to fp16 in place).
constexpr int kDecMmaRows = 16;

__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, const void* smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(sgd::smem_u32(smem_row)));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 8 elements of a 16-byte load as fp16 (bf16 input converted).
template <int IO>
__device__ __forceinline__ uint4 to_f16x8(const uint4& v) {
  if (IO == SG_DT_F16) return v;
  float f[8];
  IoVec<SG_DT_BF16>::to_f32(v, f);
  uint4 o;
  o.x = pack_half2(f[0], f[1]);
  o.y = pack_half2(f[2], f[3]);
  o.z = pack_half2(f[4], f[5]);
  o.w = pack_half2(f[6], f[7]);
  return o;
}

constexpr int kDecMmaStages = 3;     // K/V tiles in flight per block
constexpr int kDecMmaThreads = 256;  // 8 warps: 8 keys each in Q K^T, an eighth of the head dims in P V

inline size_t dec_mma_smem(int D, int R, int nsplit) {
  const size_t kvrow = (size_t)(D + 8) * 2;  // bytes per padded fp16 row
  return kDecMmaStages * 2 * kDecTile * kvrow +
         sizeof(float) * ((size_t)kDecMmaRows * kDecTile + 3 * kDecMmaRows + (size_t)nsplit * R * (D + 2));
}

template <int D, int IO>
__global__ void __launch_bounds__(kDecMmaThreads) attn_dec_mma_kernel(AArgs a) {
  namespace cg = cooperative_groups;
  constexpr int KT = kDecTile, KP = D + 8;  // padded row (halves)
  constexpr int kW = kDecMmaThreads / 32;   // 8 warps
  constexpr int NV = (D / 4) * 2 / 16;      // 16-byte loads per thread per tile (K, and V): a quarter row
  constexpr int DW = D / kW;                // head dims per warp in P V
  constexpr int NT = DW / 8;                // n-tiles per warp in P V
  extern __shared__ __align__(16) uint8_t smb[];
  __half* kvs = reinterpret_cast<__half*>(smb);        // [stage][K | V][KT][KP]
  float* ps = reinterpret_cast<float*>(kvs + kDecMmaStages * 2 * KT * KP);  // [16][KT] scores, probabilities
  float* ms = ps + kDecMmaRows * KT;                   // [16] running max (log2 units)
  float* ls = ms + kDecMmaRows;                        // [16] running sum
  float* al = ls + kDecMmaRows;                        // [16] rescale of this tile
  float* comb = al + kDecMmaRows;                      // rank 0: [rank][R][D + 2]
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  sgd::pdl_wait();  // the newest key and the queries come from the previous kernel
  sgd::pdl_launch_dependents();

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int b = blockIdx.z, hk = blockIdx.y, split = blockIdx.x;
  const int nq = a.Sq, R = a.G * nq;  // row r: head hk*G + r / nq, query r % nq
  const int q_pos0 = a.q_pos_dev ? *a.q_pos_dev : a.q_pos0;
  const int Skv = a.q_pos_dev ? min(a.Skv, q_pos0 + a.Sq) : a.Skv;
  const int kps = split_keys(a, q_pos0, Skv);
  const int j0 = split * kps;
  int j1 = min(Skv, j0 + kps);
  if (a.causal) j1 = min(j1, q_pos0 + nq);
  const int kk = tid >> 2, part = tid & 3;  // loader role: quarter `part` of key kk

  const int ntiles = j1 > j0 ? (j1 - j0 + KT - 1) / KT : 0;
  // this thread's 16-byte pieces of tile `it` into stage it % kDecMmaStages (zeros past the last key)
  auto issue_tile = [&](int it) {
    const int key = j0 + it * KT + kk;
    const bool live = key < j1;
    const int64_t e0 = kv_off(a, b, hk, live ? key : j0) + part * (D / 4);
    const uint16_t* kp = static_cast<const uint16_t*>(a.K) + e0;
    const uint16_t* vp = static_cast<const uint16_t*>(a.V) + e0;
    __half* kd = kvs + (size_t)(it % kDecMmaStages) * 2 * KT * KP + kk * KP + part * (D / 4);
    __half* vd = kd + KT * KP;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      sgd::cp_async_16(kd + 8 * i, kp + 8 * i, live);
      sgd::cp_async_16(vd + 8 * i, vp + 8 * i, live);
    }
  };
  for (int s = 0; s < kDecMmaStages - 1; ++s) {  // in flight together with the query loads
    if (s < ntiles) issue_tile(s);
    sgd::cp_async_commit();
  }

  // Q fragments (A of S = Q K^T), prescaled by scale * log2(e); rows >= R are zero.
  const float qscale = a.scale * 1.4426950408889634f;
  auto q_at = [&](int r, int d) -> float {
    if (r >= R) return 0.f;
    const int h = hk * a.G + r / nq, qi = r % nq;
    return ld_io(a.Q, a.io_dt, (((int64_t)b * a.H + h) * a.Sq + qi) * D + d) * qscale;
  };
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int s = 0; s < D / 16; ++s) {
    const int d0 = 16 * s + 2 * t;
    qf[s][0] = pack_half2(q_at(g, d0), q_at(g, d0 + 1));
    qf[s][1] = pack_half2(q_at(g + 8, d0), q_at(g + 8, d0 + 1));
    qf[s][2] = pack_half2(q_at(g, d0 + 8), q_at(g, d0 + 9));
    qf[s][3] = pack_half2(q_at(g + 8, d0 + 8), q_at(g + 8, d0 + 9));
  }
  for (int r = tid; r < kDecMmaRows; r += kDecMmaThreads) {
    ms[r] = -INFINITY;
    ls[r] = 0.f;
  }
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int q = 0; q < 4; ++q) o[n][q] = 0.f;

  for (int it = 0; it < ntiles; ++it) {
    const int jt = j0 + it * KT;
    sgd::cp_async_wait<kDecMmaStages - 2>();  // this thread's pieces of tile `it` have landed
    __half* ks = kvs + (size_t)(it % kDecMmaStages) * 2 * KT * KP;
    __half* vs = ks + KT * KP;
    if (IO == SG_DT_BF16) {  // this thread's own pieces, bf16 -> fp16 in place
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        uint4* kq = reinterpret_cast<uint4*>(ks + kk * KP + part * (D / 4) + 8 * i);
        uint4* vq = reinterpret_cast<uint4*>(vs + kk * KP + part * (D / 4) + 8 * i);
        *kq = to_f16x8<IO>(*kq);
        *vq = to_f16x8<IO>(*vq);
      }
    }
    __syncthreads();  // every piece of tile `it` is in; tile it - 1's readers are done
    if (it + kDecMmaStages - 1 < ntiles) issue_tile(it + kDecMmaStages - 1);  // into tile it - 1's stage
    sgd::cp_async_commit();
    // ---- S = Q K^T for this warp's 8 keys (one n-tile)
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const __half* krow = ks + (8 * warp + g) * KP + 2 * t;
#pragma unroll
      for (int s = 0; s < D / 16; ++s) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + 16 * s);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + 16 * s + 8);
        sgd::mma_f16_16816(sc, qf[s][0], qf[s][1], qf[s][2], qf[s][3], b0, b1);
      }
    }
    // scores to shared memory with the visibility mask (rows >= R are never read)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int r = g + 8 * (q >> 1);
      const int kl = 8 * warp + 2 * t + (q & 1);
      const int key = jt + kl;
      const bool vis = key < j1 && (!a.causal || key <= q_pos0 + r % nq);
      ps[r * KT + kl] = vis ? sc[q] : -INFINITY;
    }
    __syncthreads();
    // ---- online softmax: one warp per row
    for (int r = warp; r < R; r += kW) {
      const float s0 = ps[r * KT + lane], s1 = ps[r * KT + lane + 32];
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = ms[r];
      const float m_new = fmaxf(m_old, mx);
      const float p0 = m_new == -INFINITY ? 0.f : exp2f(s0 - m_new);
      const float p1 = m_new == -INFINITY ? 0.f : exp2f(s1 - m_new);
      ps[r * KT + lane] = p0;
      ps[r * KT + lane + 32] = p1;
      float sum = p0 + p1;
#pragma unroll
      for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      const float alpha = m_old == -INFINITY ? 0.f : exp2f(m_old - m_new);
      __syncwarp();
      if (lane == 0) {
        ms[r] = m_new;
        ls[r] = ls[r] * alpha + sum;
        al[r] = alpha;
      }
    }
    __syncthreads();
    // ---- O += P V for this warp's dims [DW * warp, DW * (warp + 1))
    const float a_lo = g < R ? al[g] : 0.f, a_hi = g + 8 < R ? al[g + 8] : 0.f;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= a_lo;
      o[n][1] *= a_lo;
      o[n][2] *= a_hi;
      o[n][3] *= a_hi;
    }
    auto p_at = [&](int r, int kl) -> float { return r < R ? ps[r * KT + kl] : 0.f; };
#pragma unroll
    for (int s = 0; s < KT / 16; ++s) {
      const int k0 = 16 * s + 2 * t;
      const uint32_t pa0 = pack_half2(p_at(g, k0), p_at(g, k0 + 1));
      const uint32_t pa1 = pack_half2(p_at(g + 8, k0), p_at(g + 8, k0 + 1));
      const uint32_t pa2 = pack_half2(p_at(g, k0 + 8), p_at(g, k0 + 9));
      const uint32_t pa3 = pack_half2(p_at(g + 8, k0 + 8), p_at(g + 8, k0 + 9));
      // ldmatrix rows: lanes 0-7 keys 16s + lane, lanes 8-15 keys 16s + 8 + (lane - 8)
      const __half* vrow = vs + (16 * s + (lane & 15)) * KP + DW * warp;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        uint32_t b0, b1;
        ldmatrix_x2_trans(b0, b1, vrow + 8 * n);
        sgd::mma_f16_16816(o[n], pa0, pa1, pa2, pa3, b0, b1);
      }
    }
  }
  __syncthreads();

  // ---- merge the splits in rank 0 (cluster rank == split)
  cg::cluster_group cluster = cg::this_cluster();
  const int nsplit = a.nsplit;
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  float* dst = cluster.map_shared_rank(comb, 0) + (size_t)split * R * (D + 2);
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int d = DW * warp + 8 * n + 2 * t;
    if (g < R) {
      dst[g * (D + 2) + d] = o[n][0];
      dst[g * (D + 2) + d + 1] = o[n][1];
    }
    if (g + 8 < R) {
      dst[(g + 8) * (D + 2) + d] = o[n][2];
      dst[(g + 8) * (D + 2) + d + 1] = o[n][3];
    }
  }
  for (int r = tid; r < R; r += kDecMmaThreads) {
    dst[r * (D + 2) + D] = ms[r];
    dst[r * (D + 2) + D + 1] = ls[r];
  }
  cluster.sync();
  if (split != 0) return;
  for (int i = tid; i < R * D; i += kDecMmaThreads) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, comb[((size_t)sp * R + r) * (D + 2) + D]);
    float L = 0.f, acc = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float* pr = comb + ((size_t)sp * R + r) * (D + 2);
      if (pr[D] == -INFINITY) continue;
      const float w = exp2f(pr[D] - M);
      L = fmaf(pr[D + 1], w, L);
      acc = fmaf(pr[d], w, acc);
    }
    const int h = hk * a.G + r / nq, qi = r % nq;
    st_io(a.O, a.io_dt, (((int64_t)b * a.H + h) * a.Sq + qi) * D + d, L > 0.f ? acc / L : 0.f);
  }
}

// ---------------------------------------------------------------------------
// Decode attention with the key range split over the warps (flash-decoding
// inside the block).  One block per (key split, kv head, batch), a cluster of
// the splits as in attn_dec_mma_kernel, but no block barrier per tile:
//   * warp w takes the 16-key groups w, w + 8, w + 16, ... of the block's range
//     and streams each group's K and V rows through its own cp.async ring;
//   * S = Q K^T (mma.sync m16n8k16, two 8-key n-tiles) stays in registers; the
//     warp keeps its own running max, sum and O for the 16 (padded) rows; the
//     score fragment is already the A fragment of O += P V (keys as k), V
//     fragments by ldmatrix.trans;
//   * at the end the 8 warps' (max, sum, O) are merged in shared memory in
//     warp order, and the block's result goes to rank 0 of the cluster, which
//     merges the splits in rank order (as attn_dec_mma_kernel).
constexpr int kDecWarpThreads = 256;
constexpr int kDecWarpGroup = 16;  // keys per warp step

template <int D>
constexpr int dec_warp_stages() { return 2; }  // groups in flight per warp

inline size_t dec_warp_smem(int D, int R, int nsplit) {
  const int st = dec_warp_stages<64>();
  const size_t ring = (size_t)8 * st * 2 * kDecWarpGroup * (D + 8) * 2;  // [warp][stage][K | V][16][D + 8] fp16
  const size_t merge = (size_t)8 * kDecMmaRows * (D + 2) * 4;           // [warp][16][D + 2] fp32
  return std::max(ring, merge) + sizeof(float) * (size_t)nsplit * R * (D + 2);
}

template <int D, int IO>
__global__ void __launch_bounds__(kDecWarpThreads) attn_dec_warp_kernel(AArgs a) {
  namespace cg = cooperative_groups;
  constexpr int KG = kDecWarpGroup, KP = D + 8;  // padded row (halves)
  constexpr int kW = kDecWarpThreads / 32;
  constexpr int ST = dec_warp_stages<D>();
  constexpr int NP = KG * D / 8 / 32;  // 16-byte pieces per lane per group (K, and V)
  constexpr int NT = D / 8;            // n-tiles of O
  extern __shared__ __align__(16) uint8_t smb[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  __half* ring = reinterpret_cast<__half*>(smb) + (size_t)warp * ST * 2 * KG * KP;  // this warp's [stage][K | V][KG][KP]
  const size_t main_bytes = std::max((size_t)kW * ST * 2 * KG * KP * 2, (size_t)kW * kDecMmaRows * (D + 2) * 4);
  float* wm = reinterpret_cast<float*>(smb);                  // after the loop: [warp][16][D + 2]
  float* comb = reinterpret_cast<float*>(smb + main_bytes);  // rank 0: [rank][R][D + 2]
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  const int b = blockIdx.z, hk = blockIdx.y, split = blockIdx.x;
  const int nq = a.Sq, R = a.G * nq;  // row r: head hk*G + r / nq, query r % nq
  const int q_pos0 = a.q_pos_dev ? *a.q_pos_dev : a.q_pos0;
  const int Skv = a.q_pos_dev ? min(a.Skv, q_pos0 + a.Sq) : a.Skv;
  const int kps = split_keys(a, q_pos0, Skv);
  const int j0 = split * kps;
  int j1 = min(Skv, j0 + kps);
  if (a.causal) j1 = min(j1, q_pos0 + nq);
  const int ngroups = j1 > j0 ? (j1 - j0 + KG - 1) / KG : 0;
  const int nmine = ngroups > warp ? (ngroups - warp + kW - 1) / kW : 0;  // groups warp, warp + kW, ...

  // Paged cache: a group of KG = 16 keys starts on a page boundary (splits are
  // whole 64-key tiles), so it is one page; the pages of the warp's first 64
  // groups are looked up once, lane l holding groups l and l + 32.
  int pgs[2] = {0, 0};
  if (a.pt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int gi = lane + 32 * h;
      if (gi < nmine) pgs[h] = kv_page(a, b, j0 + (warp + kW * gi) * KG);
    }
  }
  // lane's pieces of group i (the warp's i-th) into stage i % ST; zeros past the last key
  auto issue = [&](int i) {  // called by the whole warp with the same i
    const int key0 = j0 + (warp + kW * i) * KG;
    int64_t gbase;  // element offset of the group's first key
    if (a.pt) {
      const int pg = i < 64 ? __shfl_sync(0xffffffffu, pgs[i >> 5], i & 31) : kv_page(a, b, key0);
      gbase = (int64_t)pg * a.page_stride + (int64_t)hk * KG * D;
    } else {
      gbase = (int64_t)b * a.kv_bs + (int64_t)hk * a.kv_hs + (int64_t)key0 * D;
    }
    __half* kd = ring + (size_t)(i % ST) * 2 * KG * KP;
    __half* vd = kd + KG * KP;
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int pc = lane + 32 * u;
      const int kl = pc / (D / 8), part = pc % (D / 8);
      const bool live = key0 + kl < j1;
      const int64_t e0 = gbase + (int64_t)(live ? kl : 0) * D + part * 8;  // a dead key reads nothing
      sgd::cp_async_16(kd + kl * KP + part * 8, static_cast<const uint16_t*>(a.K) + e0, live);
      sgd::cp_async_16(vd + kl * KP + part * 8, static_cast<const uint16_t*>(a.V) + e0, live);
    }
  };
  // Keys before q_pos0 were written by earlier steps (or chunks), and the
  // position, the page table and the ranges above come from the host: the
  // warp's first group streams before the dependency wait unless it holds one
  // of the newest keys, which the previous kernel on the stream writes.
  static_assert(ST == 2, "one group in flight ahead of the loop");
  const bool pre = nmine > 0 && j0 + (warp + 1) * KG <= q_pos0;
  if (pre) issue(0);
  sgd::cp_async_commit();
  sgd::pdl_wait();  // the newest keys and the queries come from the previous kernel
  sgd::pdl_launch_dependents();
  if (nmine > 0 && !pre) issue(0);
  sgd::cp_async_commit();

  // Q fragments (A of S = Q K^T), prescaled by scale * log2(e); rows >= R are zero.
  const float qscale = a.scale * 1.4426950408889634f;
  auto q_at = [&](int r, int d) -> float {
    if (r >= R) return 0.f;
    const int h = hk * a.G + r / nq, qi = r % nq;
    return ld_io(a.Q, a.io_dt, (((int64_t)b * a.H + h) * a.Sq + qi) * D + d) * qscale;
  };
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int s2 = 0; s2 < D / 16; ++s2) {
    const int d0 = 16 * s2 + 2 * t;
    qf[s2][0] = pack_half2(q_at(g, d0), q_at(g, d0 + 1));
    qf[s2][1] = pack_half2(q_at(g + 8, d0), q_at(g + 8, d0 + 1));
    qf[s2][2] = pack_half2(q_at(g, d0 + 8), q_at(g, d0 + 9));
    qf[s2][3] = pack_half2(q_at(g + 8, d0 + 8), q_at(g + 8, d0 + 9));
  }
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int q = 0; q < 4; ++q) o[n][q] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;  // rows g and g + 8
  const int r_lo = g, r_hi = g + 8;
  const int qlo = r_lo % nq, qhi = r_hi % nq;

  for (int i = 0; i < nmine; ++i) {
    sgd::cp_async_wait<ST - 2>();  // this lane's pieces of group i have landed
    __half* ks = ring + (size_t)(i % ST) * 2 * KG * KP;
    __half* vs = ks + KG * KP;
    if (IO == SG_DT_BF16) {  // this lane's own pieces, bf16 -> fp16 in place
#pragma unroll
      for (int u = 0; u < NP; ++u) {
        const int pc = lane + 32 * u;
        const int kl = pc / (D / 8), part = pc % (D / 8);
        uint4* kq = reinterpret_cast<uint4*>(ks + kl * KP + part * 8);
        uint4* vq = reinterpret_cast<uint4*>(vs + kl * KP + part * 8);
        *kq = to_f16x8<IO>(*kq);
        *vq = to_f16x8<IO>(*vq);
      }
    }
    __syncwarp();  // the group is in for every lane; group i - 1's stage is free
    if (i + ST - 1 < nmine) issue(i + ST - 1);
    sgd::cp_async_commit();
    const int key0 = j0 + (warp + kW * i) * KG;
    // ---- S = Q K^T: n-tile h covers keys key0 + 8h .. + 7
    float sc[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int q = 0; q < 4; ++q) sc[h][q] = 0.f;
      const __half* krow = ks + (8 * h + g) * KP + 2 * t;
#pragma unroll
      for (int s2 = 0; s2 < D / 16; ++s2) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + 16 * s2);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + 16 * s2 + 8);
        sgd::mma_f16_16816(sc[h], qf[s2][0], qf[s2][1], qf[s2][2], qf[s2][3], b0, b1);
      }
    }
    // mask: keys past the range or (causal) past the row's query position
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int key = key0 + 8 * h + 2 * t + (q & 1);
        const int qi = q < 2 ? qlo : qhi;
        const bool vis = key < j1 && (!a.causal || key <= q_pos0 + qi);
        sc[h][q] = vis ? sc[h][q] : -INFINITY;
        if (q < 2) mx_lo = fmaxf(mx_lo, sc[h][q]);
        else mx_hi = fmaxf(mx_hi, sc[h][q]);
      }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
    }
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    const float al_lo = m_lo == -INFINITY ? 0.f : exp2f(m_lo - mn_lo);
    const float al_hi = m_hi == -INFINITY ? 0.f : exp2f(m_hi - mn_hi);
    float p[2][4], s_lo = 0.f, s_hi = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float mn = q < 2 ? mn_lo : mn_hi;
        p[h][q] = mn == -INFINITY ? 0.f : exp2f(sc[h][q] - mn);
        if (q < 2) s_lo += p[h][q];
        else s_hi += p[h][q];
      }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      s_lo += __shfl_xor_sync(0xffffffffu, s_lo, off);
      s_hi += __shfl_xor_sync(0xffffffffu, s_hi, off);
    }
    m_lo = mn_lo;
    m_hi = mn_hi;
    l_lo = l_lo * al_lo + s_lo;
    l_hi = l_hi * al_hi + s_hi;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= al_lo;
      o[n][1] *= al_lo;
      o[n][2] *= al_hi;
      o[n][3] *= al_hi;
    }
    // ---- O += P V: P [16 rows x 16 keys] as the A fragment straight from the scores
    const uint32_t pa0 = pack_half2(p[0][0], p[0][1]), pa1 = pack_half2(p[0][2], p[0][3]);
    const uint32_t pa2 = pack_half2(p[1][0], p[1][1]), pa3 = pack_half2(p[1][2], p[1][3]);
    const __half* vrow = vs + (lane & 15) * KP;  // ldmatrix rows: keys 0-15
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      uint32_t b0, b1;
      ldmatrix_x2_trans(b0, b1, vrow + 8 * n);
      sgd::mma_f16_16816(o[n], pa0, pa1, pa2, pa3, b0, b1);
    }
  }
  sgd::cp_async_wait<0>();
  __syncthreads();  // every warp is done with its ring: the merge buffer reuses it

  // ---- the warps' partials into [warp][row][D + 2]: O, then max, sum
  float* mine = wm + (size_t)warp * kDecMmaRows * (D + 2);
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int d = 8 * n + 2 * t;
    mine[r_lo * (D + 2) + d] = o[n][0];
    mine[r_lo * (D + 2) + d + 1] = o[n][1];
    mine[r_hi * (D + 2) + d] = o[n][2];
    mine[r_hi * (D + 2) + d + 1] = o[n][3];
  }
  if (t == 0) {
    mine[r_lo * (D + 2) + D] = m_lo;
    mine[r_lo * (D + 2) + D + 1] = l_lo;
    mine[r_hi * (D + 2) + D] = m_hi;
    mine[r_hi * (D + 2) + D + 1] = l_hi;
  }
  __syncthreads();
  // ---- block merge (warp order) straight into rank 0's [split][row][D + 2]
  cg::cluster_group cluster = cg::this_cluster();
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  float* dst = cluster.map_shared_rank(comb, 0) + (size_t)split * R * (D + 2);
  for (int i = tid; i < R * (D + 2); i += kDecWarpThreads) {
    const int r = i / (D + 2), d = i % (D + 2);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kW; ++w) M = fmaxf(M, wm[((size_t)w * kDecMmaRows + r) * (D + 2) + D]);
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) {
      const float* pr = wm + ((size_t)w * kDecMmaRows + r) * (D + 2);
      if (pr[D] == -INFINITY) continue;
      const float wt = exp2f(pr[D] - M);
      acc = fmaf(d == D ? 0.f : (d == D + 1 ? pr[D + 1] : pr[d]), wt, acc);
    }
    dst[i] = d == D ? M : acc;
  }
  cluster.sync();
  if (split != 0) return;
  const int nsplit = a.nsplit;
  for (int i = tid; i < R * D; i += kDecWarpThreads) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, comb[((size_t)sp * R + r) * (D + 2) + D]);
    float L = 0.f, acc = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float* pr = comb + ((size_t)sp * R + r) * (D + 2);
      if (pr[D] == -INFINITY) continue;
      const float wt = exp2f(pr[D] - M);
      L = fmaf(pr[D + 1], wt, L);
      acc = fmaf(pr[d], wt, acc);
    }
    const int h = hk * a.G + r / nq, qi = r % nq;
    st_io(a.O, a.io_dt, (((int64_t)b * a.H + h) * a.Sq + qi) * D + d, L > 0.f ? acc / L : 0.f);
  }
}

std::atomic<int> g_decode_kernel{4};  // decode kernel: 4 warp-split tensor-core cluster, 3 tensor-core cluster, 1 CUDA-core cluster, 2 key-parallel + combine, 0 generic
std::atomic<int> g_decode_cluster_max{kDecClusterMax};  // largest cluster of key splits

}  // namespace

namespace sg {

bool attn_tuning(std::string_view key, int value) {
  if (key == "attn.decode_kernel") {
    g_decode_kernel.store(value);
    return true;
  }
  if (key == "attn.decode_cluster_max") {
    g_decode_cluster_max.store(value);
    return true;
  }
  return false;
}


SgStatus attn_validate(const SgFlashAttentionParams* p, const char* name) {
  SG_CHECK_ARG(p != nullptr, "%s: params is NULL", name);
  SG_CHECK_ARG(p->B >= 0 && p->S >= 0 && p->num_heads >= 0 && p->head_dim >= 0, "%s: negative size", name);
  if (p->B == 0 || p->S == 0 || p->num_heads == 0) return SG_OK;
  SG_CHECK_ARG(p->Q && p->K && p->V && p->O, "%s: Q, K, V and O must be non-NULL", name);
  SG_CHECK_ARG(p->mask == nullptr, "%s: mask is not supported (the reference never reads it)", name);
  SG_CHECK_ARG(p->head_dim >= 1 && p->head_dim <= kMaxD, "%s: head_dim %d outside [1, %d]", name, p->head_dim,
               kMaxD);
  const int hkv = std::max(1, p->num_kv_heads);
  SG_CHECK_ARG(p->num_heads % hkv == 0, "%s: num_heads %d is not a multiple of num_kv_heads %d", name,
               p->num_heads, hkv);
  const int dt = p->io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->io_dtype;
  SG_CHECK_ARG(dt == SG_DT_F16 || dt == SG_DT_F32 || dt == SG_DT_BF16, "%s: io_dtype %d unsupported", name,
               p->io_dtype);
  const int skv = p->S_kv > 0 ? p->S_kv : p->S;
  SG_CHECK_ARG(skv >= 1, "%s: S_kv must be >= 1", name);
  if (const SgKvPages* pg = p->kv_pages) {
    SG_CHECK_ARG(pg->table != nullptr && pg->num_pages > 0, "%s: paged KV cache without a table or pages", name);
    SG_CHECK_ARG(pg->page_size == 16, "%s: page_size %d unsupported (16 tokens per page)", name, pg->page_size);
    SG_CHECK_ARG(pg->page_stride >= (int64_t)hkv * 16 * p->head_dim,
                 "%s: page_stride %lld smaller than a page's %d kv heads", name, (long long)pg->page_stride, hkv);
    SG_CHECK_ARG(pg->table_page_stride != 0 || skv <= 16, "%s: table_page_stride is 0", name);
  }
  return SG_OK;
}

// CUDA-core attention with up to `want_splits` key splits.
SgStatus attn_cc_run(const SgFlashAttentionParams* p, void* stream, int want_splits, void* ws, size_t ws_bytes,
                     bool ws_external) {
  const char* name = "sg_flash_attention";
  SgStatus st = attn_validate(p, name);
  if (st != SG_OK) return st;
  if (p->B == 0 || p->S == 0 || p->num_heads == 0) return SG_OK;
  int dev = 0;
  st = current_device(&dev);
  if (st != SG_OK) return st;
  cudaStream_t cs = static_cast<cudaStream_t>(stream);

  AArgs a{};
  a.Q = p->Q;
  a.K = p->K;
  a.V = p->V;
  a.O = p->O;
  a.B = p->B;
  a.H = p->num_heads;
  a.Hkv = std::max(1, p->num_kv_heads);
  a.G = a.H / a.Hkv;
  a.Sq = p->S;
  a.Skv = p->S_kv > 0 ? p->S_kv : p->S;
  a.D = p->head_dim;
  a.scale = p->scale > 0.f ? p->scale : 1.0f / sqrtf((float)p->head_dim);
  a.causal = p->causal != 0;
  a.q_pos0 = p->q_pos0 >= 0 ? p->q_pos0 : a.Skv - a.Sq;
  a.q_pos_dev = p->q_pos_device;
  a.kv_hs = p->kv_head_stride > 0 ? p->kv_head_stride : (int64_t)a.Skv * a.D;
  a.kv_bs = p->kv_batch_stride > 0 ? p->kv_batch_stride : (int64_t)a.Hkv * a.kv_hs;
  a.io_dt = p->io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->io_dtype;
  if (const SgKvPages* pg = p->kv_pages) {
    a.pt = pg->table;
    a.pt_bs = pg->table_batch_stride;
    a.pt_ps = pg->table_page_stride;
    a.page_stride = pg->page_stride;
    a.npages = pg->num_pages;
    st = device_error_word(&a.err);
    if (st != SG_OK) return st;
    a.kv_hs = (int64_t)16 * a.D;  // within a page; for the alignment checks below
    a.kv_bs = pg->page_stride;
  }
  // query positions per work item: at most kWarps * kMaxRowsPerWarp rows (G * qb)
  a.qb = std::max(1, (kWarps * kMaxRowsPerWarp) / a.G);
  SG_CHECK_ARG(a.G <= kWarps * kMaxRowsPerWarp, "%s: more than %d query heads per kv head", name,
               kWarps * kMaxRowsPerWarp);
  const int nqb = (a.Sq + a.qb - 1) / a.qb;
  const int sms = sm_count(dev);
  int nsplit = 1;
  if (want_splits > 1) {
    const int items = nqb * a.Hkv * a.B;
    nsplit = std::max(1, std::min({want_splits, (a.Skv + kKeyTile - 1) / kKeyTile, (4 * sms + items - 1) / items}));
  }
  a.nsplit = nsplit;
  a.keys_per_split = (a.Skv + nsplit - 1) / nsplit;
  if (nsplit > 1) {
    const size_t need = (size_t)a.B * a.H * a.Sq * nsplit * (a.D + 2) * sizeof(float);
    if (ws == nullptr) {
      if (ws_external) {
        set_error("%s: scratch required (%zu bytes)", name, need);
        return SG_ERR_INVALID;
      }
      st = library_workspace(stream, need, &ws, kWsAttention);
      if (st != SG_OK) return st;
    } else {
      SG_CHECK_ARG(ws_bytes >= need, "%s: workspace too small (%zu < %zu bytes)", name, ws_bytes, need);
    }
    a.part = static_cast<float*>(ws);
  }
  // Few query rows per kv head (decode): one cluster of key splits per (batch, kv head).
  const int R = a.G * a.Sq;
  const int eb = a.io_dt == SG_DT_F32 ? 4 : 2;
  const bool vec_ok = aligned16(a.K) && aligned16(a.V) && (a.kv_hs * eb) % 16 == 0 && (a.kv_bs * eb) % 16 == 0;
  const int mode = g_decode_kernel.load();
  const bool use_warp = mode == 4 && eb == 2 && (a.D == 64 || a.D == 128) && R <= kDecMmaRows && vec_ok;
  if (use_warp) {
    // splits: as many as the capacity of one wave allows (blocks per SM from shared memory)
    const int tiles = (a.Skv + kDecTile - 1) / kDecTile;
    const int items = a.Hkv * a.B;
    int cmax = std::max(1, std::min(kDecClusterMax, g_decode_cluster_max.load()));
    while (cmax > 1 && dec_warp_smem(a.D, R, cmax) > 200 * 1024) --cmax;  // rank 0 holds every split's rows
    void (*kfn)(AArgs) = a.D == 64 ? (a.io_dt == SG_DT_BF16 ? attn_dec_warp_kernel<64, SG_DT_BF16>
                                                            : attn_dec_warp_kernel<64, SG_DT_F16>)
                                   : (a.io_dt == SG_DT_BF16 ? attn_dec_warp_kernel<128, SG_DT_BF16>
                                                            : attn_dec_warp_kernel<128, SG_DT_F16>);
    const size_t smem_max = dec_warp_smem(a.D, R, cmax);
    SG_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_max));
    int per_sm = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kDecWarpThreads, smem_max) != cudaSuccess) {
      cudaGetLastError();
      per_sm = 1;
    }
    const int ns = std::max(1, std::min({cmax, tiles, (std::max(1, per_sm) * sms) / items}));
    const int tiles_per = (tiles + ns - 1) / ns;
    a.keys_per_split = tiles_per * kDecTile;
    a.nsplit = (tiles + tiles_per - 1) / tiles_per;
    const size_t smem = dec_warp_smem(a.D, R, a.nsplit);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nsplit, a.Hkv, a.B);
    cfg.blockDim = dim3(kDecWarpThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = cs;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.nsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (a.nsplit > 8) SG_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    SG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, a));
    return SG_OK;
  }
  const bool use_mma = (mode == 3 || mode == 4) && eb == 2 && (a.D == 64 || a.D == 128) && R <= kDecMmaRows && vec_ok;
  const bool use_cl = (mode == 4 || mode == 3 || mode == 1) && (a.D == 64 || (a.D == 128 && eb == 2)) && R <= kDecRows &&
                      vec_ok;
  if (use_mma || use_cl) {
    auto smem_of = [&](int ns) { return use_mma ? dec_mma_smem(a.D, R, ns) : dec_cluster_smem(a.D, R, ns); };
    const int tiles = (a.Skv + kDecTile - 1) / kDecTile;
    const int items = a.Hkv * a.B;
    const int cmax = std::max(1, std::min(kDecClusterMax, g_decode_cluster_max.load()));
    int ns = std::max(1, std::min({cmax, tiles, (2 * sms + items - 1) / items}));
    while (ns > 1 && smem_of(ns) > 200 * 1024) --ns;
    const int tiles_per = (tiles + ns - 1) / ns;
    a.keys_per_split = tiles_per * kDecTile;
    a.nsplit = (tiles + tiles_per - 1) / tiles_per;
    const size_t smem = smem_of(a.nsplit);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nsplit, a.Hkv, a.B);
    cfg.blockDim = dim3(use_mma ? kDecMmaThreads : kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = cs;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.nsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    auto launch_cl = [&](void (*kfn)(AArgs)) -> SgStatus {
      SG_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      if (a.nsplit > 8) SG_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
      SG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, a));
      return SG_OK;
    };
    if (use_mma) {
      if (a.D == 64)
        return launch_cl(a.io_dt == SG_DT_BF16 ? attn_dec_mma_kernel<64, SG_DT_BF16> : attn_dec_mma_kernel<64, SG_DT_F16>);
      return launch_cl(a.io_dt == SG_DT_BF16 ? attn_dec_mma_kernel<128, SG_DT_BF16>
                                             : attn_dec_mma_kernel<128, SG_DT_F16>);
    }
    if (a.D == 64) {
      if (a.io_dt == SG_DT_F32) return launch_cl(attn_dec_cluster_kernel<64, SG_DT_F32>);
      if (a.io_dt == SG_DT_BF16) return launch_cl(attn_dec_cluster_kernel<64, SG_DT_BF16>);
      return launch_cl(attn_dec_cluster_kernel<64, SG_DT_F16>);
    }
    if (a.io_dt == SG_DT_BF16) return launch_cl(attn_dec_cluster_kernel<128, SG_DT_BF16>);
    return launch_cl(attn_dec_cluster_kernel<128, SG_DT_F16>);
  }
  // The key-parallel kernel with a separate combine.
  if ((a.D == 64 || a.D == 128) && R <= kDecRows && g_decode_kernel.load() != 0) {
    const dim3 dgrid(nsplit, a.Hkv, a.B);
    // shared-memory attribute set once per (kernel, device)
    static std::atomic<uint64_t> set_mask[2] = {{0}, {0}};
    auto launch_dec = [&](void (*kfn)(AArgs), size_t sm, int which) -> SgStatus {
      const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
      if (!(set_mask[which].load() & bit)) {
        SG_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        set_mask[which].fetch_or(bit);
      }
      kfn<<<dgrid, kThreads, sm, cs>>>(a);
      return check_launch("attn_decode_kernel");
    };
    a.qb = a.Sq;
    st = a.D == 64 ? launch_dec(attn_decode_kernel<64>, decode_smem<64>(), 0)
                   : launch_dec(attn_decode_kernel<128>, decode_smem<128>(), 1);
    if (st != SG_OK || nsplit == 1) return st;
    attn_combine_kernel<<<a.B * a.H * a.Sq, 64, 0, cs>>>(a);
    return check_launch("attn_combine_kernel");
  }
  const size_t smem = (size_t)2 * kKeyTile * a.D * sizeof(float);
  dim3 grid(nqb * nsplit, a.Hkv, a.B);
  const int dpl = (a.D + 31) / 32;
  auto launch = [&](auto kfn) -> SgStatus {
    if (smem > 48 * 1024) SG_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kfn<<<grid, kThreads, smem, cs>>>(a);
    return check_launch("attn_cc_kernel");
  };
  if (dpl <= 1) st = launch(attn_cc_kernel<1>);
  else if (dpl <= 2) st = launch(attn_cc_kernel<2>);
  else if (dpl <= 4) st = launch(attn_cc_kernel<4>);
  else st = launch(attn_cc_kernel<8>);
  if (st != SG_OK || nsplit == 1) return st;
  attn_combine_kernel<<<a.B * a.H * a.Sq, 64, 0, cs>>>(a);
  return check_launch("attn_combine_kernel");
}

size_t attn_cc_scratch_bytes(const SgFlashAttentionParams* p, int want_splits) {
  if (attn_validate(p, "workspace_size") != SG_OK || p->B == 0 || p->S == 0 || p->num_heads == 0) return 0;
  if (want_splits <= 1) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = 0;
  }
  const int hkv = std::max(1, p->num_kv_heads), G = p->num_heads / hkv;
  const int skv = p->S_kv > 0 ? p->S_kv : p->S;
  const int qb = std::max(1, (kWarps * kMaxRowsPerWarp) / G);
  const int nqb = (p->S + qb - 1) / qb;
  const int items = nqb * hkv * p->B;
  const int nsplit =
      std::max(1, std::min({want_splits, (skv + kKeyTile - 1) / kKeyTile, (4 * sm_count(dev) + items - 1) / items}));
  if (nsplit == 1) return 0;
  return (size_t)p->B * p->num_heads * p->S * nsplit * (p->head_dim + 2) * sizeof(float);
}

}  // namespace sg

extern "C" {

SgStatus sg_flash_attention(const SgFlashAttentionParams* p, void* stream) {
  SgStatus st = sg::attn_validate(p, "sg_flash_attention");
  if (st != SG_OK) return st;
  if (p->B == 0 || p->S == 0 || p->num_heads == 0) return SG_OK;
  bool handled = false;
  st = sg::attn_tc_run(p, static_cast<cudaStream_t>(stream), p->workspace, p->workspace_bytes,
                       p->workspace != nullptr, &handled);
  if (st != SG_OK || handled) return st;
  if (p->workspace) return sg::attn_cc_run(p, stream, 8, p->workspace, p->workspace_bytes, true);
  return sg::attn_cc_run(p, stream, 8, nullptr, 0, false);
}

size_t sg_flash_attention_workspace_size(const SgFlashAttentionParams* p) {
  const size_t tc = sg::attn_tc_scratch_bytes(p);
  const size_t cc = sg::attn_cc_scratch_bytes(p, 8);
  return tc > cc ? tc : cc;
}

// Decode: split the keys over many CTAs (flash-decoding) and merge.
SgStatus sg_flash_decode(const SgFlashAttentionParams* p, void* stream) {
  if (p && p->workspace) return sg::attn_cc_run(p, stream, 64, p->workspace, p->workspace_bytes, true);
  return sg::attn_cc_run(p, stream, 64, nullptr, 0, false);
}

size_t sg_flash_decode_workspace_size(const SgFlashAttentionParams* p) { return sg::attn_cc_scratch_bytes(p, 64); }

}  // extern "C"
