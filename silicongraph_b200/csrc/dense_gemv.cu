// INT8 per-channel and fp16-weight GEMV (decode) for sm_100a.
//
// sg_matmul_int8_channel replaces the GLSL gemm_int8 shader
// (compiler/kernels/gpu/vulkan_shaders.h:53-82) / OpenCL gemm_int8_m1
// (opencl_kernels.h:36-52):  B int8 [K, N] row-major, scales f32 [N],
//   int8 A:  C[n] = float(sum_k A[k]*B[k,n] as int32) * scale_A * scales[n]
//   float A: C[n] = scales[n] * sum_k A[k]*float(B[k,n])           (fp32)
// sg_matmul_fp16 replaces matmul_fp16_neon_m1 (matmul_neon.h:48-107):
//   B fp16 [K, N] row-major, C[n] = sum_k A[k]*B[k,n] (+ bias[n]).
//
// Same streaming structure as the INT4 kernel: a lane owns 16 consecutive
// columns and reads one row of them per 128-bit load (two for fp16), 8 warps
// split the block's rows, blocks split K, and partials are reduced by the
// last block of each column tile in fixed order.
//   * int8 A: four rows of a lane are transposed 4x4 bytes with PRMT so each
//     32-bit word holds one column's four k values, then dp4a accumulates in
//     int32 -- exact, hence bit-identical to the shader for any split.
//   * float A (int8 weights): x is staged as 24-bit fixed point per 8-row chunk
//     (one power-of-two scale per chunk, |error| at most 2^-22 of the chunk's
//     largest |x|, or 2^-122 when that is below 2^-100 and the exponent is
//     clamped), split into signed hi / mid / lo bytes; the weights meet all
//     three in dp4a (exact int32) after the same 4x4 transpose, and each
//     chunk adds scale * (256 (256 hi_sum + mid_sum) + lo_sum) to the fp32
//     accumulators.  (16 bits were not enough: with one outlier of 100..1000
//     among the activations, columns whose sum nearly cancels missed
//     2e-3 + 1e-2 |y|.)
//   * fp16 B: half2 -> float2 conversion and packed fp32x2 FMAs.
#include <algorithm>
#include <atomic>

#include "sm100.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kColsPerLane = 16;
constexpr int kColsPerBlock = 32 * kColsPerLane;  // 512
constexpr int kRowsPerChunk = 8;                   // rows per warp step (multiple of 4)
constexpr int kChunkBytes = kRowsPerChunk * kColsPerBlock;  // int8: one warp step, 4 KB
constexpr int kI8Warps = 16;                       // int8: warps per block (one block per SM)
constexpr int kI8Stages = 3;                       // int8: chunks in flight per warp (cp.async ring)

enum WKind { W_INT8_IA = 0, W_INT8_FA = 1, W_F16 = 2 };

struct DArgs {
  const void* A;
  const uint8_t* B;      // byte pointer to weights
  const float* scales;   // int8: [N]
  const __half* bias;    // fp16: [N] or NULL
  void* C;
  int M, K, N, lda, ldc;
  int a_dt, c_dt;
  float scale_A;
  int rows_per_split, ksplit;
  int ring_off;        // int8: byte offset of the per-warp cp.async rings in dynamic shared memory
  float* partial;      // [ksplit][M][N] (float)  or int32 for W_INT8_IA
  unsigned* tickets;
};

__device__ __forceinline__ float load_act(const void* A, int dt, int64_t i) {
  switch (dt) {
    case SG_DT_F32: return sgd::load_as_float<SG_DT_F32>(A, i);
    case SG_DT_F16: return sgd::load_as_float<SG_DT_F16>(A, i);
    case SG_DT_BF16: return sgd::load_as_float<SG_DT_BF16>(A, i);
    default: return sgd::load_as_float<SG_DT_I8>(A, i);
  }
}

__device__ __forceinline__ void store_out(void* C, int dt, int64_t i, float v) {
  switch (dt) {
    case SG_DT_F32: sgd::store_from_float<SG_DT_F32>(C, i, v); break;
    case SG_DT_BF16: sgd::store_from_float<SG_DT_BF16>(C, i, v); break;
    default: sgd::store_from_float<SG_DT_F16>(C, i, v); break;
  }
}

template <int KIND>
__device__ __forceinline__ float finalize_f(const DArgs& a, int col, float v) {
  if (KIND == W_INT8_FA) v = v * a.scales[col];
  if (KIND == W_F16 && a.bias) v = v + __half2float(a.bias[col]);
  return v;
}

__device__ __forceinline__ float finalize_i(const DArgs& a, int col, int acc) {
  // vulkan_shaders.h:80: float(acc) * scale_A * Scales[n], left to right
  return __fmul_rn(__fmul_rn((float)acc, a.scale_A), a.scales[col]);
}

// 4x4 byte transpose: in w[r] = row r (bytes = columns 0..3); out c[b] = column b (bytes = rows 0..3).
__device__ __forceinline__ void transpose4x4(const uint32_t w0, const uint32_t w1, const uint32_t w2,
                                             const uint32_t w3, uint32_t c[4]) {
  const uint32_t t0 = __byte_perm(w0, w1, 0x5140);  // w0.b0 w1.b0 w0.b1 w1.b1
  const uint32_t t1 = __byte_perm(w2, w3, 0x5140);  // w2.b0 w3.b0 w2.b1 w3.b1
  const uint32_t t2 = __byte_perm(w0, w1, 0x7362);  // w0.b2 w1.b2 w0.b3 w1.b3
  const uint32_t t3 = __byte_perm(w2, w3, 0x7362);
  c[0] = __byte_perm(t0, t1, 0x5410);
  c[1] = __byte_perm(t0, t1, 0x7632);
  c[2] = __byte_perm(t2, t3, 0x5410);
  c[3] = __byte_perm(t2, t3, 0x7632);
}

template <int KIND>
__global__ void __launch_bounds__(KIND == W_F16 ? kThreads : kI8Warps * 32, KIND == W_F16 ? 2 : 1) dense_gemv_kernel(DArgs a) {
  constexpr int W = KIND == W_F16 ? kWarps : kI8Warps;  // warps per block
  constexpr int T = W * 32;
  extern __shared__ float xs_f[];  // staged activations for this block's rows
  const int tile = blockIdx.x, split = blockIdx.y;
  const int r_begin = split * a.rows_per_split;
  const int r_end = min(a.K, r_begin + a.rows_per_split);
  const int nrows = r_end - r_begin;
  const int nrows_pad = (nrows + kRowsPerChunk - 1) / kRowsPerChunk * kRowsPerChunk;

  // stage x (zero padded to a whole number of chunks)
  if (KIND == W_INT8_IA) {
    int32_t* xq = reinterpret_cast<int32_t*>(xs_f);  // packed int8 quads
    for (int i = threadIdx.x; i < nrows_pad / 4; i += T) {
      uint32_t v = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = r_begin + 4 * i + j;
        const int8_t x = (k < r_end) ? static_cast<const int8_t*>(a.A)[k] : (int8_t)0;
        v |= (uint32_t)(uint8_t)x << (8 * j);
      }
      xq[i] = (int32_t)v;
    }
  } else if (KIND == W_INT8_FA) {
    // float activations as 24-bit fixed point per 8-row chunk: x = 2^(E-21) q, E the
    // exponent of the chunk's largest |x| (|q| <= 2^22, error at most 2^-22 of that
    // value), q = 65536 hi + 256 mid + lo in signed bytes, so the weights meet them in dp4a
    int8_t* xhi = reinterpret_cast<int8_t*>(xs_f);
    int8_t* xmid = xhi + nrows_pad;
    int8_t* xlo = xhi + 2 * nrows_pad;
    float* sx = reinterpret_cast<float*>(xhi + 3 * nrows_pad);
    const int lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < (nrows_pad + T - 1) / T * T; i += T) {
      const int k = r_begin + i;
      const float x = (i < nrows_pad && k < r_end) ? load_act(a.A, a.a_dt, k) : 0.f;
      float m = fabsf(x);
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const int E = max((__float_as_int(m) >> 23) - 127, -100);
      const int q = __float2int_rn(x * __int_as_float((127 + 21 - E) << 23));
      const int lo = ((q + 128) & 255) - 128, r = (q - lo) >> 8;
      const int mid = ((r + 128) & 255) - 128, hi = (r - mid) >> 8;
      if (i < nrows_pad) {
        xhi[i] = (int8_t)hi;
        xmid[i] = (int8_t)mid;
        xlo[i] = (int8_t)lo;
        if ((lane & 7) == 0) sx[i / 8] = __int_as_float((127 - 21 + E) << 23);  // 2^(E - 21)
      }
    }
  } else {
    for (int i = threadIdx.x; i < nrows_pad; i += T) {
      const int k = r_begin + i;
      xs_f[i] = (k < r_end) ? load_act(a.A, a.a_dt, k) : 0.f;
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col0 = tile * kColsPerBlock + lane * kColsPerLane;
  const bool col_ok = col0 < a.N;
  constexpr int ESZ = (KIND == W_F16) ? 2 : 1;

  float accf[16];
  int acci[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    accf[c] = 0.f;
    acci[c] = 0;
  }

  if (col_ok && KIND == W_F16) {
    const uint8_t* Bcol = a.B + (int64_t)col0 * ESZ;
    for (int ch = warp * kRowsPerChunk; ch < nrows_pad; ch += W * kRowsPerChunk) {
      {
        uint4 wv[kRowsPerChunk][2];
#pragma unroll
        for (int r = 0; r < kRowsPerChunk; ++r) {
          const int k = r_begin + ch + r;
          if (k < r_end) {
            const uint8_t* p = Bcol + (int64_t)k * a.N * 2;
            wv[r][0] = sgd::ldg_stream(p);
            wv[r][1] = sgd::ldg_stream(p + 16);
          } else {
            wv[r][0] = wv[r][1] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
#pragma unroll
        for (int r = 0; r < kRowsPerChunk; ++r) {
          const float x = xs_f[ch + r];
          const float2 xx = make_float2(x, x);
          const uint32_t words[8] = {wv[r][0].x, wv[r][0].y, wv[r][0].z, wv[r][0].w,
                                     wv[r][1].x, wv[r][1].y, wv[r][1].z, wv[r][1].w};
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float2 w2 = __half22float2(*reinterpret_cast<const __half2*>(&words[q]));
            const float2 acc2 = sgd::ffma2(w2, xx, make_float2(accf[2 * q], accf[2 * q + 1]));
            accf[2 * q] = acc2.x;
            accf[2 * q + 1] = acc2.y;
          }
        }
      }
    }
  }
  if (col_ok && KIND != W_F16) {
    // int8 weights: every lane streams its own 16 bytes of each row of its warp's
    // chunks through a cp.async ring in shared memory (kI8Stages chunks in flight
    // per warp); a lane reads back only what it copied, so no warp barrier
    uint8_t* ring = reinterpret_cast<uint8_t*>(xs_f) + a.ring_off + (size_t)warp * kI8Stages * kChunkBytes + lane * 16;
    const uint8_t* Bcol = a.B + (int64_t)col0;
    constexpr int kStep = W * kRowsPerChunk;
    const int first = warp * kRowsPerChunk;
    const int nmy = first < nrows_pad ? (nrows_pad - first + kStep - 1) / kStep : 0;
    auto issue = [&](int i) {
      const int ch = first + i * kStep;
      uint8_t* dst = ring + (i % kI8Stages) * kChunkBytes;
#pragma unroll
      for (int r = 0; r < kRowsPerChunk; ++r) {
        const int k = r_begin + ch + r;
        const bool live = k < r_end;
        sgd::cp_async_16(dst + r * kColsPerBlock, Bcol + (int64_t)(live ? k : r_begin) * a.N, live);
      }
    };
    for (int i = 0; i < kI8Stages - 1; ++i) {
      if (i < nmy) issue(i);
      sgd::cp_async_commit();
    }
    for (int i = 0; i < nmy; ++i) {
      sgd::cp_async_wait<kI8Stages - 2>();  // this lane's copies of chunk i have landed
      if (i + kI8Stages - 1 < nmy) issue(i + kI8Stages - 1);  // into chunk i - 1's stage (read already)
      sgd::cp_async_commit();
      const int ch = first + i * kStep;
      const uint8_t* src = ring + (i % kI8Stages) * kChunkBytes;
      uint4 wv[kRowsPerChunk];
#pragma unroll
      for (int r = 0; r < kRowsPerChunk; ++r) wv[r] = *reinterpret_cast<const uint4*>(src + r * kColsPerBlock);
      if (KIND == W_INT8_IA) {
        const int32_t* xq = reinterpret_cast<const int32_t*>(xs_f);
#pragma unroll
        for (int r4 = 0; r4 < kRowsPerChunk; r4 += 4) {
          const int32_t a4 = xq[(ch + r4) / 4];
          const uint32_t rows[4][4] = {{wv[r4].x, wv[r4].y, wv[r4].z, wv[r4].w},
                                       {wv[r4 + 1].x, wv[r4 + 1].y, wv[r4 + 1].z, wv[r4 + 1].w},
                                       {wv[r4 + 2].x, wv[r4 + 2].y, wv[r4 + 2].z, wv[r4 + 2].w},
                                       {wv[r4 + 3].x, wv[r4 + 3].y, wv[r4 + 3].z, wv[r4 + 3].w}};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t cw[4];
            transpose4x4(rows[0][q], rows[1][q], rows[2][q], rows[3][q], cw);
#pragma unroll
            for (int b = 0; b < 4; ++b) acci[4 * q + b] = __dp4a((int)cw[b], a4, acci[4 * q + b]);
          }
        }
      } else {
        // exact int32 dot products with the hi, mid and lo bytes of this chunk's fixed-point x
        const int32_t* xh = reinterpret_cast<const int32_t*>(xs_f);
        const int32_t* xm = reinterpret_cast<const int32_t*>(reinterpret_cast<const int8_t*>(xs_f) + nrows_pad);
        const int32_t* xl = reinterpret_cast<const int32_t*>(reinterpret_cast<const int8_t*>(xs_f) + 2 * nrows_pad);
        const float* sx = reinterpret_cast<const float*>(reinterpret_cast<const int8_t*>(xs_f) + 3 * nrows_pad);
        int ah[16], am[16], al[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) ah[c] = am[c] = al[c] = 0;
#pragma unroll
        for (int r4 = 0; r4 < kRowsPerChunk; r4 += 4) {
          const int32_t h4 = xh[(ch + r4) / 4], m4 = xm[(ch + r4) / 4], l4 = xl[(ch + r4) / 4];
          const uint32_t rows[4][4] = {{wv[r4].x, wv[r4].y, wv[r4].z, wv[r4].w},
                                       {wv[r4 + 1].x, wv[r4 + 1].y, wv[r4 + 1].z, wv[r4 + 1].w},
                                       {wv[r4 + 2].x, wv[r4 + 2].y, wv[r4 + 2].z, wv[r4 + 2].w},
                                       {wv[r4 + 3].x, wv[r4 + 3].y, wv[r4 + 3].z, wv[r4 + 3].w}};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t cw[4];
            transpose4x4(rows[0][q], rows[1][q], rows[2][q], rows[3][q], cw);
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              ah[4 * q + b] = __dp4a((int)cw[b], h4, ah[4 * q + b]);
              am[4 * q + b] = __dp4a((int)cw[b], m4, am[4 * q + b]);
              al[4 * q + b] = __dp4a((int)cw[b], l4, al[4 * q + b]);
            }
          }
        }
        const float sc = sx[ch / kRowsPerChunk];
#pragma unroll
        for (int c = 0; c < 16; ++c)  // |256 ah + am| <= 2^24 + 2^16: int32, one rounding as a float
          accf[c] = fmaf(fmaf(256.f, (float)(ah[c] * 256 + am[c]), (float)al[c]), sc, accf[c]);
      }
    }
    sgd::cp_async_wait<0>();
  }

  // ---- reduce the 8 warps (fixed order), then split-K
  __syncthreads();
  __shared__ bool s_last;
  float* red = xs_f;  // [W][512] (int32 bits for W_INT8_IA)
  if (col_ok) {
#pragma unroll
    for (int c = 0; c < 16; ++c)
      red[warp * kColsPerBlock + lane * kColsPerLane + c] =
          (KIND == W_INT8_IA) ? __int_as_float(acci[c]) : accf[c];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < kColsPerBlock; c += T) {
    const int col = tile * kColsPerBlock + c;
    if (col >= a.N) continue;
    if (KIND == W_INT8_IA) {
      int v = 0;
#pragma unroll
      for (int w = 0; w < W; ++w) v += __float_as_int(red[w * kColsPerBlock + c]);
      if (a.ksplit == 1) store_out(a.C, a.c_dt, col, finalize_i(a, col, v));
      else reinterpret_cast<int*>(a.partial)[(int64_t)split * a.N + col] = v;
    } else {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) v += red[w * kColsPerBlock + c];
      if (a.ksplit == 1) store_out(a.C, a.c_dt, col, finalize_f<KIND>(a, col, v));
      else a.partial[(int64_t)split * a.N + col] = v;
    }
  }
  if (a.ksplit == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.tickets[tile], 1u);
    s_last = (prev == (unsigned)(a.ksplit - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int c = threadIdx.x; c < kColsPerBlock; c += T) {
    const int col = tile * kColsPerBlock + c;
    if (col >= a.N) continue;
    if (KIND == W_INT8_IA) {
      int v = 0;
      for (int sp = 0; sp < a.ksplit; ++sp)
        v += __ldcg(&reinterpret_cast<const int*>(a.partial)[(int64_t)sp * a.N + col]);
      store_out(a.C, a.c_dt, col, finalize_i(a, col, v));
    } else {
      float v = 0.f;
      for (int sp = 0; sp < a.ksplit; ++sp) v += __ldcg(&a.partial[(int64_t)sp * a.N + col]);
      store_out(a.C, a.c_dt, col, finalize_f<KIND>(a, col, v));
    }
  }
  if (threadIdx.x == 0) a.tickets[tile] = 0u;
}

// Reference-order loops, one thread per output (any shape / alignment).
template <int KIND>
__global__ void dense_gemv_generic_kernel(DArgs a) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= a.N || m >= a.M) return;
  if (KIND == W_INT8_IA) {
    int acc = 0;
    for (int k = 0; k < a.K; ++k)
      acc += (int)static_cast<const int8_t*>(a.A)[(int64_t)m * a.lda + k] *
             (int)reinterpret_cast<const int8_t*>(a.B)[(int64_t)k * a.N + n];
    store_out(a.C, a.c_dt, (int64_t)m * a.ldc + n, finalize_i(a, n, acc));
  } else {
    float acc = 0.f;
    for (int k = 0; k < a.K; ++k) {
      const float w = (KIND == W_F16) ? __half2float(reinterpret_cast<const __half*>(a.B)[(int64_t)k * a.N + n])
                                      : (float)reinterpret_cast<const int8_t*>(a.B)[(int64_t)k * a.N + n];
      acc = __fadd_rn(acc, __fmul_rn(load_act(a.A, a.a_dt, (int64_t)m * a.lda + k), w));
    }
    if (KIND == W_INT8_FA) acc = __fmul_rn(acc, a.scales[n]);
    if (KIND == W_F16 && a.bias) acc = __fadd_rn(acc, __half2float(a.bias[n]));
    store_out(a.C, a.c_dt, (int64_t)m * a.ldc + n, acc);
  }
}

struct Plan {
  bool fast = false;
  int rows_per_split = 0, ksplit = 1, n_tiles = 0, ring_off = 0;
  size_t smem = 0, ws_bytes = 0, tickets_bytes = 0;
};

Plan make_plan(int kind, const SgMatMulParams* p, int sms) {
  Plan pl;
  const int esz = kind == W_F16 ? 2 : 1;
  pl.fast = p->M >= 1 && p->K > 0 && (p->N % 16 == 0) && sg::aligned16(p->B);
  if (!pl.fast) return pl;
  (void)esz;
  pl.n_tiles = (p->N + kColsPerBlock - 1) / kColsPerBlock;
  // chunks of 8 rows are the unit of work of one warp step
  const long chunks = (p->K + kRowsPerChunk - 1) / kRowsPerChunk;
  long chunks_per_split;
  if (kind == W_F16) {
    const long units = (long)pl.n_tiles * chunks;
    const long target = (long)sms * 4 * kWarps * 2;  // ~2 chunks per warp, ~4 blocks per SM
    chunks_per_split = std::max<long>(kWarps, (units + target - 1) / target * kWarps);
  } else {
    // int8: one 16-warp block per SM (its warps' cp.async rings fill the shared
    // memory), each warp streaming several chunks; rounded down to one wave
    const long ks = std::max<long>(1, std::min<long>(chunks / kI8Warps, (long)sms / pl.n_tiles));
    chunks_per_split = std::max<long>(kI8Warps, ((chunks + ks - 1) / ks + kI8Warps - 1) / kI8Warps * kI8Warps);
  }
  chunks_per_split = std::min<long>(chunks_per_split, 4096 / kRowsPerChunk);  // x stage <= 16 KB
  pl.rows_per_split = (int)(chunks_per_split * kRowsPerChunk);
  pl.ksplit = (p->K + pl.rows_per_split - 1) / pl.rows_per_split;
  const size_t xs_bytes = (size_t)pl.rows_per_split * 4;
  const size_t red_bytes = (size_t)(kind == W_F16 ? kWarps : kI8Warps) * kColsPerBlock * 4;
  pl.smem = std::max(xs_bytes, red_bytes);
  if (kind != W_F16) {
    pl.ring_off = (int)sg::align_up(pl.smem, (size_t)16);
    pl.smem = (size_t)pl.ring_off + (size_t)kI8Warps * kI8Stages * kChunkBytes;
  }
  if (pl.ksplit > 1) {
    pl.tickets_bytes = sg::ticket_bytes(pl.n_tiles);
    pl.ws_bytes = pl.tickets_bytes + (size_t)pl.ksplit * p->N * 4;
  }
  return pl;
}

int kind_of(bool int8_weights, int a_dt) {
  if (!int8_weights) return W_F16;
  return a_dt == SG_DT_I8 ? W_INT8_IA : W_INT8_FA;
}

SgStatus validate(const char* name, const SgMatMulParams* p, bool int8_weights) {
  SG_CHECK_ARG(p != nullptr, "%s: params is NULL", name);
  SG_CHECK_ARG(p->M >= 0 && p->K >= 0 && p->N >= 0, "%s: negative size", name);
  if (p->M == 0 || p->N == 0) return SG_OK;
  SG_CHECK_ARG(p->C != nullptr, "%s: C is NULL", name);
  SG_CHECK_ARG(p->K == 0 || (p->A && p->B), "%s: A and B must be non-NULL", name);
  SG_CHECK_ARG(!int8_weights || p->scales_B, "%s: scales_B must be non-NULL", name);
  SG_CHECK_ARG(p->ldb <= 0 || p->ldb == p->N, "%s: ldb must be N", name);
  SG_CHECK_ARG(p->lda <= 0 || p->lda >= p->K, "%s: lda < K", name);
  SG_CHECK_ARG(p->ldc <= 0 || p->ldc >= p->N, "%s: ldc < N", name);
  const int adt = p->a_dtype == SG_DT_DEFAULT ? (int8_weights ? SG_DT_I8 : SG_DT_F16) : p->a_dtype;
  SG_CHECK_ARG(adt >= SG_DT_F32 && adt <= SG_DT_I8, "%s: bad a_dtype %d", name, p->a_dtype);
  const int cdt = p->c_dtype == SG_DT_DEFAULT ? (int8_weights ? SG_DT_F32 : SG_DT_F16) : p->c_dtype;
  SG_CHECK_ARG(cdt == SG_DT_F32 || cdt == SG_DT_F16 || cdt == SG_DT_BF16, "%s: bad c_dtype %d", name,
               p->c_dtype);
  return SG_OK;
}

SgStatus dense_run(const char* name, const SgMatMulParams* p, void* stream, bool int8_weights) {
  SgStatus st = validate(name, p, int8_weights);
  if (st != SG_OK) return st;
  if (p->M == 0 || p->N == 0) return SG_OK;
  int dev = 0;
  st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  cudaStream_t cs = static_cast<cudaStream_t>(stream);

  DArgs a{};
  a.A = p->A;
  a.B = static_cast<const uint8_t*>(p->B);
  a.scales = static_cast<const float*>(p->scales_B);
  a.bias = static_cast<const __half*>(p->bias);
  a.C = p->C;
  a.M = p->M;
  a.K = p->K;
  a.N = p->N;
  a.lda = p->lda > 0 ? p->lda : p->K;
  a.ldc = p->ldc > 0 ? p->ldc : p->N;
  a.a_dt = p->a_dtype == SG_DT_DEFAULT ? (int8_weights ? SG_DT_I8 : SG_DT_F16) : p->a_dtype;
  a.c_dt = p->c_dtype == SG_DT_DEFAULT ? (int8_weights ? SG_DT_F32 : SG_DT_F16) : p->c_dtype;
  a.scale_A = p->scale_A;
  const int kind = kind_of(int8_weights, a.a_dt);

  // Float activations over many rows with INT8 weights: tcgen05 GEMM (gemm_tc.cu).
  if (int8_weights) {
    bool tc_ok = false;
    const size_t tc_ws = sg::gemm_tc_scratch_bytes(p, true, &tc_ok);
    if (tc_ok) {
      void* ws = p->workspace;
      size_t ws_bytes = p->workspace_bytes;
      if (ws == nullptr && tc_ws > 0) {
        st = sg::library_workspace(stream, tc_ws, &ws, sg::kWsPrefillGemm);
        if (st != SG_OK) return st;
        ws_bytes = tc_ws;
      }
      int* err = nullptr;
      st = sg::device_error_word(&err);
      if (st != SG_OK) return st;
      bool handled = false;
      st = sg::gemm_tc_run(p, true, cs, sg::sm_count(dev), ws, ws_bytes, err, &handled);
      if (handled || st != SG_OK) return st;
    }
  }
  // One float activation row: the int8 tensor-core GEMV when a cluster split fills the GPU.
  if (kind == W_INT8_FA && p->M == 1 && p->bias == nullptr) {
    int* err = nullptr;
    st = sg::device_error_word(&err);
    if (st != SG_OK) return st;
    bool handled = false;
    st = sg::w8_gemv_mma_run(p, cs, sg::sm_count(dev), err, &handled);
    if (handled || st != SG_OK) return st;
  }
  const Plan pl = make_plan(kind, p, sg::sm_count(dev));
  if (!pl.fast) {
    dim3 grid((p->N + 127) / 128, p->M);
    switch (kind) {
      case W_INT8_IA: dense_gemv_generic_kernel<W_INT8_IA><<<grid, 128, 0, cs>>>(a); break;
      case W_INT8_FA: dense_gemv_generic_kernel<W_INT8_FA><<<grid, 128, 0, cs>>>(a); break;
      default: dense_gemv_generic_kernel<W_F16><<<grid, 128, 0, cs>>>(a); break;
    }
    return sg::check_launch(name);
  }
  a.rows_per_split = pl.rows_per_split;
  a.ksplit = pl.ksplit;
  a.ring_off = pl.ring_off;
  if (kind != W_F16) {  // the int8 rings need the shared-memory opt-in (once per kernel and device)
    static std::atomic<uint64_t> attr_set[2] = {};
    const int ki = kind == W_INT8_IA ? 0 : 1;
    const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
    if (!(attr_set[ki].load() & bit)) {
      auto kfn = kind == W_INT8_IA ? dense_gemv_kernel<W_INT8_IA> : dense_gemv_kernel<W_INT8_FA>;
      const cudaError_t ae = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - 2048);
      if (ae != cudaSuccess) {
        cudaGetLastError();
        sg::set_error("%s: cudaFuncSetAttribute failed: %s", name, cudaGetErrorString(ae));
        return SG_ERR_RUNTIME;
      }
      attr_set[ki].fetch_or(bit);
    }
  }
  if (pl.ksplit > 1) {
    void* ws = p->workspace;
    if (ws == nullptr) {
      st = sg::library_workspace(stream, pl.ws_bytes, &ws, sg::kWsDenseGemv);
      if (st != SG_OK) return st;
    } else {
      SG_CHECK_ARG(p->workspace_bytes >= pl.ws_bytes && sg::aligned16(ws),
                   "%s: workspace too small or unaligned (%zu < %zu bytes)", name, p->workspace_bytes,
                   pl.ws_bytes);
    }
    a.tickets = static_cast<unsigned*>(ws);
    a.partial = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.tickets_bytes);
  }
  dim3 grid(pl.n_tiles, pl.ksplit);
  for (int m = 0; m < p->M; ++m) {
    DArgs ar = a;
    ar.M = 1;
    ar.A = static_cast<const char*>(p->A) + (size_t)m * a.lda * sg::elem_size(a.a_dt);
    ar.C = static_cast<char*>(p->C) + (size_t)m * a.ldc * sg::elem_size(a.c_dt);
    switch (kind) {
      case W_INT8_IA: dense_gemv_kernel<W_INT8_IA><<<grid, kI8Warps * 32, pl.smem, cs>>>(ar); break;
      case W_INT8_FA: dense_gemv_kernel<W_INT8_FA><<<grid, kI8Warps * 32, pl.smem, cs>>>(ar); break;
      default: dense_gemv_kernel<W_F16><<<grid, kThreads, pl.smem, cs>>>(ar); break;
    }
    st = sg::check_launch(name);
    if (st != SG_OK) return st;
  }
  return SG_OK;
}

size_t dense_ws(const SgMatMulParams* p, bool int8_weights) {
  if (validate("workspace_size", p, int8_weights) != SG_OK || p->M == 0 || p->N == 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = 0;
  }
  if (int8_weights) {
    bool tc_ok = false;
    const size_t tws = sg::gemm_tc_scratch_bytes(p, true, &tc_ok);
    if (tc_ok) return tws;
  }
  const int adt = p->a_dtype == SG_DT_DEFAULT ? (int8_weights ? SG_DT_I8 : SG_DT_F16) : p->a_dtype;
  return make_plan(kind_of(int8_weights, adt), p, sg::sm_count(dev)).ws_bytes;
}

}  // namespace

extern "C" {

SgStatus sg_matmul_int8_channel(const SgMatMulParams* p, void* stream) {
  return dense_run("sg_matmul_int8_channel", p, stream, true);
}
size_t sg_matmul_int8_channel_workspace_size(const SgMatMulParams* p) { return dense_ws(p, true); }

SgStatus sg_matmul_fp16(const SgMatMulParams* p, void* stream) {
  return dense_run("sg_matmul_fp16", p, stream, false);
}
size_t sg_matmul_fp16_workspace_size(const SgMatMulParams* p) { return dense_ws(p, false); }

}  // extern "C"
