// INT4 group-quantised dequant GEMV (decode) for sm_100a.
//
// Replaces the reference's matmul_int4_grouped_neon
// (compiler/kernels/cpu/matmul_neon.h:113-148) and keeps its weight layout:
//   B       u8  [ceil(K/2), N]  byte (k/2)*N + n, low nibble = even k   (:127)
//   scales  f16 [ceil(K/gs), N]                                          (:132)
//   zeros   i8  [ceil(K/gs), N] in [-8, 7], or none                      (:133)
//   C[m,n] = sum_k A[m,k] * scale * ((nibble - 8) - zero)                (:128-139)
//
// Fast path (N % 16 == 0, group_size % 16 == 0, 16-byte aligned operands):
//   * HBM layout is consumed as stored: a lane owns 16 consecutive columns and
//     streams k-pair rows with one 128-bit load per row, so a warp reads 512
//     contiguous bytes of a row (four full 128-byte lines).
//   * Nibbles become exact fp32 integers in registers: (word & (0xF << 4p)) |
//     0x4B000000 is the float 2^23 + q*16^p (one LOP3), and a packed
//     fma.rn.f32x2 with (16^-p, -2^23*16^-p) yields q exactly.  A second packed
//     FMA accumulates x*q for two columns.  No x rounding: activations stay fp32.
//   * Per (group, column) the zero point and scale are applied once:
//     acc += scale * (sum_k x_k q_k - (8 + zero) * sum_k x_k).
//   * 8 warps of a block split the block's groups; blocks split K further
//     (split-K).  Partials go to scratch; the last block to finish a column
//     tile (atomic ticket) reduces them in fixed split order, so results are
//     deterministic, and resets its ticket so the scratch stays zero-filled.
// Generic path (any shape): one thread per output running the reference's
// sequential loop with explicit round-to-nearest mul/add, bit-identical to
// the reference arithmetic for every activation dtype.
#include <algorithm>
#include <atomic>
#include <string_view>

#include "sm100.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kColsPerLane = 16;
constexpr int kColsPerBlock = 32 * kColsPerLane;  // 512
constexpr int kRowsPerChunk = 8;
constexpr int kMaxRowsPerLaunch = 4;

std::atomic<int> g_tune_groups_per_warp{0};  // 0 = heuristic
std::atomic<int> g_tune_path{0};              // 0 = auto, 1 = CUDA-core kernel, 2 = generic kernel
std::atomic<int> g_tune_rows_two_pass{32};    // most rows taken by the few-row kernel (two passes above 16)

struct W4Args {
  const void* A;
  const uint8_t* B;
  const __half* scales;
  const int8_t* zeros;
  const __half* bias;
  void* C;
  int M, K, N, lda, ldc, gs, G, KP;
  int a_dt, c_dt;
  float scale_A;
  int groups_per_split, ksplit;
  float* partial;      // [ksplit][M][N]
  unsigned* tickets;   // [n_tiles]
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

__device__ __forceinline__ float finalize(const W4Args& a, int col, float v) {
  if (a.a_dt == SG_DT_I8) v = v * a.scale_A;
  if (a.bias) v = v + __half2float(a.bias[col]);
  return v;
}

// One word = 4 columns of one k-pair row.  Pairs (c0,c2) and (c1,c3).
__device__ __forceinline__ void dequant_word(uint32_t w, float2& e02, float2& o02, float2& e13,
                                             float2& o13) {
  constexpr uint32_t MAGIC = 0x4B000000u;  // 2^23
  const float f0 = __uint_as_float(sgd::lop3_and_or(w, 0x0000000Fu, MAGIC));  // c0 even, 16^0
  const float f1 = __uint_as_float(sgd::lop3_and_or(w, 0x000000F0u, MAGIC));  // c0 odd , 16^1
  const float f2 = __uint_as_float(sgd::lop3_and_or(w, 0x00000F00u, MAGIC));  // c1 even, 16^2
  const float f3 = __uint_as_float(sgd::lop3_and_or(w, 0x0000F000u, MAGIC));  // c1 odd , 16^3
  const float f4 = __uint_as_float(sgd::lop3_and_or(w, 0x000F0000u, MAGIC));  // c2 even, 16^4
  const uint32_t w2 = w >> 12;
  const float f5 = __uint_as_float(sgd::lop3_and_or(w2, 0x00000F00u, MAGIC));  // c2 odd , 16^2
  const float f6 = __uint_as_float(sgd::lop3_and_or(w2, 0x0000F000u, MAGIC));  // c3 even, 16^3
  const float f7 = __uint_as_float(sgd::lop3_and_or(w2, 0x000F0000u, MAGIC));  // c3 odd , 16^4
  constexpr float P0 = 1.0f, P1 = 1.0f / 16, P2 = 1.0f / 256, P3 = 1.0f / 4096, P4 = 1.0f / 65536;
  constexpr float T = 8388608.0f;
  e02 = sgd::ffma2(make_float2(f0, f4), make_float2(P0, P4), make_float2(-T * P0, -T * P4));
  o02 = sgd::ffma2(make_float2(f1, f5), make_float2(P1, P2), make_float2(-T * P1, -T * P2));
  e13 = sgd::ffma2(make_float2(f2, f6), make_float2(P2, P3), make_float2(-T * P2, -T * P3));
  o13 = sgd::ffma2(make_float2(f3, f7), make_float2(P3, P4), make_float2(-T * P3, -T * P4));
}

template <int MR>
__global__ void __launch_bounds__(kThreads, (MR >= 4 ? 1 : 2)) w4_gemv_fast_kernel(W4Args a) {
  extern __shared__ float4 smem4[];
  const int tile = blockIdx.x;
  const int split = blockIdx.y;
  const int g_begin = split * a.groups_per_split;
  const int g_end = min(a.G, g_begin + a.groups_per_split);
  const int ng = g_end - g_begin;
  const int rows_per_group = a.gs >> 1;
  const int rows_blk = ng * rows_per_group;
  const int k_begin = g_begin * a.gs;

  // ---- stage x for this block's k range: float4 (xe, xe, xo, xo) per k-pair row
  float4* xs = smem4;                                     // [MR][rows_blk]
  float* xg = reinterpret_cast<float*>(xs + MR * rows_blk);  // [MR][ng] group sums
  for (int i = threadIdx.x; i < MR * rows_blk; i += kThreads) {
    const int m = i / rows_blk, r = i - m * rows_blk;
    const int k = k_begin + 2 * r;
    float xe = 0.f, xo = 0.f;
    if (m < a.M) {
      if (k < a.K) xe = load_act(a.A, a.a_dt, (int64_t)m * a.lda + k);
      if (k + 1 < a.K) xo = load_act(a.A, a.a_dt, (int64_t)m * a.lda + k + 1);
    }
    xs[i] = make_float4(xe, xe, xo, xo);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < MR * ng; i += kThreads) {
    const int m = i / ng, gl = i - m * ng;
    const float4* xr = xs + m * rows_blk + gl * rows_per_group;
    float s = 0.f;
    for (int r = 0; r < rows_per_group; ++r) s += xr[r].x + xr[r].z;
    xg[i] = s;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col0 = tile * kColsPerBlock + lane * kColsPerLane;
  const bool col_ok = col0 < a.N;

  float acc[MR][16];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int c = 0; c < 16; ++c) acc[m][c] = 0.f;

  if (col_ok) {
    const uint8_t* Bcol = a.B + col0;
    for (int gl = warp; gl < ng; gl += kWarps) {
      const int g = g_begin + gl;
      float2 pacc[MR][8];
#pragma unroll
      for (int m = 0; m < MR; ++m)
#pragma unroll
        for (int j = 0; j < 8; ++j) pacc[m][j] = make_float2(0.f, 0.f);

      const int row_g0 = g * rows_per_group;
      for (int ch = 0; ch < rows_per_group; ch += kRowsPerChunk) {
        uint4 wv[kRowsPerChunk];
#pragma unroll
        for (int r = 0; r < kRowsPerChunk; ++r) {
          const int row = row_g0 + ch + r;
          wv[r] = (row < a.KP) ? sgd::ldg_stream(Bcol + (int64_t)row * a.N)
                               : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int r = 0; r < kRowsPerChunk; ++r) {
          const uint32_t words[4] = {wv[r].x, wv[r].y, wv[r].z, wv[r].w};
          float4 xq[MR];
#pragma unroll
          for (int m = 0; m < MR; ++m) xq[m] = xs[m * rows_blk + gl * rows_per_group + ch + r];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float2 e02, o02, e13, o13;
            dequant_word(words[q], e02, o02, e13, o13);
#pragma unroll
            for (int m = 0; m < MR; ++m) {
              const float2 xe = make_float2(xq[m].x, xq[m].y);
              const float2 xo = make_float2(xq[m].z, xq[m].w);
              pacc[m][2 * q] = sgd::ffma2(e02, xe, pacc[m][2 * q]);
              pacc[m][2 * q] = sgd::ffma2(o02, xo, pacc[m][2 * q]);
              pacc[m][2 * q + 1] = sgd::ffma2(e13, xe, pacc[m][2 * q + 1]);
              pacc[m][2 * q + 1] = sgd::ffma2(o13, xo, pacc[m][2 * q + 1]);
            }
          }
        }
      }
      // ---- group epilogue: scale and zero point, once per (group, column)
      float xsum[MR];
#pragma unroll
      for (int m = 0; m < MR; ++m) xsum[m] = xg[m * ng + gl];
      const uint4 s_lo = *reinterpret_cast<const uint4*>(a.scales + (int64_t)g * a.N + col0);
      const uint4 s_hi = *reinterpret_cast<const uint4*>(a.scales + (int64_t)g * a.N + col0 + 8);
      const __half* sh_lo = reinterpret_cast<const __half*>(&s_lo);
      const __half* sh_hi = reinterpret_cast<const __half*>(&s_hi);
      uint4 zv = make_uint4(0u, 0u, 0u, 0u);
      if (a.zeros) zv = *reinterpret_cast<const uint4*>(a.zeros + (int64_t)g * a.N + col0);
      const int8_t* zb = reinterpret_cast<const int8_t*>(&zv);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int c = 4 * q + b;
          const float s = __half2float(c < 8 ? sh_lo[c] : sh_hi[c - 8]);
          const float zc = 8.0f + (float)zb[c];
          // pair index: (c0,c2) -> 2q (x = c0, y = c2); (c1,c3) -> 2q+1
          const int pi = 2 * q + (b & 1);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            const float sxq = (b < 2) ? pacc[m][pi].x : pacc[m][pi].y;
            acc[m][c] = fmaf(s, fmaf(-zc, xsum[m], sxq), acc[m][c]);
          }
        }
      }
    }
  }

  // ---- reduce the 8 warps of the block (fixed order), then split-K
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem4);  // [kWarps][512]
  __shared__ bool s_last;
  for (int m = 0; m < MR; ++m) {
    if (col_ok) {
      float4* dst = reinterpret_cast<float4*>(red + warp * kColsPerBlock + lane * kColsPerLane);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        dst[j] = make_float4(acc[m][4 * j], acc[m][4 * j + 1], acc[m][4 * j + 2], acc[m][4 * j + 3]);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < kColsPerBlock; c += kThreads) {
      const int col = tile * kColsPerBlock + c;
      if (col < a.N && m < a.M) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[w * kColsPerBlock + c];
        if (a.ksplit == 1) {
          store_out(a.C, a.c_dt, (int64_t)m * a.ldc + col, finalize(a, col, v));
        } else {
          a.partial[((int64_t)split * a.M + m) * a.N + col] = v;
        }
      }
    }
    __syncthreads();
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
  for (int i = threadIdx.x; i < MR * kColsPerBlock; i += kThreads) {
    const int m = i / kColsPerBlock, c = i - m * kColsPerBlock;
    const int col = tile * kColsPerBlock + c;
    if (m >= a.M || col >= a.N) continue;
    float v = 0.f;
    for (int sp = 0; sp < a.ksplit; ++sp) v += __ldcg(&a.partial[((int64_t)sp * a.M + m) * a.N + col]);
    store_out(a.C, a.c_dt, (int64_t)m * a.ldc + col, finalize(a, col, v));
  }
  if (threadIdx.x == 0) a.tickets[tile] = 0u;
}

// Reference-order loop, one thread per output (any shape / alignment).
__global__ void w4_gemv_generic_kernel(W4Args a) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= a.N || m >= a.M) return;
  float acc = 0.0f;
  for (int k = 0; k < a.K; k += 2) {
    const uint8_t packed = a.B[(int64_t)(k / 2) * a.N + n];
    const int w0 = (int)(packed & 0x0F) - 8;
    const int w1 = (int)(packed >> 4) - 8;
    const int group = k / a.gs;
    const float scale = __half2float(a.scales[(int64_t)group * a.N + n]);
    const int zero = a.zeros ? (int)a.zeros[(int64_t)group * a.N + n] : 0;
    const float w0f = __fmul_rn(scale, (float)(w0 - zero));
    const float w1f = __fmul_rn(scale, (float)(w1 - zero));
    acc = __fadd_rn(acc, __fmul_rn(load_act(a.A, a.a_dt, (int64_t)m * a.lda + k), w0f));
    acc = __fadd_rn(acc, (k + 1 < a.K)
                             ? __fmul_rn(load_act(a.A, a.a_dt, (int64_t)m * a.lda + k + 1), w1f)
                             : 0.0f);
  }
  if (a.a_dt == SG_DT_I8) acc = __fmul_rn(acc, a.scale_A);
  if (a.bias) acc = __fadd_rn(acc, __half2float(a.bias[n]));
  store_out(a.C, a.c_dt, (int64_t)m * a.ldc + n, acc);
}

struct Plan {
  bool fast = false;
  int rows_per_launch = 1;
  int groups_per_split = 0;
  int ksplit = 1;
  int n_tiles = 0;
  size_t smem = 0;
  size_t ws_bytes = 0;
  size_t tickets_bytes = 0;
};

SgStatus validate(const SgMatMulParams* p) {
  SG_CHECK_ARG(p != nullptr, "sg_matmul_int4_grouped: params is NULL");
  SG_CHECK_ARG(p->M >= 0 && p->K >= 0 && p->N >= 0, "sg_matmul_int4_grouped: negative size M=%d K=%d N=%d",
               p->M, p->K, p->N);
  if (p->M == 0 || p->N == 0) return SG_OK;
  SG_CHECK_ARG(p->C, "sg_matmul_int4_grouped: C must be non-NULL");
  SG_CHECK_ARG(p->K == 0 || (p->A && p->B && p->scales_B),
               "sg_matmul_int4_grouped: A, B and scales_B must be non-NULL");
  SG_CHECK_ARG(p->ldb <= 0 || p->ldb == p->N, "sg_matmul_int4_grouped: ldb must be N (got %d)", p->ldb);
  SG_CHECK_ARG(p->lda <= 0 || p->lda >= p->K, "sg_matmul_int4_grouped: lda %d < K %d", p->lda, p->K);
  SG_CHECK_ARG(p->ldc <= 0 || p->ldc >= p->N, "sg_matmul_int4_grouped: ldc %d < N %d", p->ldc, p->N);
  const int adt = p->a_dtype == SG_DT_DEFAULT ? SG_DT_I8 : p->a_dtype;
  const int cdt = p->c_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->c_dtype;
  SG_CHECK_ARG(adt >= SG_DT_F32 && adt <= SG_DT_I8, "sg_matmul_int4_grouped: bad a_dtype %d", p->a_dtype);
  if (p->flags & SG_MM_A_SWIGLU) {
    SG_CHECK_ARG(adt == SG_DT_F16 || adt == SG_DT_BF16, "sg_matmul_int4_grouped: SG_MM_A_SWIGLU needs fp16 or bf16 A");
    SG_CHECK_ARG(p->lda <= 0 || p->lda >= 2 * p->K, "sg_matmul_int4_grouped: SG_MM_A_SWIGLU needs lda >= 2K (got %d)",
                 p->lda);
  }
  SG_CHECK_ARG(cdt == SG_DT_F32 || cdt == SG_DT_F16 || cdt == SG_DT_BF16,
               "sg_matmul_int4_grouped: bad c_dtype %d", p->c_dtype);
  if (p->flags & SG_MM_A_RMSNORM) {
    SG_CHECK_ARG((adt == SG_DT_F16 || adt == SG_DT_BF16) && p->norm_weight && p->K % 8 == 0 && p->K <= 8192 &&
                     sg::aligned16(p->A) && sg::aligned16(p->norm_weight) && !(p->flags & SG_MM_A_SWIGLU),
                 "sg_matmul_int4_grouped: SG_MM_A_RMSNORM needs a 16-bit, 16-byte aligned A row of K %% 8 == 0 "
                 "<= 8192 values, a norm_weight, and no SG_MM_A_SWIGLU");
  }
  if (p->flags & SG_MM_C_ACCUMULATE) {
    SG_CHECK_ARG(cdt == SG_DT_F16 || cdt == SG_DT_BF16, "sg_matmul_int4_grouped: SG_MM_C_ACCUMULATE needs a 16-bit C");
  }
  return SG_OK;
}

Plan make_plan(const SgMatMulParams* p, int sms) {
  Plan pl;
  const int gs = p->group_size > 0 ? p->group_size : 128;
  const int G = (p->K + gs - 1) / gs;
  const bool fast = (p->K > 0) && (p->N % 16 == 0) && (gs % 16 == 0) && sg::aligned16(p->B) &&
                    sg::aligned16(p->scales_B) && (p->zeros_B == nullptr || sg::aligned16(p->zeros_B));
  pl.fast = fast;
  if (!fast) return pl;
  pl.rows_per_launch = std::min(p->M, kMaxRowsPerLaunch);
  pl.n_tiles = (p->N + kColsPerBlock - 1) / kColsPerBlock;
  int gpw = g_tune_groups_per_warp.load();
  if (gpw <= 0) {
    // Aim for about four resident blocks' worth of work per SM.
    const long units = (long)pl.n_tiles * G;  // (column tile, group) units, one warp each
    const long target_warps = (long)sms * 4 * kWarps;
    gpw = (int)std::max<long>(1, units / target_warps);
    // Long groups already give each warp plenty of rows.
    if (gs >= 128) gpw = std::max(1, gpw / 2);
  }
  const int MR = pl.rows_per_launch == 3 ? 4 : pl.rows_per_launch;
  size_t xs_bytes = 0;
  for (;;) {
    pl.groups_per_split = kWarps * gpw;
    pl.ksplit = (G + pl.groups_per_split - 1) / pl.groups_per_split;
    if (pl.ksplit == 1) pl.groups_per_split = G;
    const int rows_blk = pl.groups_per_split * (gs / 2);
    xs_bytes = (size_t)MR * rows_blk * sizeof(float4) + (size_t)MR * pl.groups_per_split * 4;
    if (xs_bytes <= 96 * 1024 || gpw == 1) break;
    gpw = std::max(1, gpw / 2);
  }
  if (xs_bytes > 200 * 1024) {  // very large groups: leave them to the generic kernel
    pl.fast = false;
    return pl;
  }
  const size_t red_bytes = (size_t)kWarps * kColsPerBlock * sizeof(float);
  pl.smem = std::max(xs_bytes, red_bytes);
  if (pl.ksplit > 1) {
    pl.tickets_bytes = sg::ticket_bytes(pl.n_tiles);
    pl.ws_bytes = pl.tickets_bytes + (size_t)pl.ksplit * MR * p->N * sizeof(float);
  }
  return pl;
}

template <int MR>
SgStatus launch_fast(const W4Args& a, const Plan& pl, cudaStream_t st) {
  auto kfn = w4_gemv_fast_kernel<MR>;
  if (pl.smem > 48 * 1024) {
    SG_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem));
  }
  dim3 grid(pl.n_tiles, pl.ksplit);
  kfn<<<grid, kThreads, pl.smem, st>>>(a);
  return sg::check_launch("w4_gemv_fast_kernel");
}

}  // namespace

namespace sg {
size_t w4_gemv_mma_scratch_bytes(const SgMatMulParams* p, int sms, bool* applicable);
SgStatus w4_gemv_mma_run(const SgMatMulParams* p, cudaStream_t cs, int sms, void* ws, size_t ws_bytes,
                         int* err_word, bool* handled, const SgRopeAppend* rope = nullptr);
bool w4_gemv_mma_tuning(std::string_view key, int value);
bool w8_gemv_mma_tuning(std::string_view key, int value);
SgStatus w4_rows_run(const SgMatMulParams* p, cudaStream_t cs, int sms, int* err_word, bool* handled);
bool w4_rows_tuning(std::string_view key, int value);
bool gemm_tc_tuning(std::string_view key, int value);
bool attn_tc_tuning(std::string_view key, int value);
bool attn_tuning(std::string_view key, int value);
bool sdk_tuning(std::string_view key, int value);
bool tp_allreduce_tuning(std::string_view key, int value);
}  // namespace sg

// Core entry.  ws == NULL: library scratch (unless ws_external, then an error
// if scratch is needed).  err_word == NULL: the library's per-device error word.
static SgStatus w4_run(const SgMatMulParams* p, void* stream, void* ws, size_t ws_bytes,
                       bool ws_external, int* err_word) {
  SgStatus st = validate(p);
  if (st != SG_OK) return st;
  if (p->M == 0 || p->N == 0) return SG_OK;
  int dev = 0;
  st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  const int sms = sg::sm_count(dev);
  cudaStream_t cs = static_cast<cudaStream_t>(stream);

  W4Args a{};
  a.A = p->A;
  a.B = static_cast<const uint8_t*>(p->B);
  a.scales = static_cast<const __half*>(p->scales_B);
  a.zeros = p->zeros_B;
  a.bias = static_cast<const __half*>(p->bias);
  a.C = p->C;
  a.M = p->M;
  a.K = p->K;
  a.N = p->N;
  a.lda = p->lda > 0 ? p->lda : p->K;
  a.ldc = p->ldc > 0 ? p->ldc : p->N;
  a.gs = p->group_size > 0 ? p->group_size : 128;
  a.G = (p->K + a.gs - 1) / a.gs;
  a.KP = (p->K + 1) / 2;
  a.a_dt = p->a_dtype == SG_DT_DEFAULT ? SG_DT_I8 : p->a_dtype;
  a.c_dt = p->c_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->c_dtype;
  a.scale_A = p->scale_A;

  const int path = g_tune_path.load();
  // 2..16 activation rows (batched decode): fp16-dequant mma.sync GEMM (w4_gemm_rows.cu);
  // up to g_tune_rows_two_pass rows as two passes of at most 16 rows over the same
  // weights (the second pass reads them mostly from L2).  Measured on B200 at 24-32 rows
  // (Qwen-7B shapes, g128): q|k|v 30.2 -> 19.7 us, o 30.6 -> 15.4, gate|up 58.3 -> 54.7,
  // LM head 244 -> 203 against the tcgen05 GEMM, whose 128-row tiles are mostly empty there.
  const bool fused_norm = (p->flags & (SG_MM_A_RMSNORM | SG_MM_C_ACCUMULATE)) != 0;  // one-row kernel only
  if (path == 0 && !fused_norm && p->M >= 2 && p->M <= std::max(16, g_tune_rows_two_pass.load())) {
    if (err_word == nullptr) {
      st = sg::device_error_word(&err_word);
      if (st != SG_OK) return st;
    }
    bool handled = false;
    if (p->M <= 16) {
      st = sg::w4_rows_run(p, cs, sms, err_word, &handled);
      if (handled || st != SG_OK) return st;
    } else {
      SgMatMulParams q = *p;
      q.M = 16;
      st = sg::w4_rows_run(&q, cs, sms, err_word, &handled);
      if (st != SG_OK) return st;
      if (handled) {
        const int64_t lda = p->lda > 0 ? p->lda : ((p->flags & SG_MM_A_SWIGLU) ? 2 * p->K : p->K);
        const int64_t ldc = p->ldc > 0 ? p->ldc : p->N;
        SgMatMulParams r = *p;
        r.M = p->M - 16;
        r.A = static_cast<const char*>(p->A) + 16 * lda * sg::elem_size(a.a_dt);
        r.C = static_cast<char*>(p->C) + 16 * ldc * sg::elem_size(a.c_dt);
        handled = false;
        st = sg::w4_rows_run(&r, cs, sms, err_word, &handled);
        if (handled || st != SG_OK) return st;
      }
      // otherwise a path below computes all M rows
    }
  }
  const bool swiglu = (p->flags & SG_MM_A_SWIGLU) != 0;
  // Many activation rows: tcgen05 GEMM with the weights dequantized into TMEM (gemm_tc.cu).
  bool tc_ok = false;
  const size_t tc_ws = path == 0 && !swiglu && !fused_norm ? sg::gemm_tc_scratch_bytes(p, false, &tc_ok) : 0;
  if (tc_ok) {
    if (ws == nullptr && tc_ws > 0) {
      if (ws_external) {
        sg::set_error("sg_matmul_int4_grouped: scratch required (%zu bytes)", tc_ws);
        return SG_ERR_INVALID;
      }
      st = sg::library_workspace(stream, tc_ws, &ws, sg::kWsPrefillGemm);
      if (st != SG_OK) return st;
      ws_bytes = tc_ws;
    }
    if (err_word == nullptr) {
      st = sg::device_error_word(&err_word);
      if (st != SG_OK) return st;
    }
    bool handled = false;
    st = sg::gemm_tc_run(p, false, cs, sms, ws, ws_bytes, err_word, &handled);
    if (handled || st != SG_OK) return st;
  }
  // One activation row and groups of 32k: tensor-core reduction (w4_gemv_mma.cu).
  bool mma_ok = false;
  const size_t mma_ws = sg::w4_gemv_mma_scratch_bytes(p, sms, &mma_ok);
  if (mma_ok && path == 0) {
    if (ws == nullptr && mma_ws > 0) {
      if (ws_external) {
        sg::set_error("sg_matmul_int4_grouped: scratch required (%zu bytes)", mma_ws);
        return SG_ERR_INVALID;
      }
      st = sg::library_workspace(stream, mma_ws, &ws, sg::kWsInt4Gemv);
      if (st != SG_OK) return st;
      ws_bytes = mma_ws;
    }
    if (err_word == nullptr) {
      st = sg::device_error_word(&err_word);
      if (st != SG_OK) return st;
    }
    bool handled = false;
    st = sg::w4_gemv_mma_run(p, cs, sms, ws, ws_bytes, err_word, &handled);
    if (handled || st != SG_OK) return st;
  }
  if (swiglu) {
    sg::set_error("sg_matmul_int4_grouped: SG_MM_A_SWIGLU is fused only on the one-row and 2..16-row kernels "
                  "(M=%d K=%d N=%d group %d)", p->M, p->K, p->N, p->group_size);
    return SG_ERR_UNSUPPORTED;
  }
  if (p->flags & (SG_MM_A_RMSNORM | SG_MM_C_ACCUMULATE)) {
    sg::set_error("sg_matmul_int4_grouped: SG_MM_A_RMSNORM / SG_MM_C_ACCUMULATE are fused only on the one-row "
                  "tensor-core kernel (M=%d K=%d N=%d group %d)", p->M, p->K, p->N, p->group_size);
    return SG_ERR_UNSUPPORTED;
  }

  Plan pl = make_plan(p, sms);
  if (path == 2) pl.fast = false;
  if (!pl.fast) {
    dim3 grid((p->N + 127) / 128, p->M);
    w4_gemv_generic_kernel<<<grid, 128, 0, cs>>>(a);
    return sg::check_launch("w4_gemv_generic_kernel");
  }
  a.groups_per_split = pl.groups_per_split;
  a.ksplit = pl.ksplit;
  if (pl.ksplit > 1) {
    if (ws == nullptr) {
      if (ws_external) {
        sg::set_error("sg_matmul_int4_grouped: scratch required (%zu bytes)", pl.ws_bytes);
        return SG_ERR_INVALID;
      }
      st = sg::library_workspace(stream, pl.ws_bytes, &ws, sg::kWsInt4Gemv);
      if (st != SG_OK) return st;
    } else {
      SG_CHECK_ARG(ws_bytes >= pl.ws_bytes && sg::aligned16(ws),
                   "sg_matmul_int4_grouped: workspace too small or unaligned (%zu < %zu bytes)",
                   ws_bytes, pl.ws_bytes);
    }
    a.tickets = static_cast<unsigned*>(ws);
    a.partial = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.tickets_bytes);
  }
  // Rows are processed kMaxRowsPerLaunch at a time (each launch re-streams B).
  for (int m0 = 0; m0 < p->M; m0 += kMaxRowsPerLaunch) {
    W4Args ar = a;
    const int rows = std::min(kMaxRowsPerLaunch, p->M - m0);
    ar.M = rows;
    ar.A = static_cast<const char*>(p->A) + (size_t)m0 * a.lda * sg::elem_size(a.a_dt);
    ar.C = static_cast<char*>(p->C) + (size_t)m0 * a.ldc * sg::elem_size(a.c_dt);
    switch (rows) {
      case 1: st = launch_fast<1>(ar, pl, cs); break;
      case 2: st = launch_fast<2>(ar, pl, cs); break;
      default: st = launch_fast<4>(ar, pl, cs); break;
    }
    if (st != SG_OK) return st;
  }
  return SG_OK;
}

namespace sg {
// Entry with caller-chosen scratch and error word (see w4_run).
SgStatus w4_gemv_run(const SgMatMulParams* p, void* stream, void* ws, size_t ws_bytes, bool ws_external,
                     int* err_word) {
  return w4_run(p, stream, ws, ws_bytes, ws_external, err_word);
}
size_t w4_gemv_scratch_bytes(const SgMatMulParams* p, bool minimal) {
  if (validate(p) != SG_OK || p->M == 0 || p->N == 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = 0;
  }
  const int sms = sm_count(dev);
  const int path = g_tune_path.load();
  bool tc_ok = false;
  const size_t tws = gemm_tc_scratch_bytes(p, false, &tc_ok, minimal);
  if (tc_ok && path == 0) return tws;
  bool mma_ok = false;
  const size_t mws = w4_gemv_mma_scratch_bytes(p, sms, &mma_ok);
  if (mma_ok && path == 0) return mws;
  if (path == 2) return 0;
  return make_plan(p, sms).ws_bytes;
}
}  // namespace sg

extern "C" {

SgStatus sg_qkv_gemv_rope_append(const SgMatMulParams* p, const SgRopeAppend* r, void* stream) {
  SgStatus st = validate(p);
  if (st != SG_OK) return st;
  SG_CHECK_ARG(r != nullptr, "sg_qkv_gemv_rope_append: rope is NULL");
  SG_CHECK_ARG(p->M == 1, "sg_qkv_gemv_rope_append: one row only (M=%d)", p->M);
  SG_CHECK_ARG(r->heads > 0 && r->kv_heads > 0 && (r->head_dim == 64 || r->head_dim == 128) &&
                   p->N == (r->heads + 2 * r->kv_heads) * r->head_dim,
               "sg_qkv_gemv_rope_append: N must be (heads + 2 kv_heads) * head_dim with head_dim 64 or 128");
  const int cdt = p->c_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->c_dtype;
  SG_CHECK_ARG(cdt == SG_DT_F16 || cdt == SG_DT_BF16, "sg_qkv_gemv_rope_append: 16-bit output only");
  SG_CHECK_ARG(r->q_out && r->k_cache && r->v_cache, "sg_qkv_gemv_rope_append: NULL q / k / v");
  SG_CHECK_ARG(!(p->flags & SG_MM_C_ACCUMULATE), "sg_qkv_gemv_rope_append: SG_MM_C_ACCUMULATE does not apply");
  if (r->kv_pages) {
    SG_CHECK_ARG(r->kv_pages->table && r->kv_pages->page_size == 16 && r->kv_pages->num_pages > 0,
                 "sg_qkv_gemv_rope_append: bad SgKvPages");
  } else {
    SG_CHECK_ARG(r->kv_head_stride >= r->head_dim, "sg_qkv_gemv_rope_append: kv_head_stride < head_dim");
  }
  int dev = 0;
  st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  int* err = nullptr;
  st = sg::device_error_word(&err);
  if (st != SG_OK) return st;
  bool handled = false;
  st = sg::w4_gemv_mma_run(p, static_cast<cudaStream_t>(stream), sg::sm_count(dev), nullptr, 0, err, &handled, r);
  if (st != SG_OK) return st;
  if (!handled) {
    sg::set_error("sg_qkv_gemv_rope_append: the one-row kernel does not take K=%d N=%d group %d with a cluster "
                  "split; use sg_matmul_int4_grouped and sg_qkv_rope_append", p->K, p->N, p->group_size);
    return SG_ERR_UNSUPPORTED;
  }
  return SG_OK;
}

SgStatus sg_matmul_int4_grouped(const SgMatMulParams* p, void* stream) {
  if (p && p->workspace) return w4_run(p, stream, p->workspace, p->workspace_bytes, true, nullptr);
  return w4_run(p, stream, nullptr, 0, false, nullptr);
}

size_t sg_matmul_int4_grouped_workspace_size(const SgMatMulParams* p) {
  return sg::w4_gemv_scratch_bytes(p, false);
}

int32_t sg_set_tuning(const char* key, int32_t value) {
  if (key && std::string_view(key) == "w4_rows.two_pass_rows") {
    g_tune_rows_two_pass.store(value);
    return SG_OK;
  }
  if (key && std::string_view(key) == "w4_gemv.groups_per_warp") {
    g_tune_groups_per_warp.store(value);
    return SG_OK;
  }
  if (key && std::string_view(key) == "w4_gemv.path") {
    g_tune_path.store(value);
    return SG_OK;
  }
  if (key && sg::w4_gemv_mma_tuning(std::string_view(key), value)) return SG_OK;
  if (key && sg::w8_gemv_mma_tuning(std::string_view(key), value)) return SG_OK;
  if (key && sg::w4_rows_tuning(std::string_view(key), value)) return SG_OK;
  if (key && sg::gemm_tc_tuning(std::string_view(key), value)) return SG_OK;
  if (key && sg::attn_tc_tuning(std::string_view(key), value)) return SG_OK;
  if (key && sg::attn_tuning(std::string_view(key), value)) return SG_OK;
  if (key && sg::sdk_tuning(std::string_view(key), value)) return SG_OK;
  if (key && sg::tp_allreduce_tuning(std::string_view(key), value)) return SG_OK;
  sg::set_error("sg_set_tuning: unknown key");
  return SG_ERR_NOT_FOUND;
}

}  // extern "C"
