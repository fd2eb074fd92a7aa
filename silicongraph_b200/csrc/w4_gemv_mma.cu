// INT4 group-quantised GEMV for one activation row with a tensor-core
// reduction (sm_100a).  Same contract and weight layout as w4_gemv.cu
// (compiler/kernels/cpu/matmul_neon.h:113-143); used when M == 1 and
// group_size % 32 == 0.
//
// Memory side (HBM-bound):
//   * Work unit = a chunk of 32 k-pair rows (64 k) x one tile of 1, 2 or 4
//     128-column strips.  A block has 16 warps = strips x phases; warp
//     (strip, phase) takes every phases-th chunk of the block's range for its
//     strip.
//   * Each warp streams its own 2-stage ring by TMA: a 128-byte x 32-row box
//     of packed weights (128-byte swizzle), the chunk's two scale rows and two
//     zero-point rows.
// Math side (few instructions per weight):
//   * The activation is staged once per block as 24-bit fixed point with one
//     power-of-two scale per 32 k (x = 2^(E-21) x_q, E the exponent of the
//     largest |x| there, so |x_q| <= 2^22 and the rounding error is below
//     2^-23 of that largest value), split as x_q = 65536 hi + 256 mid + lo,
//     signed bytes.  (16 bits were not enough: with one outlier of 100..1000
//     per 32 k, columns whose sum nearly cancels missed 2e-3 + 1e-2 |y|.)
//   * A 32-bit word (4 columns x one k pair, low nibble = even k) gives the
//     unsigned bytes of both k with one shift and two AND masks.  mma.sync
//     m16n8k32 (u8 x s8 -> exact int32) reduces over k: A rows are words of
//     4 columns, A k-slots their columns at 4 k-pair rows x even/odd k, and
//     B column 2e + v carries hi (v = 0) or mid (v = 1) of x at column slot
//     e and zero elsewhere, so every D entry is one column's hi or mid
//     partial dot product and every lane owns 4 columns outright; a second
//     MMA on the same A fragments takes lo (v = 0; v = 1 is zero).
//   * Per 32-k half and column, with S_hm = sum (x_q >> 8) and S_lo = sum lo
//     (integers exact in int32 until the last two roundings):
//     acc += scale * 2^(E-21) * (256 (256 D_hi + D_mid - (8 + zero) S_hm)
//                                + D_lo - (8 + zero) S_lo).
//   * Rows are assigned to the 4 lanes of a quad so that their (row mod 8)
//     values differ by 2: with the 128-byte swizzle the 8 lanes of a quarter
//     warp hit 8 distinct 16-byte bank groups (no bank conflicts).
//   * Scheduling: either clusters of ksplit blocks per tile that reduce
//     through distributed shared memory, or a balanced stream-K split of all
//     (512-column tile, chunk) units over one block per SM.  In the latter a
//     block's range touches one or more tiles ("segments"); every warp flushes
//     its column sums per segment into a private shared-memory slot, the
//     block sums its phases, owns interior tiles outright, and hands the
//     partial of a tile shared with its neighbours to global scratch, where
//     the last block to arrive (atomic ticket) adds the partials in block
//     order (deterministic).
//   * With SG_MM_STATIC_WEIGHTS the first weight stages are requested before
//     griddepcontrol.wait, so the weight stream overlaps the tail of the
//     previous kernel on the stream; the activation is read after the wait.
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string_view>

#include "rownorm.cuh"
#include "sm100.cuh"

namespace {

constexpr int kRows = 32;                    // k-pair rows per chunk
constexpr int kStreamKStrips = 4;           // stream-K tiles are 512 columns
constexpr int kStreamKCols = kStreamKStrips * 128;
constexpr int kWBytes = 128 * kRows;         // 4096
constexpr int kSBytes = 128 * 2 * 2;         // 2 scale rows x 128 fp16
constexpr int kZBytes = 128 * 2;             // 2 zero rows x 128 int8
constexpr int kSZBytes = kSBytes + kZBytes;  // 768
constexpr int kStaticSmemReserve = 2048;
// Launch shapes: warps per block (4 column strips x warps/4 phases) and TMA
// stages per warp.  Variant 0 is the default; the others are selectable with
// sg_set_tuning("w4_gemv_mma.variant", v) for measurement.
constexpr int kVariantWarps[5] = {16, 20, 12, 8, 8};
constexpr int kVariantStages[5] = {2, 2, 3, 5, 2};
constexpr int kPairVariant = 4;                // 8 warps: two blocks per SM
constexpr size_t kPairSmemLimit = 110 * 1024;  // dynamic shared memory that lets two blocks share an SM
constexpr int off_sz(int warps, int stages) { return warps * stages * kWBytes; }
constexpr int off_x(int warps, int stages) { return off_sz(warps, stages) + warps * stages * kSZBytes; }
// Dynamic shared memory after the stages (bytes): the staged activation (one
// word per k-pair row, scale and sum per half chunk), the stage barriers, the
// cluster's [rank][column] partials (rank 0's copy is the one used), then the
// per-segment, per-phase partial sums.
constexpr size_t kXSlotBytes = (size_t)kRows * 8 + 2 * 16;
inline size_t tail_bytes(int warps, int stages, int strips, int x_slots, int max_segs, int ksplit) {
  const size_t cols = (size_t)strips * 128;
  return (size_t)x_slots * kXSlotBytes + (size_t)warps * stages * 8 + (size_t)ksplit * cols * 4 +
         (size_t)max_segs * (warps / strips) * cols * 4;
}
std::atomic<int> g_variant{0};
std::atomic<int> g_sleep{0};
std::atomic<int> g_cluster_mode{1};
std::atomic<int> g_pair{1};  // allow two 8-warp blocks per SM
std::atomic<int> g_strips{0};  // 0: any tile width; 1, 2, 4: only that many 128-column strips

struct MArgs {
  const void* A;
  const __half* bias;
  void* C;
  int K, N, gs;
  int a_dt, c_dt;
  float scale_A;
  int has_zeros;
  int n_tiles, cpt, nblocks, total;
  int q, r;            // stream-K: block b owns chunks [b q + min(b, r), ...); the first r own q + 1
  int ksplit;          // cluster mode: blocks (cluster ranks) per tile
  int x_slots;         // activation staging capacity in 32-row chunks
  int x_by_row;        // slot of chunk c: c % cpt (range longer than K) or c - range start
  int max_segs;        // tiles one block's range can touch
  int gs_shift;        // log2(gs) when gs is a power of two, else -1
  int sleep_wait;      // back off with nanosleep while waiting for a stage
  int static_w;        // weights may be requested before the dependency wait
  int swiglu;          // A is [gate | up]: x = SwiGLU(A[k], A[K + k]) (SG_MM_A_SWIGLU)
  int norm;            // A is a residual-stream row: x = RMSNorm(A)[k] (SG_MM_A_RMSNORM)
  const void* norm_w;
  float norm_eps;
  int accum;           // C = round(C + round(y)) (SG_MM_C_ACCUMULATE)
  // q|k|v epilogue (sg_qkv_gemv_rope_append): rank 0 of each cluster owns its
  // whole tile, rounds it to C's type, rotates q and k and writes q / k / v
  int rope;
  int r_heads, r_kv, r_dim;
  const int32_t* r_pos;
  int r_pos0;
  float r_base;
  void* r_q;
  void* r_k;
  void* r_v;
  int64_t r_kv_hs;
  const int32_t* r_pt;
  int64_t r_pt_bs, r_pt_ps, r_page_stride;
  int r_npages;
  float* slots;        // [nblocks][2][512]: first / last segment partials
  unsigned* tickets;   // [n_tiles]
  int* err;
};

__device__ __forceinline__ int range_start(const MArgs& a, int b) { return b * a.q + min(b, a.r); }

__device__ __forceinline__ int block_of_chunk(const MArgs& a, int c) {
  const int big = a.r * (a.q + 1);
  return c < big ? c / (a.q + 1) : a.r + (c - big) / a.q;
}

__device__ __forceinline__ float load_act(const void* A, int dt, int i) {
  switch (dt) {
    case SG_DT_F32: return static_cast<const float*>(A)[i];
    case SG_DT_F16: return __half2float(static_cast<const __half*>(A)[i]);
    case SG_DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(A)[i]);
    default: return (float)static_cast<const int8_t*>(A)[i];
  }
}

// Activation k of the row: A[k]; with SG_MM_A_SWIGLU the SwiGLU of gate
// A[k] and up A[K + k] rounded to A's type, as sg_swiglu_rows writes it; with
// SG_MM_A_RMSNORM h[k] * rms_inv * w[k] rounded to A's type, as sg_rmsnorm
// writes it (rms_inv of the whole row, formed as sg_rmsnorm forms it).
__device__ __forceinline__ float load_x(const MArgs& a, int k, float rms_inv) {
  if (a.norm) {
    if (a.a_dt == SG_DT_BF16) {
      const float h = __bfloat162float(static_cast<const __nv_bfloat16*>(a.A)[k]);
      const float w = __bfloat162float(static_cast<const __nv_bfloat16*>(a.norm_w)[k]);
      return __bfloat162float(__float2bfloat16_rn(h * rms_inv * w));
    }
    const float h = __half2float(static_cast<const __half*>(a.A)[k]);
    const float w = __half2float(static_cast<const __half*>(a.norm_w)[k]);
    return __half2float(__float2half_rn(h * rms_inv * w));
  }
  if (a.swiglu) {
    if (a.a_dt == SG_DT_BF16) {
      const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(a.A);
      return __bfloat162float(sgd::swiglu_value<__nv_bfloat16>(__bfloat162float(p[k]), __bfloat162float(p[a.K + k])));
    }
    const __half* p = static_cast<const __half*>(a.A);
    return __half2float(sgd::swiglu_value<__half>(__half2float(p[k]), __half2float(p[a.K + k])));
  }
  return load_act(a.A, a.a_dt, k);
}

__device__ __forceinline__ void store_out(void* C, int dt, int64_t i, float v) {
  switch (dt) {
    case SG_DT_F32: sgd::store_from_float<SG_DT_F32>(C, i, v); break;
    case SG_DT_BF16: sgd::store_from_float<SG_DT_BF16>(C, i, v); break;
    default: sgd::store_from_float<SG_DT_F16>(C, i, v); break;
  }
}

__device__ __forceinline__ float finalize(const MArgs& a, int col, float v) {
  if (a.a_dt == SG_DT_I8) v = v * a.scale_A;
  if (a.bias) v = v + __half2float(a.bias[col]);
  return v;
}

// The column's final value: finalize, then either stored, or (SG_MM_C_ACCUMULATE)
// rounded to C's type and added to C with one more rounding -- the residual add
// of sg_rmsnorm, h = round(x + residual).
__device__ __forceinline__ void store_final(const MArgs& a, int col, float v) {
  v = finalize(a, col, v);
  if (a.accum) {
    if (a.c_dt == SG_DT_BF16) {
      __nv_bfloat16* c = static_cast<__nv_bfloat16*>(a.C);
      c[col] = __float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(v)) + __bfloat162float(c[col]));
    } else {
      __half* c = static_cast<__half*>(a.C);
      c[col] = __float2half_rn(__half2float(__float2half_rn(v)) + __half2float(c[col]));
    }
    return;
  }
  store_out(a.C, a.c_dt, col, v);
}

// sg_qkv_gemv_rope_append's epilogue on rank 0 of a cluster, which holds every
// rank's partial of the whole tile in csum[rank][kTC]: each column's sum
// rounded to C's type (the q|k|v output sg_qkv_rope_append would read), then
// the rotary pairs (i, i + D/2) of q and k heads and the plain v rows go to
// q_out and the KV cache, as qkv_rope_append_kernel writes them.  Heads never
// straddle tiles (D divides 128).
__device__ __forceinline__ void rope_epilogue(const MArgs& a, float* csum, int tile, int kTC, int nthreads) {
  const bool bf = a.c_dt == SG_DT_BF16;
  auto rnd = [&](float v) {
    return bf ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
  };
  for (int cc = threadIdx.x; cc < kTC; cc += nthreads) {
    float v = 0.f;
    for (int r = 0; r < a.ksplit; ++r) v += csum[r * kTC + cc];
    const int col = tile * kTC + cc;
    csum[cc] = col < a.N ? rnd(finalize(a, col, v)) : 0.f;  // in place: only this thread reads column cc
  }
  __syncthreads();
  const int D = a.r_dim, half = D / 2;
  const int p = a.r_pos ? *a.r_pos : a.r_pos0;
  for (int pc = threadIdx.x; pc < kTC / 2; pc += nthreads) {
    const int cc = (pc / half) * D + pc % half;
    const int col = tile * kTC + cc;
    if (col >= a.N) continue;
    const int slot = col / D, i = col % D;
    float x0 = csum[cc], x1 = csum[cc + half];
    if (slot < a.r_heads + a.r_kv) {
      float y0, y1;
      sgd::rope_pair(x0, x1, p, i, D, a.r_base, &y0, &y1);
      x0 = y0;
      x1 = y1;
    }
    int64_t off;
    void* base;
    if (slot < a.r_heads) {
      base = a.r_q;
      off = (int64_t)slot * D;
    } else {
      const bool is_k = slot < a.r_heads + a.r_kv;
      const int hk = is_k ? slot - a.r_heads : slot - a.r_heads - a.r_kv;
      base = is_k ? a.r_k : a.r_v;
      if (a.r_pt) {
        const int pg = __ldg(a.r_pt + (int64_t)(p >> 4) * a.r_pt_ps);
        if ((unsigned)pg >= (unsigned)a.r_npages) {  // no such page: dropped and reported
          if (i == 0) atomicOr(a.err, 4);
          continue;
        }
        off = (int64_t)pg * a.r_page_stride + ((int64_t)hk * 16 + (p & 15)) * D;
      } else {
        off = (int64_t)hk * a.r_kv_hs + (int64_t)p * D;
      }
    }
    if (bf) {
      __nv_bfloat16* d = static_cast<__nv_bfloat16*>(base) + off;
      d[i] = __float2bfloat16_rn(x0);
      d[i + half] = __float2bfloat16_rn(x1);
    } else {
      __half* d = static_cast<__half*>(base) + off;
      d[i] = __float2half_rn(x0);
      d[i + half] = __float2half_rn(x1);
    }
  }
}

__device__ __forceinline__ int group_of(const MArgs& a, int k) { return a.gs_shift >= 0 ? (k >> a.gs_shift) : k / a.gs; }

// CLUSTER: grid (ksplit, n_tiles), clusters of ksplit blocks own one tile and
// reduce their partials through distributed shared memory (no scratch).
// Otherwise: flat split of all chunks over the blocks, reduced through scratch.
// STRIPS: 128-column strips per tile (tile = STRIPS x 128 columns); the
// block's warps are STRIPS strips x WARPS / STRIPS phases.
template <bool HAS_Z, int WARPS, int STAGES, bool CLUSTER, int STRIPS>
__global__ void __launch_bounds__(WARPS * 32, WARPS <= 8 ? 2 : 1)
    w4_gemv_mma_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                       const __grid_constant__ CUtensorMap tmZ, MArgs a) {
  constexpr int kWarps = WARPS, kThreads = WARPS * 32, kPhases = WARPS / STRIPS, kStages = STAGES;
  constexpr int kTC = STRIPS * 128;
  constexpr int kOffW = 0, kOffSZ = off_sz(WARPS, STAGES), kOffX = off_x(WARPS, STAGES);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = sgd::align_smem_1024(smem_raw);
  uint2* xst = reinterpret_cast<uint2*>(smem + kOffX);               // [slot][32 rows]: x_q bytes
  int4* xgrp = reinterpret_cast<int4*>(xst + a.x_slots * kRows);     // [slot][half]: scale bits, S_hm, S_lo
  uint64_t* bars = reinterpret_cast<uint64_t*>(xgrp + a.x_slots * 2);
  float* csum = reinterpret_cast<float*>(bars + kWarps * kStages);  // cluster: [rank][kTC]
  float* red = csum + (CLUSTER ? a.ksplit * kTC : 0);                // [seg][phase][kTC]
  __shared__ int s_last;
  __shared__ int s_abort;
  __shared__ int s_aborts[16];  // cluster: rank r's abort flag, pushed to every rank
  __shared__ __align__(8) uint64_t s_rbar;  // cluster: the other ranks' pushes have landed

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int strip = warp % STRIPS, phase = warp / STRIPS;
  const int b = blockIdx.x;
  int cs, ce;
  if (CLUSTER) {
    const int tile = blockIdx.y, sp = blockIdx.x;
    cs = tile * a.cpt + (a.cpt * sp) / a.ksplit;
    ce = tile * a.cpt + (a.cpt * (sp + 1)) / a.ksplit;
  } else {
    cs = range_start(a, b);
    ce = range_start(a, b + 1);
  }
  const int t_first = cs / a.cpt;
  const int nseg = CLUSTER ? 1 : (ce - 1) / a.cpt - t_first + 1;
  const int nslots = a.x_by_row ? a.cpt : ce - cs;

  // cluster reduction: rank r owns columns [r * per, r * per + own) of the
  // tile and receives the other ranks' partials of them (plus their abort
  // flags) by st.async on s_rbar
  const int per = CLUSTER ? (a.rope ? kTC : ((kTC + a.ksplit - 1) / a.ksplit + 3) & ~3) : 1;
  const int own_lo = CLUSTER ? min(kTC, (int)blockIdx.x * per) : 0;
  const int own = CLUSTER ? min(kTC, own_lo + per) - own_lo : 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kWarps * kStages; ++i) sgd::mbar_init(&bars[i], 1);
    if (CLUSTER && a.ksplit > 1) {
      sgd::mbar_init(&s_rbar, 1);
      sgd::mbar_arrive_expect_tx(&s_rbar, (uint32_t)((a.ksplit - 1) * (own * 4 + 4)));
    }
    sgd::fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  // Distributed shared memory is touched only after every block of the
  // cluster has started: arrive now, wait before the first remote store.
  if (CLUSTER) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  sgd::pdl_launch_dependents();

  uint64_t* my_bars = bars + warp * kStages;
  const int c_first = cs + phase;
  const int n_my = (c_first < ce) ? (ce - c_first + kPhases - 1) / kPhases : 0;
  const uint32_t tx_bytes = kWBytes + kSBytes + (HAS_Z ? kZBytes : 0);

  // chunk position trackers (tile, row-chunk within tile), advanced by kPhases per step
  int it_tile = c_first / a.cpt, it_crow = c_first - it_tile * a.cpt;  // next chunk to issue
  auto issue = [&](int i) {
    const int tile = it_tile;
    const int row0 = it_crow * kRows;
    it_crow += kPhases;
    while (it_crow >= a.cpt) {
      it_crow -= a.cpt;
      ++it_tile;
    }
    const int gA = group_of(a, 2 * row0);
    const int x0 = tile * kTC + strip * 128;
    const int s = i % kStages;
    uint8_t* wdst = smem + kOffW + (warp * kStages + s) * kWBytes;
    uint8_t* szdst = smem + kOffSZ + (warp * kStages + s) * kSZBytes;
    uint64_t* bar = &my_bars[s];
    sgd::mbar_arrive_expect_tx(bar, tx_bytes);
    sgd::tma_load_2d(wdst, &tmW, x0, row0, bar);
    sgd::tma_load_2d(szdst, &tmS, x0, gA, bar);
    if (HAS_Z) sgd::tma_load_2d(szdst + kSBytes, &tmZ, x0, gA, bar);
  };

  // Weights that no earlier kernel writes stream before the dependency wait.
  if (a.static_w && lane == 0) {
    for (int i = 0; i < min(kStages, n_my); ++i) issue(i);
  }
  // The activation depends on the previous kernel; without the static-weight
  // promise it is requested first, so that its few bytes are not queued
  // behind this block's weight stream.
  sgd::pdl_wait();
  // SG_MM_A_RMSNORM: the row's 1 / rms over all K values, as sg_rmsnorm forms it
  __shared__ float s_red[32];
  float rms_inv = 0.f;
  if (a.norm) {
    rms_inv = a.a_dt == SG_DT_BF16
                  ? sgn::row_rms_inv(static_cast<const __nv_bfloat16*>(a.A), a.K, a.norm_eps, s_red)
                  : sgn::row_rms_inv(static_cast<const __half*>(a.A), a.K, a.norm_eps, s_red);
  }
  auto slot_row = [&](int idx, int& k) {  // staging row idx -> k of its even element
    const int sl = idx / kRows, r = idx - sl * kRows;
    const int crow = a.x_by_row ? sl : (cs + sl) % a.cpt;
    k = 2 * (crow * kRows + r);
  };
  constexpr int kPrefetchRows = 2;
  float xe_pf[kPrefetchRows], xo_pf[kPrefetchRows];
#pragma unroll
  for (int j = 0; j < kPrefetchRows; ++j) {
    const int idx = threadIdx.x + j * kThreads;
    xe_pf[j] = xo_pf[j] = 0.f;
    if (idx < nslots * kRows) {
      int k;
      slot_row(idx, k);
      if (k < a.K) xe_pf[j] = load_x(a, k, rms_inv);
      if (k + 1 < a.K) xo_pf[j] = load_x(a, k + 1, rms_inv);
    }
  }
  if (!a.static_w && lane == 0) {
    for (int i = 0; i < min(kStages, n_my); ++i) issue(i);
  }

  // ---- stage the activation as 24-bit fixed point, one power-of-two scale
  //      per half chunk (32 k): x = 2^(E-21) x_q with E the exponent of the
  //      half's largest |x|, so |x_q| <= 2^22, written as x_q = 65536 hi +
  //      256 mid + lo with hi, mid, lo signed bytes.  Per k-pair row two words
  //      [hi_even, hi_odd, mid_even, mid_odd], [lo_even, lo_odd, 0, 0]; per
  //      half the scale, S_hm = sum_k (x_q >> 8) and S_lo = sum_k lo.  A half
  //      is 16 rows = 16 lanes (rows per pass are a multiple of 32: whole warps).
  for (int idx = threadIdx.x, j = 0; idx < nslots * kRows; idx += kThreads, ++j) {
    int k;
    slot_row(idx, k);
    float xe, xo;
    if (j < kPrefetchRows) {
      xe = j == 0 ? xe_pf[0] : xe_pf[1];
      xo = j == 0 ? xo_pf[0] : xo_pf[1];
    } else {
      xe = (k < a.K) ? load_x(a, k, rms_inv) : 0.f;
      xo = (k + 1 < a.K) ? load_x(a, k + 1, rms_inv) : 0.f;
    }
    float m = fmaxf(fabsf(xe), fabsf(xo));
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // m >= 0; tiny halves clamp (2^(21+100) and 2^(-100-21) are normal floats)
    const int E = max((__float_as_int(m) >> 23) - 127, -100);
    const float inv = __int_as_float((127 + 21 - E) << 23);      // 2^(21 - E), exact scaling
    const float sxv = __int_as_float((127 - 21 + E) << 23);      // 2^(E - 21)
    const int qe = __float2int_rn(xe * inv), qo = __float2int_rn(xo * inv);
    const int le = ((qe + 128) & 255) - 128, lo = ((qo + 128) & 255) - 128;
    const int re = (qe - le) >> 8, ro = (qo - lo) >> 8;  // 256 hi + mid, exact
    const int me = ((re + 128) & 255) - 128, mo = ((ro + 128) & 255) - 128;
    const int he = (re - me) >> 8, ho = (ro - mo) >> 8;
    xst[idx] = make_uint2((uint32_t)(he & 255) | ((uint32_t)(ho & 255) << 8) | ((uint32_t)(me & 255) << 16) |
                              ((uint32_t)(mo & 255) << 24),
                          (uint32_t)(le & 255) | ((uint32_t)(lo & 255) << 8));
    int shm = re + ro, slo = le + lo;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
      shm += __shfl_xor_sync(0xffffffffu, shm, o);
      slo += __shfl_xor_sync(0xffffffffu, slo, o);
    }
    if ((lane & 15) == 0) xgrp[idx >> 4] = make_int4(__float_as_int(sxv), shm, slo, 0);
  }
  __syncthreads();

  // ---- lane roles in mma.sync m16n8k32 (A u8 row-major, B s8 col-major):
  //      A row m = g (m + 8) is the word of columns 16g + 8jm + 0..3 (+ 4..7)
  //      of k-pair row r_t, A k-slot 4t + e (16 + 4t + e) its column e at the
  //      even (odd) k; B column n = 2e + v holds byte v of a staged word of
  //      x at k-slot 4t + e, zero elsewhere: hi / mid from the first word,
  //      lo / zero from the second.  D[m][2t] / D[m][2t + 1] are then those
  //      partial dot products of column t of the word: every lane owns
  //      columns 16g + t + 4i, i = 0..3, with no cross-lane reduction.
  const int g = lane >> 2, t = lane & 3;
  const int be = g >> 1, bv = g & 1;  // as B provider: column n = g
  const uint32_t sel_e = (0x4444u & ~(0xFu << (4 * be))) | ((uint32_t)(2 * bv) << (4 * be));
  const uint32_t sel_o = (0x4444u & ~(0xFu << (4 * be))) | ((uint32_t)(2 * bv + 1) << (4 * be));
  // Step st covers k-pair rows base(st) + 2t, base = 16 (st / 4) + 8 (st / 2 % 2) + st % 2:
  // with the 128-byte swizzle the 8 lanes of a quarter warp read 8 distinct
  // 16-byte bank groups.  Lane offsets for even / odd base:
  const uint32_t woff0 = 256u * t + ((uint32_t)(g ^ (2 * t)) << 4);
  const uint32_t woff1 = 256u * t + ((uint32_t)(g ^ (2 * t + 1)) << 4);

  float acc[4];  // columns 16g + t + 4i of this warp's strip
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = 0.f;
  // Stores this lane's columns of segment seg into the warp's private slot and clears them.
  auto flush = [&](int seg) {
    float* r0 = red + (seg * kPhases + phase) * kTC + strip * 128 + 16 * g + t;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      r0[4 * i] = acc[i];
      acc[i] = 0.f;
    }
  };
  int cur_seg = 0;

  int ok = 1;
  int tile = c_first / a.cpt, crow = c_first - tile * a.cpt;
  for (int i = 0; i < n_my; ++i) {
    if (i > 0) {
      crow += kPhases;
      while (crow >= a.cpt) {
        crow -= a.cpt;
        ++tile;
      }
    }
    const int c = c_first + i * kPhases;
    const int sl = a.x_by_row ? crow : c - cs;
    const int s = i % kStages;
    if (!CLUSTER) {
      while (cur_seg < tile - t_first) flush(cur_seg++);  // warp-uniform
    }
    const bool waited = a.sleep_wait ? sgd::mbar_wait_sleep(&my_bars[s], (i / kStages) & 1, a.err)
                                     : sgd::mbar_wait(&my_bars[s], (i / kStages) & 1, a.err);
    if (!__all_sync(0xffffffffu, waited)) {
      ok = 0;
      break;
    }
    const uint8_t* wst = smem + kOffW + (warp * kStages + s) * kWBytes;
    const uint8_t* xr = reinterpret_cast<const uint8_t*>(xst + sl * kRows) + 16 * t;  // row 2t
    int d[2][2][4];  // [half][jm][fragment]: hi, mid
    int e[2][2][4];  // [half][jm][fragment]: lo, zero
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int jm = 0; jm < 2; ++jm)
#pragma unroll
        for (int q = 0; q < 4; ++q) d[h][jm][q] = e[h][jm][q] = 0;
#pragma unroll
    for (int st = 0; st < 8; ++st) {
      const int base = 16 * (st >> 2) + 8 * ((st >> 1) & 1) + (st & 1);
      const uint4 wv = *reinterpret_cast<const uint4*>(wst + base * 128 + ((st & 1) ? woff1 : woff0));
      const uint2 X = *reinterpret_cast<const uint2*>(xr + base * 8);
      const uint32_t b0 = __byte_perm(X.x, 0u, sel_e), b1 = __byte_perm(X.x, 0u, sel_o);
      const uint32_t c0 = __byte_perm(X.y, 0u, sel_e), c1 = __byte_perm(X.y, 0u, sel_o);
      const int h = st >> 2;
      const uint32_t a0 = wv.x & 0x0F0F0F0Fu, a1 = wv.y & 0x0F0F0F0Fu, a2 = (wv.x >> 4) & 0x0F0F0F0Fu,
                     a3 = (wv.y >> 4) & 0x0F0F0F0Fu;
      const uint32_t a4 = wv.z & 0x0F0F0F0Fu, a5 = wv.w & 0x0F0F0F0Fu, a6 = (wv.z >> 4) & 0x0F0F0F0Fu,
                     a7 = (wv.w >> 4) & 0x0F0F0F0Fu;
      sgd::mma_u8s8_16832(d[h][0], a0, a1, a2, a3, b0, b1);
      sgd::mma_u8s8_16832(d[h][1], a4, a5, a6, a7, b0, b1);
      sgd::mma_u8s8_16832(e[h][0], a0, a1, a2, a3, c0, c1);
      sgd::mma_u8s8_16832(e[h][1], a4, a5, a6, a7, c0, c1);
    }
    // ---- chunk epilogue per half and column:
    //      acc += scale * 2^(E-21) * (256 (256 D_hi + D_mid - (8 + zero) S_hm) + D_lo - (8 + zero) S_lo)
    //      |256 D_hi + D_mid - (8 + zero) S_hm| < 2^24: exact in int32 and as a float
    const uint8_t* szs = smem + kOffSZ + (warp * kStages + s) * kSZBytes;
    const int k0 = 2 * crow * kRows;
    const int gA = group_of(a, k0), gB = group_of(a, k0 + 32);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int srow = h ? (gB - gA) : 0;
      const int4 xg = xgrp[sl * 2 + h];
      const float sxh = __int_as_float(xg.x);
      const __half* sc_row = reinterpret_cast<const __half*>(szs + srow * 256) + 16 * g + t;
      const int8_t* z_row = reinterpret_cast<const int8_t*>(szs + kSBytes + srow * 128) + 16 * g + t;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int jm = i >> 1, fr = (i & 1) * 2;
        const int z8 = HAS_Z ? 8 + (int)z_row[4 * i] : 8;
        const int hm = d[h][jm][fr] * 256 + d[h][jm][fr + 1] - z8 * xg.y;
        const int lw = e[h][jm][fr] - z8 * xg.z;
        acc[i] = fmaf(__half2float(sc_row[4 * i]) * sxh, fmaf(256.f, (float)hm, (float)lw), acc[i]);
      }
    }
    __syncwarp();
    if (lane == 0 && i + kStages < n_my) issue(i + kStages);
  }
  if (!ok) s_abort = 1;
  while (cur_seg < nseg) flush(cur_seg++);  // the last touched segment, then zeros for any not reached
  __syncthreads();
  if (!CLUSTER && s_abort) return;

  if (CLUSTER) {
    // Each rank adds its phases and pushes the sums of the columns that
    // another rank owns straight into that rank's [rank][column] buffer with
    // st.async (completion counted on the owner's s_rbar), keeps its own, and
    // then adds the ranks' partials of its columns in rank order and stores
    // them.  One-sided: no cluster-wide barrier after the pushes.
    const int rank = blockIdx.x;  // cluster dims (ksplit, 1, 1): rank == blockIdx.x
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every rank has started
    for (int c4 = threadIdx.x; c4 < kTC / 4; c4 += kThreads) {
      const int cc = 4 * c4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int ph = 0; ph < kPhases; ++ph) {
        const float4 r = *reinterpret_cast<const float4*>(&red[ph * kTC + cc]);
        v.x += r.x;
        v.y += r.y;
        v.z += r.z;
        v.w += r.w;
      }
      const int owner = cc / per;
      if (owner == rank || a.ksplit == 1) {
        *reinterpret_cast<float4*>(&csum[rank * kTC + cc]) = v;
      } else {
        sgd::st_async_v4(sgd::cluster_addr(&csum[rank * kTC + cc], owner), v, sgd::cluster_addr(&s_rbar, owner));
      }
    }
    if (a.ksplit > 1 && threadIdx.x < a.ksplit && threadIdx.x != rank) {
      const uint32_t q = threadIdx.x;
      sgd::st_async_u32(sgd::cluster_addr(&s_aborts[rank], q), (uint32_t)s_abort, sgd::cluster_addr(&s_rbar, q));
    }
    int ok_wait = 1;
    if (a.ksplit > 1) ok_wait = sgd::mbar_wait(&s_rbar, 0, a.err) ? 1 : 0;
    __syncthreads();  // the local partial and (through s_rbar) the pushed ones are visible
    int aborted = s_abort || !ok_wait;
    for (int r = 0; r < a.ksplit; ++r)
      if (r != rank) aborted |= s_aborts[r];
    if (!aborted && a.rope) {
      if (own > 0) rope_epilogue(a, csum, blockIdx.y, kTC, kThreads);  // rank 0: the whole tile
    } else if (!aborted) {
      const int tile = blockIdx.y;
      for (int cc = own_lo + threadIdx.x; cc < own_lo + own; cc += kThreads) {
        float v = 0.f;
        for (int r = 0; r < a.ksplit; ++r) v += csum[r * kTC + cc];
        const int col = tile * kTC + cc;
        if (col < a.N) store_final(a, col, v);
      }
    }
    return;
  }

  for (int s2 = 0; s2 < nseg; ++s2) {
    const int tile = t_first + s2;
    const int tc0 = tile * a.cpt;
    const int b_lo = block_of_chunk(a, tc0), b_hi = block_of_chunk(a, tc0 + a.cpt - 1);
    const bool shared_tile = b_lo != b_hi;  // only a first or last segment can be shared
    const int slot = s2 == 0 ? 0 : 1;
    for (int cc = threadIdx.x; cc < kTC; cc += kThreads) {
      float v = 0.f;
#pragma unroll
      for (int ph = 0; ph < kPhases; ++ph) v += red[(s2 * kPhases + ph) * kTC + cc];
      const int col = tile * kTC + cc;
      if (!shared_tile) {
        if (col < a.N) store_final(a, col, v);
      } else {
        a.slots[((int64_t)b * 2 + slot) * kTC + cc] = v;
      }
    }
    if (!shared_tile) continue;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(&a.tickets[tile], 1u);
      s_last = (prev == (unsigned)(b_hi - b_lo)) ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) continue;
    __threadfence();
    for (int cc = threadIdx.x; cc < kTC; cc += kThreads) {
      const int col = tile * kTC + cc;
      // Partials in block order; loads batched so that they are in flight
      // together.  The tile is block bb's first segment (slot 0) when bb
      // starts inside it, else its last (slot 1).
      float v = 0.f;
      for (int b0 = b_lo; b0 <= b_hi; b0 += 8) {
        float pv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int bb = b0 + u;
          pv[u] = 0.f;
          if (bb <= b_hi) {
            const int sb = range_start(a, bb) >= tc0 ? 0 : 1;
            pv[u] = __ldcg(&a.slots[((int64_t)bb * 2 + sb) * kTC + cc]);
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (b0 + u <= b_hi) v += pv[u];
      }
      if (col < a.N) store_final(a, col, v);
    }
    if (threadIdx.x == 0) a.tickets[tile] = 0u;
  }
}

struct MPlan {
  bool ok = false;
  int variant = 0;
  int cluster = 0, ksplit = 1, strips = kStreamKStrips;
  int n_tiles = 0, cpt = 0, nblocks = 0, total = 0, q = 0, r = 0;
  int x_slots = 0, x_by_row = 0, max_segs = 1;
  size_t smem = 0, ws_bytes = 0, tickets_bytes = 0;
};

// Clusters of k blocks that can be resident at once: one 16-warp block per
// SM, or (pair) two 8-warp blocks per SM.  The cache is process-wide: it
// assumes every GPU of the process is the same model (true of one B200 node).
int max_active_clusters(int k, int pair) {
  static std::mutex mu;
  static int cache[2][17] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (k < 1 || k > 16) return 0;
  if (cache[pair][k] != 0) return cache[pair][k];
  const int smem = pair ? (int)kPairSmemLimit : 225 * 1024;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(k, 1);
  cfg.blockDim = dim3(pair ? 256 : 512);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = k;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  auto kfn = pair ? w4_gemv_mma_kernel<true, 8, 2, true, 2> : w4_gemv_mma_kernel<true, 16, 2, true, 4>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = -1;
  }
  cache[pair][k] = n;
  return n;
}

MPlan make_mplan(const SgMatMulParams* p, int sms) {
  MPlan pl;
  const int gs = p->group_size > 0 ? p->group_size : 128;
  if (p->M != 1 || p->K <= 0 || (p->N % 16) != 0 || (gs % 32) != 0) return pl;
  if (!sg::aligned16(p->B) || !sg::aligned16(p->scales_B) || (p->zeros_B && !sg::aligned16(p->zeros_B))) return pl;
  const int KP = (p->K + 1) / 2;
  pl.cpt = (KP + kRows - 1) / kRows;
  // Cluster split: tiles of 4, 2 or 1 strips (512 / 256 / 128 columns), each
  // split over k <= 8 blocks that reduce through distributed shared memory
  // (no global scratch), with one 16-warp block per SM or, when no such
  // shape fits, two 8-warp blocks per SM.  The shape that keeps the most
  // warps busy in one wave (clusters must fit inside a GPC) wins; ties go to
  // wider tiles.  Mode 1 (default) falls back to the stream-K split when no cluster
  // shape fills at least half the SMs, mode 2 always takes a cluster shape
  // that fits, mode 0 never does.
  const int mode = g_cluster_mode.load();
  long long best_score = 0;
  int best_strips = 0, best_k = 0, best_pair = 0;
  if (mode != 0) {
    for (int pair : {0, 1}) {
      // two blocks per SM only when the tiles outnumber the SMs: with fewer
      // tiles they measured slower than one 16-warp block per SM
      if (pair && (!g_pair.load() || best_score > 0)) continue;
      const int slots = sms * (pair ? 2 : 1);
      const int vv = pair ? kPairVariant : 0;
      for (int strips : {4, 2, 1}) {
        if (g_strips.load() != 0 && strips != g_strips.load()) continue;
        const int n_tiles = (p->N + strips * 128 - 1) / (strips * 128);
        if (n_tiles > slots) continue;
        for (int k = std::min({8, pl.cpt, slots / n_tiles}); k >= 1; --k) {
          if (max_active_clusters(k, pair) < n_tiles) continue;
          const size_t smem = 1024 + off_x(kVariantWarps[vv], kVariantStages[vv]) +
                              tail_bytes(kVariantWarps[vv], kVariantStages[vv], strips, (pl.cpt + k - 1) / k, 1, k);
          if (pair && smem > kPairSmemLimit) continue;
          const long long score = (long long)n_tiles * k * kVariantWarps[vv];
          if (score > best_score) {
            best_score = score;
            best_strips = strips;
            best_k = k;
            best_pair = pair;
          }
          break;
        }
      }
    }
    if (mode == 1 && 2 * best_score < (long long)sms * 16) best_score = 0;
  }
  pl.variant = std::min(kPairVariant, std::max(0, g_variant.load()));
  if (best_score > 0) {
    pl.cluster = 1;
    pl.strips = best_strips;
    pl.ksplit = best_k;
    if (best_pair) {
      pl.variant = kPairVariant;
    } else if (best_strips != 4) {
      pl.variant = 0;  // the narrow tiles come in the default launch shape only
    }
    pl.n_tiles = (p->N + best_strips * 128 - 1) / (best_strips * 128);
    pl.total = pl.n_tiles * pl.cpt;
    pl.nblocks = pl.n_tiles * best_k;
    pl.x_slots = (pl.cpt + best_k - 1) / best_k;
    pl.x_by_row = 0;
    pl.max_segs = 1;
  } else {
    pl.strips = kStreamKStrips;
    pl.n_tiles = (p->N + kStreamKCols - 1) / kStreamKCols;
    const long long total = (long long)pl.n_tiles * pl.cpt;
    if (total >= (1ll << 30)) return pl;
    pl.total = (int)total;
    pl.nblocks = (int)std::min<long long>(sms, total);
    pl.q = pl.total / pl.nblocks;
    pl.r = pl.total % pl.nblocks;
    const int longest = pl.q + (pl.r > 0 ? 1 : 0);
    pl.x_by_row = longest > pl.cpt ? 1 : 0;
    pl.x_slots = pl.x_by_row ? pl.cpt : longest;
    pl.max_segs = (longest - 1 + pl.cpt - 1) / pl.cpt + 1;
  }
  const int vw = kVariantWarps[pl.variant], vs = kVariantStages[pl.variant];
  pl.smem = 1024 + off_x(vw, vs) +
            tail_bytes(vw, vs, pl.strips, pl.x_slots, pl.max_segs, pl.cluster ? pl.ksplit : 0);
  // opt-in limit per block (227 KB on sm_100) minus this kernel's static shared memory
  if (pl.smem > 227 * 1024 - kStaticSmemReserve) return pl;
  if (pl.cluster) {
    pl.tickets_bytes = 0;
    pl.ws_bytes = 0;  // partials stay in distributed shared memory
  } else {
    pl.tickets_bytes = sg::ticket_bytes(pl.n_tiles);
    pl.ws_bytes = pl.tickets_bytes + (size_t)pl.nblocks * 2 * kStreamKCols * sizeof(float);
  }
  pl.ok = true;
  return pl;
}

}  // namespace

namespace sg {

size_t w4_gemv_mma_scratch_bytes(const SgMatMulParams* p, int sms, bool* applicable) {
  const MPlan pl = make_mplan(p, sms);
  *applicable = pl.ok;
  return pl.ok ? pl.ws_bytes : 0;
}

// Runs the tensor-core GEMV if it applies; *handled tells the caller.
SgStatus w4_gemv_mma_run(const SgMatMulParams* p, cudaStream_t cs, int sms, void* ws, size_t ws_bytes,
                         int* err_word, bool* handled, const SgRopeAppend* rope) {
  *handled = false;
  const MPlan pl = make_mplan(p, sms);
  if (!pl.ok) return SG_OK;
  if (rope && !pl.cluster) return SG_OK;  // the fused epilogue needs the cluster split
  *handled = true;
  SG_CHECK_ARG(pl.ws_bytes == 0 || (ws != nullptr && ws_bytes >= pl.ws_bytes && aligned16(ws)),
               "sg_matmul_int4_grouped: workspace too small (%zu < %zu bytes)", ws_bytes, pl.ws_bytes);
  const int gs = p->group_size > 0 ? p->group_size : 128;
  const int KP = (p->K + 1) / 2;
  const int G = (p->K + gs - 1) / gs;
  CUtensorMap tw, ts, tz;
  SgStatus st;
  {
    const uint64_t dims[2] = {(uint64_t)p->N, (uint64_t)KP};
    const uint64_t strides[1] = {(uint64_t)p->N};
    const uint32_t box[2] = {128, (uint32_t)kRows};
    st = make_tensor_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(p->B), dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SG_OK) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)p->N, (uint64_t)G};
    const uint64_t sstr[1] = {(uint64_t)p->N * 2};
    const uint32_t box[2] = {128, 2};
    st = make_tensor_map(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(p->scales_B), dims, sstr, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != SG_OK) return st;
    if (p->zeros_B) {
      const uint64_t zstr[1] = {(uint64_t)p->N};
      st = make_tensor_map(&tz, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(p->zeros_B), dims, zstr, box,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
      if (st != SG_OK) return st;
    } else {
      tz = ts;  // never read
    }
  }
  MArgs a{};
  a.A = p->A;
  a.bias = static_cast<const __half*>(p->bias);
  a.C = p->C;
  a.K = p->K;
  a.N = p->N;
  a.gs = gs;
  a.a_dt = p->a_dtype == SG_DT_DEFAULT ? SG_DT_I8 : p->a_dtype;
  a.c_dt = p->c_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->c_dtype;
  a.scale_A = p->scale_A;
  a.has_zeros = p->zeros_B != nullptr;
  a.n_tiles = pl.n_tiles;
  a.cpt = pl.cpt;
  a.nblocks = pl.nblocks;
  a.total = pl.total;
  a.q = pl.q;
  a.r = pl.r;
  a.ksplit = pl.ksplit;
  a.x_slots = pl.x_slots;
  a.x_by_row = pl.x_by_row;
  a.max_segs = pl.max_segs;
  a.gs_shift = ((gs & (gs - 1)) == 0) ? __builtin_ctz((unsigned)gs) : -1;
  a.sleep_wait = g_sleep.load() ? 1 : 0;
  a.static_w = (p->flags & SG_MM_STATIC_WEIGHTS) ? 1 : 0;
  a.swiglu = (p->flags & SG_MM_A_SWIGLU) ? 1 : 0;
  a.norm = (p->flags & SG_MM_A_RMSNORM) ? 1 : 0;
  a.norm_w = p->norm_weight;
  a.norm_eps = p->norm_eps;
  a.accum = (p->flags & SG_MM_C_ACCUMULATE) ? 1 : 0;
  if (rope) {
    a.rope = 1;
    a.r_heads = rope->heads;
    a.r_kv = rope->kv_heads;
    a.r_dim = rope->head_dim;
    a.r_pos = rope->positions;
    a.r_pos0 = rope->pos0;
    a.r_base = rope->base;
    a.r_q = rope->q_out;
    a.r_k = rope->k_cache;
    a.r_v = rope->v_cache;
    a.r_kv_hs = rope->kv_head_stride;
    if (const SgKvPages* pg = rope->kv_pages) {
      a.r_pt = pg->table;
      a.r_pt_ps = pg->table_page_stride;
      a.r_page_stride = pg->page_stride;
      a.r_npages = pg->num_pages;
    }
  }
  a.tickets = static_cast<unsigned*>(ws);
  a.slots = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.tickets_bytes);
  a.err = err_word;

  using KFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, MArgs);
  // [zeros][variant]: stream-K (512-column tiles), cluster with 512-column
  // tiles; [zeros][strips 1 / 2]: cluster with narrow tiles, default shape
#define SG_W4MMA_KFNS(Z, C)                                                                                   \
  {w4_gemv_mma_kernel<Z, 16, 2, C, 4>, w4_gemv_mma_kernel<Z, 20, 2, C, 4>, w4_gemv_mma_kernel<Z, 12, 3, C, 4>, \
   w4_gemv_mma_kernel<Z, 8, 5, C, 4>}
  static const KFn kstream[2][4] = {SG_W4MMA_KFNS(false, false), SG_W4MMA_KFNS(true, false)};
  static const KFn kcluster[2][4] = {SG_W4MMA_KFNS(false, true), SG_W4MMA_KFNS(true, true)};
#undef SG_W4MMA_KFNS
  static const KFn knarrow[2][2] = {{w4_gemv_mma_kernel<false, 16, 2, true, 1>, w4_gemv_mma_kernel<false, 16, 2, true, 2>},
                                    {w4_gemv_mma_kernel<true, 16, 2, true, 1>, w4_gemv_mma_kernel<true, 16, 2, true, 2>}};
  static const KFn kpair[2][3] = {{w4_gemv_mma_kernel<false, 8, 2, true, 1>, w4_gemv_mma_kernel<false, 8, 2, true, 2>,
                                   w4_gemv_mma_kernel<false, 8, 2, true, 4>},
                                  {w4_gemv_mma_kernel<true, 8, 2, true, 1>, w4_gemv_mma_kernel<true, 8, 2, true, 2>,
                                   w4_gemv_mma_kernel<true, 8, 2, true, 4>}};
  const int zi = a.has_zeros ? 1 : 0;
  const int si = pl.strips == 4 ? 2 : pl.strips == 2 ? 1 : 0;
  int ki;
  KFn kfn;
  if (!pl.cluster) {
    ki = pl.variant;
    kfn = kstream[zi][pl.variant];
  } else if (pl.variant == kPairVariant) {
    ki = 10 + si;
    kfn = kpair[zi][si];
  } else if (pl.strips == 4) {
    ki = 4 + pl.variant;
    kfn = kcluster[zi][pl.variant];
  } else {
    ki = 8 + si;
    kfn = knarrow[zi][si];
  }
  // the shared-memory opt-in belongs to each device's copy of the kernel
  static std::mutex mu;
  static size_t attr_smem[64][2][13] = {};
  {
    int dev = 0;
    const SgStatus dst = sg::current_device(&dev);
    if (dst != SG_OK) return dst;
    std::lock_guard<std::mutex> lk(mu);
    size_t scratch = 0;
    size_t& done = dev >= 0 && dev < 64 ? attr_smem[dev][zi][ki] : scratch;
    if (done < pl.smem) {
      cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
      if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("w4_gemv_mma: cudaFuncSetAttribute(%zu) failed: %s", pl.smem, cudaGetErrorString(e));
        return SG_ERR_RUNTIME;
      }
      done = pl.smem;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = pl.cluster ? dim3(pl.ksplit, pl.n_tiles) : dim3(pl.nblocks);
  cfg.blockDim = dim3(kVariantWarps[pl.variant] * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = cs;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = pl.ksplit;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pl.cluster ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, tw, ts, tz, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("w4_gemv_mma_kernel launch failed: %s", cudaGetErrorString(e));
    return SG_ERR_RUNTIME;
  }
  return SG_OK;
}

bool w4_gemv_mma_tuning(std::string_view key, int value) {
  if (key == "w4_gemv_mma.variant") {
    g_variant.store(value);
    return true;
  }
  if (key == "w4_gemv_mma.cluster") {
    g_cluster_mode.store(value);
    return true;
  }
  if (key == "w4_gemv_mma.strips") {
    g_strips.store(value);
    return true;
  }
  if (key == "w4_gemv_mma.pair") {
    g_pair.store(value);
    return true;
  }
  if (key == "w4_gemv_mma.sleep") {
    g_sleep.store(value);
    return true;
  }
  return false;
}

}  // namespace sg
