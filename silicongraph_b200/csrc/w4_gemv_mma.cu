// INT4 group-quantised GEMV for one activation row with a tensor-core
// reduction (sm_100a).  Same contract and weight layout as w4_gemv.cu
// (compiler/kernels/cpu/matmul_neon.h:113-143); used when M == 1 and
// group_size % 32 == 0.
//
// Memory side (HBM-bound):
//   * Work unit = a chunk of 32 k-pair rows (64 k) x one 512-column tile.
//     Chunks are split evenly over one block per SM.  A block has 16 warps =
//     4 column strips (128 columns each) x 4 phases; warp (strip, phase)
//     takes every 4th chunk of the block's range for its strip.
//   * Each warp streams its own 2-stage ring by TMA: a 128-byte x 32-row box
//     of packed weights (128-byte swizzle), the chunk's two scale rows and two
//     zero-point rows.  The first stages are issued before griddepcontrol.wait,
//     so with programmatic dependent launch the next GEMV's weights start
//     streaming while the previous kernel drains.
// Math side (few instructions per weight):
//   * A 32-bit word (4 columns x one k pair) becomes four fp16x2 registers
//     with one shift and four LOP3 (0x6400 magic): 1024 + q for even k and
//     1024 + 16 q for odd k; pairs hold columns (c0,c2) / (c1,c3) of one k.
//     Odd-k activations are pre-divided by 16 (exact), and the constant part
//     (1024 * sum of the B entries) is subtracted after the MMA.
//   * mma.sync m16n8k16 (fp16 x fp16 -> fp32) reduces over k: A = those
//     registers (16 column pairs x 16 logical k), B = the activation.  Logical
//     k 2t+e carries column e of a pair, so B holds x in column n = 2v + e and
//     zeros elsewhere; the 8 B columns carry 4 "variants" v: the two halves of
//     the chunk (rows 0-15 and 16-31, each inside one quantisation group) times
//     x split as fp16 hi + lo (x - hi), which keeps fp32 activation accuracy.
//     Every lane of the D fragment then holds useful partial sums.
//   * Per chunk half, variant and column (packed fp32x2 FMAs):
//     acc += scale * (D - 1024 * sum b - (8 + zero) * sum_k x_k); halves and
//     variants are summed with two warp shuffles at the end.
//   * Rows are assigned to the 4 lanes of a quad so that their (row mod 8)
//     values differ by 2: with the 128-byte swizzle the 8 lanes of a quarter
//     warp hit 8 distinct 16-byte bank groups (no bank conflicts).
//   * Blocks reduce their phases in shared memory; a 512-column tile shared by
//     two blocks is finished by the later one (atomic ticket, fixed order).
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string_view>

#include "sm100.cuh"

namespace {

constexpr int kStrips = 4;
constexpr int kRows = 32;                    // k-pair rows per chunk
constexpr int kTileCols = kStrips * 128;     // 512
constexpr int kWBytes = 128 * kRows;         // 4096
constexpr int kSBytes = 128 * 2 * 2;         // 2 scale rows x 128 fp16
constexpr int kZBytes = 128 * 2;             // 2 zero rows x 128 int8
constexpr int kSZBytes = kSBytes + kZBytes;  // 768
constexpr int kXRowBytes = 32;               // 8 B-fragment words per k-pair row
constexpr int kStaticSmemReserve = 2048;
// Launch shapes: warps per block (4 column strips x warps/4 phases) and TMA
// stages per warp.  Variant 0 is the default; the others are selectable with
// sg_set_tuning("w4_gemv_mma.variant", v) for measurement.
constexpr int kVariantWarps[4] = {16, 20, 12, 8};
constexpr int kVariantStages[4] = {2, 2, 3, 5};
constexpr int off_sz(int warps, int stages) { return warps * stages * kWBytes; }
constexpr int off_x(int warps, int stages) { return off_sz(warps, stages) + warps * stages * kSZBytes; }
std::atomic<int> g_variant{0};
std::atomic<int> g_sleep{0};
std::atomic<int> g_cluster_mode{1};

struct MArgs {
  const void* A;
  const __half* bias;
  void* C;
  int K, N, gs;
  int a_dt, c_dt;
  float scale_A;
  int has_zeros;
  int n_tiles, cpt, nblocks, flat, total;
  int ksplit;          // cluster mode: blocks (cluster ranks) per 512-column tile
  int max_chunks;      // x staging capacity (chunks per block)
  int gs_shift;        // log2(gs) when gs is a power of two, else -1
  int sleep_wait;      // back off with nanosleep while waiting for a stage
  float* slots;        // [nblocks][2][512]
  unsigned* tickets;   // [n_tiles]
  int* err;
};

__device__ __forceinline__ void block_range(const MArgs& a, int b, int& cs, int& ce) {
  if (a.flat) {
    cs = (int)((long long)a.total * b / a.nblocks);
    ce = (int)((long long)a.total * (b + 1) / a.nblocks);
  } else {  // one block per tile
    cs = b * a.cpt;
    ce = cs + a.cpt;
  }
}

__device__ __forceinline__ int block_of_chunk(const MArgs& a, int c) {
  if (!a.flat) return c / a.cpt;
  int b = (int)((long long)c * a.nblocks / a.total);
  while (b + 1 < a.nblocks && (long long)a.total * (b + 1) / a.nblocks <= c) ++b;
  while (b > 0 && (long long)a.total * b / a.nblocks > c) --b;
  return b;
}

__device__ __forceinline__ float load_act(const void* A, int dt, int i) {
  switch (dt) {
    case SG_DT_F32: return static_cast<const float*>(A)[i];
    case SG_DT_F16: return __half2float(static_cast<const __half*>(A)[i]);
    case SG_DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(A)[i]);
    default: return (float)static_cast<const int8_t*>(A)[i];
  }
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

__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}


// Raw nibble carriers as fp16 pairs (no offset removal): for a word of 4
// columns x one k pair, lo = 1024 + q (even k), hi = 1024 + 16 q (odd k);
// pairs (c0,c2) and (c1,c3).  The constant 1024 (resp. 1024 / 16 with the
// odd activations pre-divided by 16) is removed after the MMA through a
// per-chunk correction, so each word costs one shift and four LOP3.
__device__ __forceinline__ void nibbles_h(uint32_t w, uint32_t& e02, uint32_t& o02, uint32_t& e13, uint32_t& o13) {
  const uint32_t MAGIC = 0x64006400u;  // fp16 1024 in both halves
  const uint32_t w8 = w >> 8;
  e02 = sgd::lop3_and_or(w, 0x000F000Fu, MAGIC);
  o02 = sgd::lop3_and_or(w, 0x00F000F0u, MAGIC);
  e13 = sgd::lop3_and_or(w8, 0x000F000Fu, MAGIC);
  o13 = sgd::lop3_and_or(w8, 0x00F000F0u, MAGIC);
}

__device__ __forceinline__ int group_of(const MArgs& a, int k) { return a.gs_shift >= 0 ? (k >> a.gs_shift) : k / a.gs; }

// CLUSTER: grid (ksplit, n_tiles), clusters of ksplit blocks own one tile and
// reduce their partials through distributed shared memory (no scratch).
// Otherwise: flat split of all chunks over the blocks, reduced through scratch.
template <bool HAS_Z, int WARPS, int STAGES, bool CLUSTER>
__global__ void __launch_bounds__(WARPS * 32, 1)
    w4_gemv_mma_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                       const __grid_constant__ CUtensorMap tmZ, MArgs a) {
  constexpr int kWarps = WARPS, kThreads = WARPS * 32, kPhases = WARPS / kStrips, kStages = STAGES;
  constexpr int kOffW = 0, kOffSZ = off_sz(WARPS, STAGES), kOffX = off_x(WARPS, STAGES);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xst = smem + kOffX;                                             // [chunk][32 rows][32 B]
  float4* xrow = reinterpret_cast<float4*>(xst + a.max_chunks * kRows * kXRowBytes);  // [chunk][32]
  float4* xhalf = xrow + a.max_chunks * kRows;                             // [chunk][2]: Xhi, Phi, Xlo, Plo
  uint8_t* zrow = reinterpret_cast<uint8_t*>(xhalf + a.max_chunks * 2);   // 16 zero bytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(zrow + 16);
  __shared__ int s_last;
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int strip = warp % kStrips, phase = warp / kStrips;
  const int b = blockIdx.x;
  int cs, ce;
  if (CLUSTER) {
    const int tile = blockIdx.y, sp = blockIdx.x;
    cs = tile * a.cpt + (a.cpt * sp) / a.ksplit;
    ce = tile * a.cpt + (a.cpt * (sp + 1)) / a.ksplit;
  } else {
    block_range(a, b, cs, ce);
  }
  const int t_first = cs / a.cpt;
  const int nchunks = ce - cs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kWarps * kStages; ++i) sgd::mbar_init(&bars[i], 1);
    sgd::fence_mbar_init();
    s_abort = 0;
  }
  if (threadIdx.x < 4) reinterpret_cast<uint32_t*>(zrow)[threadIdx.x] = 0u;
  __syncthreads();
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
    const int x0 = tile * kTileCols + strip * 128;
    const int s = i % kStages;
    uint8_t* wdst = smem + kOffW + (warp * kStages + s) * kWBytes;
    uint8_t* szdst = smem + kOffSZ + (warp * kStages + s) * kSZBytes;
    uint64_t* bar = &my_bars[s];
    sgd::mbar_arrive_expect_tx(bar, tx_bytes);
    sgd::tma_load_2d(wdst, &tmW, x0, row0, bar);
    sgd::tma_load_2d(szdst, &tmS, x0, gA, bar);
    if (HAS_Z) sgd::tma_load_2d(szdst + kSBytes, &tmZ, x0, gA, bar);
  };

  // The activation depends on the previous kernel; request it first, so that
  // its few bytes are not queued behind this block's weight stream.
  sgd::pdl_wait();
  constexpr int kPrefetchRows = 2;
  float xe_pf[kPrefetchRows], xo_pf[kPrefetchRows];
#pragma unroll
  for (int j = 0; j < kPrefetchRows; ++j) {
    const int idx = threadIdx.x + j * kThreads;
    xe_pf[j] = xo_pf[j] = 0.f;
    if (idx < nchunks * kRows) {
      const int cl = idx / kRows, r = idx - cl * kRows;
      const int k = 2 * (((cs + cl) % a.cpt) * kRows + r);
      if (k < a.K) xe_pf[j] = load_act(a.A, a.a_dt, k);
      if (k + 1 < a.K) xo_pf[j] = load_act(a.A, a.a_dt, k + 1);
    }
  }
  if (lane == 0) {
    for (int i = 0; i < min(kStages, n_my); ++i) issue(i);
  }

  // ---- stage the activation as ready-made B fragments.  Per k-pair row:
  //      8 words [hi/lo][column select e][even, odd] with even entries x and odd
  //      entries x/16 (fp16, x split as hi + lo), and per-row sums used to undo
  //      the nibble carriers' constant: X = sum_k x_eff, P = 1024 * sum b.
  for (int idx = threadIdx.x, j = 0; idx < nchunks * kRows; idx += kThreads, ++j) {
    const int cl = idx / kRows, r = idx - cl * kRows;
    const int c = cs + cl;
    const int row = (c % a.cpt) * kRows + r;
    const int k = 2 * row;
    float xe, xo;
    if (j < kPrefetchRows) {
      xe = j == 0 ? xe_pf[0] : xe_pf[1];
      xo = j == 0 ? xo_pf[0] : xo_pf[1];
    } else {
      xe = (k < a.K) ? load_act(a.A, a.a_dt, k) : 0.f;
      xo = (k + 1 < a.K) ? load_act(a.A, a.a_dt, k + 1) : 0.f;
    }
    const __half he = __float2half_rn(xe);
    const __half hoF = __float2half_rn(xo);
    const __half le = __float2half_rn(xe - __half2float(he));
    const __half loF = __float2half_rn(xo - __half2float(hoF));
    const __half ho = __float2half_rn(__half2float(hoF) * 0.0625f);  // exact: power-of-two scaling
    const __half lo = __float2half_rn(__half2float(loF) * 0.0625f);
    const __half z = __ushort_as_half(0);
    uint4 w0, w1;
    w0.x = pack_h2(he, z);  // hi, e=0 (even, odd)
    w0.y = pack_h2(ho, z);
    w0.z = pack_h2(z, he);  // hi, e=1
    w0.w = pack_h2(z, ho);
    w1.x = pack_h2(le, z);  // lo, e=0
    w1.y = pack_h2(lo, z);
    w1.z = pack_h2(z, le);  // lo, e=1
    w1.w = pack_h2(z, lo);
    uint4* dst = reinterpret_cast<uint4*>(xst + (size_t)idx * kXRowBytes);
    dst[0] = w0;
    dst[1] = w1;
    const float bhe = __half2float(he), bho = __half2float(ho), ble = __half2float(le), blo = __half2float(lo);
    xrow[idx] = make_float4(bhe + 16.f * bho, 1024.f * (bhe + bho), ble + 16.f * blo, 1024.f * (ble + blo));
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < nchunks * 2; idx += kThreads) {
    const float4* xr = xrow + idx * 16;
    float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      s4.x += xr[r].x;
      s4.y += xr[r].y;
      s4.z += xr[r].z;
      s4.w += xr[r].w;
    }
    xhalf[idx] = s4;
  }
  __syncthreads();

  const int g = lane >> 2, t = lane & 3;
  // As a B-operand provider this lane serves variant bv = g / 2 (0 A-hi, 1 A-lo,
  // 2 B-hi, 3 B-lo) with column select be = g % 2, for the row of quad lane t.
  const int bv = g >> 1, be = g & 1;
  const bool b_live = ((bv >= 2) == (t >= 2));
  const int b_off = ((bv & 1) * 2 + be) * 8;
  // As a D-fragment holder this lane owns variant t: chunk half t / 2, hi/lo t % 2.
  const int d_half = t >> 1, d_lo = t & 1;
  // Per-step shared-memory offsets of this lane (constant over chunks): the
  // weight row it provides (swizzled 16-byte group g) and its B fragment.
  uint32_t woff[8], xoff[8];
#pragma unroll
  for (int st = 0; st < 8; ++st) {
    const int h8 = st >> 2;
    const int p = (st & 1) + ((st & 2) << 1);  // 0, 1, 4, 5
    const int rA0 = 8 * h8 + p, rA1 = 8 * h8 + p + 2;
    const int rB0 = 16 + 8 * h8 + ((p + 4) & 7), rB1 = 16 + 8 * h8 + ((p + 6) & 7);
    const int row = (t == 0) ? rA0 : (t == 1) ? rA1 : (t == 2) ? rB0 : rB1;
    woff[st] = row * 128 + ((g ^ (row & 7)) << 4);
    xoff[st] = b_live ? (uint32_t)(row * kXRowBytes + b_off) : 0xFFFFFFFFu;
  }

  float2 acc[8];    // current tile segment: pairs (4j, 4j+2) -> acc[2j], (4j+1, 4j+3) -> acc[2j+1]
  float2 acc0[CLUSTER ? 1 : 8];  // first tile segment, when the warp's chunks cross a tile boundary
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < (CLUSTER ? 1 : 8); ++i) acc0[i] = make_float2(0.f, 0.f);
  int cur_tile = t_first;

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
    const int cl = c_first + i * kPhases - cs;
    const int s = i % kStages;
    if (!CLUSTER && tile != cur_tile) {  // warp-uniform, at most once
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        acc0[CLUSTER ? 0 : q] = acc[q];
        acc[q] = make_float2(0.f, 0.f);
      }
      cur_tile = tile;
    }
    const bool waited = a.sleep_wait ? sgd::mbar_wait_sleep(&my_bars[s], (i / kStages) & 1, a.err)
                                     : sgd::mbar_wait(&my_bars[s], (i / kStages) & 1, a.err);
    if (!__all_sync(0xffffffffu, waited)) {
      ok = 0;
      break;
    }
    const uint8_t* wst = smem + kOffW + (warp * kStages + s) * kWBytes;
    const uint8_t* xrows = xst + (size_t)cl * kRows * kXRowBytes;
    float d[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) d[j][q] = 0.f;
#pragma unroll
    for (int st = 0; st < 8; ++st) {
      const uint4 wv = *reinterpret_cast<const uint4*>(wst + woff[st]);
      const uint2 bw = *reinterpret_cast<const uint2*>(xoff[st] == 0xFFFFFFFFu ? zrow : xrows + xoff[st]);
      const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t e02, o02, e13, o13;
        nibbles_h(words[j], e02, o02, e13, o13);
        sgd::mma_f16_16816(d[j], e02, e13, o02, o13, bw.x, bw.y);
      }
    }
    // ---- chunk epilogue: acc += scale * (D - P - (8 + zero) * X) for this lane's variant
    const uint8_t* szs = smem + kOffSZ + (warp * kStages + s) * kSZBytes;
    const int k0 = 2 * crow * kRows;
    const int gA = group_of(a, k0), gB = group_of(a, k0 + 32);
    const int srow = d_half ? (gB - gA) : 0;
    const uint4 s_lo = *reinterpret_cast<const uint4*>(szs + srow * 256 + g * 32);
    const uint4 s_hi = *reinterpret_cast<const uint4*>(szs + srow * 256 + g * 32 + 16);
    const float4 xp = xhalf[cl * 2 + d_half];
    const float X = d_lo ? xp.z : xp.x;
    const float P = d_lo ? xp.w : xp.y;
    uint4 zv = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);  // biased zeros = 0
    if (HAS_Z) {
      zv = *reinterpret_cast<const uint4*>(szs + kSBytes + srow * 128 + g * 16);
      zv.x ^= 0x80808080u;
      zv.y ^= 0x80808080u;
      zv.z ^= 0x80808080u;
      zv.w ^= 0x80808080u;
    }
    const float2 mP = make_float2(-P, -P), XX = make_float2(X, X);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        // pair h: d[j][2h], d[j][2h+1] -> columns 4j+h and 4j+h+2
        const int ca = 4 * j + h, cb = 4 * j + h + 2;
        const float2 sc = make_float2(sgd::half16_at(s_lo, s_hi, ca), sgd::half16_at(s_lo, s_hi, cb));
        // 8 + zero: byte (zero ^ 0x80) placed in the mantissa of 2^23, minus (2^23 + 120)
        const uint32_t zwa = sgd::u4_get(zv, ca >> 2), zwb = sgd::u4_get(zv, cb >> 2);
        const float za = __uint_as_float(__byte_perm(zwa, 0x4B000000u, 0x7440 | (ca & 3)));
        const float zb = __uint_as_float(__byte_perm(zwb, 0x4B000000u, 0x7440 | (cb & 3)));
        const float2 z8 = sgd::ffma2(make_float2(za, zb), make_float2(-1.f, -1.f),
                                     make_float2(8388728.f, 8388728.f));  // -(z + 8)
        const float2 dp = sgd::ffma2(make_float2(d[j][2 * h], d[j][2 * h + 1]), make_float2(1.f, 1.f), mP);
        const float2 tq = sgd::ffma2(z8, XX, dp);
        acc[2 * j + h] = sgd::ffma2(sc, tq, acc[2 * j + h]);
      }
    }
    __syncwarp();
    if (lane == 0 && i + kStages < n_my) issue(i + kStages);
  }
  if (!ok) s_abort = 1;
  // segment index of the registers: acc0 holds the first tile when the warp crossed into a second
  const bool crossed = cur_tile != t_first;

  // ---- sum the 4 lanes of a quad (variants x halves)
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    acc[q].x += __shfl_xor_sync(0xffffffffu, acc[q].x, 1);
    acc[q].y += __shfl_xor_sync(0xffffffffu, acc[q].y, 1);
    acc[q].x += __shfl_xor_sync(0xffffffffu, acc[q].x, 2);
    acc[q].y += __shfl_xor_sync(0xffffffffu, acc[q].y, 2);
  }
  if (!CLUSTER) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int qq = CLUSTER ? 0 : q;
      acc0[qq].x += __shfl_xor_sync(0xffffffffu, acc0[qq].x, 1);
      acc0[qq].y += __shfl_xor_sync(0xffffffffu, acc0[qq].y, 1);
      acc0[qq].x += __shfl_xor_sync(0xffffffffu, acc0[qq].x, 2);
      acc0[qq].y += __shfl_xor_sync(0xffffffffu, acc0[qq].y, 2);
    }
  }
  __syncthreads();
  if (!CLUSTER && s_abort) return;

  // ---- block reduction over phases: red[seg][phase][512] aliases the weight stages.
  // Column of pair entry: acc[2j+h].x -> 4j+h, .y -> 4j+h+2.  Lane t writes tile j = t.
  float* red = reinterpret_cast<float*>(smem + kOffW);
  {
    const float2 a0 = t == 0 ? acc[0] : t == 1 ? acc[2] : t == 2 ? acc[4] : acc[6];
    const float2 a1 = t == 0 ? acc[1] : t == 1 ? acc[3] : t == 2 ? acc[5] : acc[7];
    const float2 b0 = CLUSTER ? make_float2(0.f, 0.f)
                              : (t == 0 ? acc0[0] : t == 1 ? acc0[CLUSTER ? 0 : 2] : t == 2 ? acc0[CLUSTER ? 0 : 4]
                                                                                           : acc0[CLUSTER ? 0 : 6]);
    const float2 b1 = CLUSTER ? make_float2(0.f, 0.f)
                              : (t == 0 ? acc0[CLUSTER ? 0 : 1] : t == 1 ? acc0[CLUSTER ? 0 : 3]
                                         : t == 2 ? acc0[CLUSTER ? 0 : 5] : acc0[CLUSTER ? 0 : 7]);
    // segment 0 = first tile of the block range, segment 1 = second
    const float2 s0e = crossed ? b0 : a0, s0o = crossed ? b1 : a1;
    const float2 s1e = crossed ? a0 : make_float2(0.f, 0.f), s1o = crossed ? a1 : make_float2(0.f, 0.f);
    float* r0 = red + (0 * kPhases + phase) * kTileCols + strip * 128 + g * 16 + 4 * t;
    float* r1 = red + (1 * kPhases + phase) * kTileCols + strip * 128 + g * 16 + 4 * t;
    r0[0] = s0e.x; r0[2] = s0e.y; r0[1] = s0o.x; r0[3] = s0o.y;
    r1[0] = s1e.x; r1[2] = s1e.y; r1[1] = s1o.x; r1[3] = s1o.y;
  }
  __syncthreads();

  if (CLUSTER) {
    // this block's partial of its tile; rank 0 of the cluster sums the ranks in order
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    float* tsum = red + 2 * kPhases * kTileCols;
    for (int cc = threadIdx.x; cc < kTileCols; cc += kThreads) {
      float v = 0.f;
#pragma unroll
      for (int ph = 0; ph < kPhases; ++ph) v += red[ph * kTileCols + cc];
      tsum[cc] = v;
    }
    cluster.sync();
    if (cluster.block_rank() == 0) {
      const int tile = blockIdx.y;
      int aborted = 0;
      for (int r = 0; r < a.ksplit; ++r) aborted |= *cluster.map_shared_rank(&s_abort, r);
      if (!aborted) {
        for (int cc = threadIdx.x; cc < kTileCols; cc += kThreads) {
          float v = 0.f;
          for (int r = 0; r < a.ksplit; ++r) v += cluster.map_shared_rank(tsum, r)[cc];
          const int col = tile * kTileCols + cc;
          if (col < a.N) store_out(a.C, a.c_dt, col, finalize(a, col, v));
        }
      }
    }
    cluster.sync();  // peers keep their shared memory alive until rank 0 has read it
    return;
  }

  const int t_last = (ce - 1) / a.cpt;
  for (int s2 = 0; s2 < 2 && t_first + s2 <= t_last; ++s2) {
    const int tile = t_first + s2;
    const int tc0 = tile * a.cpt;
    const int b_lo = block_of_chunk(a, tc0), b_hi = block_of_chunk(a, tc0 + a.cpt - 1);
    const bool shared_tile = b_lo != b_hi;
    for (int cc = threadIdx.x; cc < kTileCols; cc += kThreads) {
      float v = 0.f;
#pragma unroll
      for (int ph = 0; ph < kPhases; ++ph) v += red[(s2 * kPhases + ph) * kTileCols + cc];
      const int col = tile * kTileCols + cc;
      if (!shared_tile) {
        if (col < a.N) store_out(a.C, a.c_dt, col, finalize(a, col, v));
      } else {
        a.slots[((int64_t)b * 2 + s2) * kTileCols + cc] = v;
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
    for (int cc = threadIdx.x; cc < kTileCols; cc += kThreads) {
      const int col = tile * kTileCols + cc;
      float v = 0.f;
      for (int bb = b_lo; bb <= b_hi; ++bb) {
        int bcs, bce;
        block_range(a, bb, bcs, bce);
        const int sb = tile - bcs / a.cpt;
        v += __ldcg(&a.slots[((int64_t)bb * 2 + sb) * kTileCols + cc]);
      }
      if (col < a.N) store_out(a.C, a.c_dt, col, finalize(a, col, v));
    }
    if (threadIdx.x == 0) a.tickets[tile] = 0u;
  }
}

struct MPlan {
  bool ok = false;
  int variant = 0;
  int cluster = 0, ksplit = 1;
  int n_tiles = 0, cpt = 0, nblocks = 0, flat = 0, max_chunks = 0, total = 0;
  size_t smem = 0, ws_bytes = 0, tickets_bytes = 0;
};

// Clusters of k blocks (one per SM: the kernel's shared memory allows one
// block per SM) that can be resident at once.
int max_active_clusters(int k) {
  static std::mutex mu;
  static int cache[17] = {0};
  std::lock_guard<std::mutex> lk(mu);
  if (k < 1 || k > 16) return 0;
  if (cache[k] != 0) return cache[k];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(k, 1);
  cfg.blockDim = dim3(512);
  cfg.dynamicSmemBytes = 225 * 1024;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = k;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  auto kfn = w4_gemv_mma_kernel<true, 16, 2, true>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024) != cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = -1;
  }
  cache[k] = n;
  return n;
}

MPlan make_mplan(const SgMatMulParams* p, int sms) {
  MPlan pl;
  const int gs = p->group_size > 0 ? p->group_size : 128;
  if (p->M != 1 || p->K <= 0 || (p->N % 16) != 0 || (gs % 32) != 0) return pl;
  if (!sg::aligned16(p->B) || !sg::aligned16(p->scales_B) || (p->zeros_B && !sg::aligned16(p->zeros_B))) return pl;
  const int KP = (p->K + 1) / 2;
  pl.n_tiles = (p->N + kTileCols - 1) / kTileCols;
  pl.cpt = (KP + kRows - 1) / kRows;
  const long long total = (long long)pl.n_tiles * pl.cpt;
  if (total >= (1ll << 30)) return pl;
  pl.total = (int)total;
  // Cluster mode when a tile-aligned split with <= 8 blocks per tile runs in
  // one wave (clusters must fit inside a GPC) and fills most SMs.
  int ks = 0;
  if (g_cluster_mode.load()) {
    for (int k = std::min({8, pl.cpt, pl.n_tiles > 0 ? sms / pl.n_tiles : 0}); k >= 2; --k) {
      if (pl.n_tiles * k < (sms * 3) / 4) break;
      if (max_active_clusters(k) >= pl.n_tiles) {
        ks = k;
        break;
      }
    }
  }
  if (ks >= 2) {
    pl.cluster = 1;
    pl.ksplit = ks;
    pl.flat = 0;
    pl.nblocks = pl.n_tiles * ks;
    pl.max_chunks = (pl.cpt + ks - 1) / ks;
  } else if (pl.n_tiles <= sms) {
    pl.flat = 1;
    pl.nblocks = (int)std::min<long long>(sms, total);
    pl.max_chunks = (int)((total + pl.nblocks - 1) / pl.nblocks);
  } else {
    pl.flat = 0;
    pl.nblocks = pl.n_tiles;
    pl.max_chunks = pl.cpt;
  }
  pl.variant = std::min(3, std::max(0, g_variant.load()));
  const int vw = kVariantWarps[pl.variant], vs = kVariantStages[pl.variant];
  pl.smem = 1024 + off_x(vw, vs) + (size_t)pl.max_chunks * (kRows * kXRowBytes + kRows * 16 + 2 * 16) + 16 +
            vw * vs * 8;
  // opt-in limit per block (227 KB on sm_100) minus this kernel's static shared memory
  if (pl.smem > 227 * 1024 - kStaticSmemReserve) return pl;
  if (pl.cluster) {
    pl.tickets_bytes = 0;
    pl.ws_bytes = 0;  // partials stay in distributed shared memory
  } else {
    pl.tickets_bytes = sg::ticket_bytes(pl.n_tiles);
    pl.ws_bytes = pl.tickets_bytes + (size_t)pl.nblocks * 2 * kTileCols * sizeof(float);
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
                         int* err_word, bool* handled) {
  *handled = false;
  const MPlan pl = make_mplan(p, sms);
  if (!pl.ok) return SG_OK;
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
  a.flat = pl.flat;
  a.total = pl.total;
  a.max_chunks = pl.max_chunks;
  a.ksplit = pl.ksplit;
  a.gs_shift = ((gs & (gs - 1)) == 0) ? __builtin_ctz((unsigned)gs) : -1;
  a.sleep_wait = g_sleep.load() ? 1 : 0;
  a.tickets = static_cast<unsigned*>(ws);
  a.slots = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.tickets_bytes);
  a.err = err_word;

  using KFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, MArgs);
#define SG_W4MMA_KFNS(Z, C)                                                                              \
  {w4_gemv_mma_kernel<Z, 16, 2, C>, w4_gemv_mma_kernel<Z, 20, 2, C>, w4_gemv_mma_kernel<Z, 12, 3, C>, \
   w4_gemv_mma_kernel<Z, 8, 5, C>}
  static const KFn kfns[2][2][4] = {{SG_W4MMA_KFNS(false, false), SG_W4MMA_KFNS(false, true)},
                                    {SG_W4MMA_KFNS(true, false), SG_W4MMA_KFNS(true, true)}};
#undef SG_W4MMA_KFNS
  const int zi = a.has_zeros ? 1 : 0, ci = pl.cluster ? 1 : 0;
  const KFn kfn = kfns[zi][ci][pl.variant];
  static std::mutex mu;
  static size_t attr_smem[2][2][4] = {};
  {
    std::lock_guard<std::mutex> lk(mu);
    size_t& done = attr_smem[zi][ci][pl.variant];
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
  if (key == "w4_gemv_mma.sleep") {
    g_sleep.store(value);
    return true;
  }
  return false;
}

}  // namespace sg
