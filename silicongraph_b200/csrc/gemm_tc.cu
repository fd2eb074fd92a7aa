// Prefill dequant-GEMM on the 5th-generation tensor cores (tcgen05 + TMEM):
//   C[m, n] = sum_k A[m, k] * W[k, n]
// with W held as the reference's INT4 group-quantized layout
// (compiler/kernels/cpu/matmul_neon.h:113-147, per-row semantics applied to
// every row m) or as INT8 per-channel weights with float activations
// (dense GEMV FA form: C = scales[n] * sum_k A*float(B), opencl_kernels.h:36-52
// restated for float A).
//
// Design (one persistent CTA per SM, 768 threads with two dequant groups,
// warp-specialised; roles listed below the constants):
//   * The weights are the MMA's A operand and live in TMEM: dequant warps read
//     the packed bytes that TMA staged in shared memory, expand them in
//     registers (fp16(scale * (q - 8 - zero)) for INT4, exact integers for
//     INT8) and write them with tcgen05.st.  The dequantized weights never
//     touch shared memory, which leaves the shared-memory bandwidth to the
//     activation operand.
//   * The activations are the MMA's B operand: TMA copies [BT tokens x 64 k]
//     tiles (128-byte swizzle, K-major) into shared memory.
//   * One thread issues tcgen05.mma (M = 128 weight columns, N = BT tokens,
//     K = 16) into a TMEM accumulator of 128 lanes x BT columns.
//   * Four epilogue warps (one per TMEM lane quarter) read the accumulator
//     with tcgen05.ld, apply scale_A / per-channel scales / bias and store C.
//     With two accumulators (token tiles up to 192) the epilogue of one tile
//     overlaps the main loop of the next; the 256-token tile has room for one,
//     and the MMA waits for its epilogue at each tile boundary.
//   * A last round of tiles that fills at most half of the SMs runs as two k
//     halves per tile (fp32 partials in the scratch, added by the second half
//     to finish); optionally, clusters of two CTAs share each MMA
//     (tcgen05 cta_group::2, 256 weight columns per tile).
//   * Every wait is bounded (2 s); a timed-out wait records an error code in
//     the device error word, the CTA drains its copies in flight, frees TMEM
//     and exits.
//
// Tile size: 128 weight columns (the TMEM lanes) x BT tokens, K step 64.
// Operand type: fp16 for INT4 weights (bf16 weights would round
// scale*(q-8-zero) to 8 significant bits, too coarse for the 2e-3 absolute
// tolerance at K = 2048); for INT8 weights the integers are exact in either
// type, so bf16 activations are used as they are.  Activations in other types
// are first converted to the operand type by a small kernel (exact for int8
// and for bf16 -> fp16 within fp16's range; fp32 rounds to fp16).
#include <algorithm>
#include <atomic>
#include <string_view>

#include "sm100.cuh"

namespace {

using namespace sgd;

constexpr int kKStep = 64;    // k per pipeline step: one 128-byte swizzle row of 16-bit values
constexpr int kWCols = 128;   // weight columns per tile = TMEM lanes = UMMA M
// Warp roles.  Warps 0..3: epilogue, TMEM lane quarter = warp.  Then 8 * PAR
// dequant warps: lane quarter = warp % 4, k half of the step = bit 2 of the
// dequant index, and with PAR = 2 the step parity = bit 3 (two steps are
// dequantized concurrently).  Then three TMA producer warps (activation
// tiles; packed weights; scale and zero rows) and the MMA warp.  One thread
// cannot issue tcgen05.mma faster than about one per 120 cycles, and under the
// kernel's load one thread issues a TMA copy only every ~450 cycles (per-role
// clock64 timeline: with weights and scales on one thread, that thread set the
// pace of the whole pipeline at ~920 cycles per 64-k step), so every
// single-thread role gets its own warp and each producer issues one copy per step.
constexpr int kEpiWarps = 4;
constexpr int kStepWarps = 8;  // dequant warps that complete one step (4 quarters x 2 k halves)
__host__ __device__ constexpr int prep_warps(int par) { return kStepWarps * par; }
__host__ __device__ constexpr int warp_tma_act(int par) { return kEpiWarps + prep_warps(par); }
__host__ __device__ constexpr int warp_tma_w(int par) { return warp_tma_act(par) + 1; }
__host__ __device__ constexpr int warp_tma_s(int par) { return warp_tma_w(par) + 1; }
__host__ __device__ constexpr int warp_mma(int par) { return warp_tma_s(par) + 1; }
__host__ __device__ constexpr int threads_of(int par) { return (warp_mma(par) + 1) * 32; }
constexpr int kOutChunk = 32;                         // tokens per epilogue TMA store
constexpr int kOutBuf = kOutChunk * 128 * 2;          // one 16-bit [32 x 128] staging tile
constexpr int kOutBufs = 3;                           // staging ring (one barrier per chunk)
constexpr int kEpiBarrier = 1;                        // named barrier of the epilogue warps
constexpr int kTmemCols = 512;

enum WKind : int { kW4Grouped = 0, kW8Channel = 1 };

// PAIR: two CTAs of a cluster share one MMA (tcgen05 cta_group::2) over 256
// weight columns x BT tokens; each holds its 128 columns in TMEM and half of
// the tokens' activations in shared memory.
template <int BT, int WK, bool PAIR = false>
struct Cfg {
  static constexpr int kActRows = PAIR ? BT / 2 : BT;                     // token rows of this CTA
  static constexpr int kActBytes = kActRows * 128;                       // rows x 64 x 16-bit
  static constexpr int kWBytes = (WK == kW4Grouped ? kKStep / 2 : kKStep) * kWCols;  // packed rows x 128
  static constexpr int kSBytes = (WK == kW4Grouped) ? 4 * kWCols * 2 : 0;          // <= 4 scale rows
  static constexpr int kZBytes = (WK == kW4Grouped) ? 4 * kWCols : 0;              // <= 4 zero rows
  static constexpr int kStageBytes = kActBytes + kWBytes + kSBytes + kZBytes;
  static constexpr int kStride = (kStageBytes + 1023) / 1024 * 1024;  // act tile stays 1024-aligned
  static constexpr int kAcc = (2 * BT + 4 * 32 <= kTmemCols) ? 2 : 1;
  // Two rings: shared-memory stages (TMA -> dequant / MMA) and TMEM slots of
  // dequantized weights (dequant -> MMA), each as deep as its memory allows.
  static constexpr int kSlots0 = (kTmemCols - kAcc * BT) / 32;
  static constexpr int kSlots = kSlots0 > 8 ? 8 : kSlots0;
  static constexpr int kStages0 = (227 * 1024 - 2048 - kOutBufs * kOutBuf) / kStride;
  static constexpr int kStages = kStages0 > 12 ? 12 : kStages0;
  static constexpr int kBarBytes = (2 * kStages + 2 * kSlots + 2 * 2 + 2) * 8 + 16;
  static constexpr int kOutOff = kStages * kStride;  // epilogue staging ring
  static constexpr int kBarOff = kOutOff + kOutBufs * kOutBuf;
  static constexpr int kSmem = kBarOff + kBarBytes + 1024;  // + alignment slack
  static_assert(kStages >= 2 && kSlots >= 2, "pipeline needs two stages");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
  static_assert(BT % 32 == 0 && BT >= 32 && BT <= 256, "token tile");
  // the other half's fp32 sums of a split tile land in the (then idle) stage ring
  static_assert(BT * kWCols * 4 <= kStages * kStride, "split-tile partial fits the stage ring");
};

struct GArgs {
  void* C;
  const __half* bias;    // INT4: fp16 [N] or NULL
  const float* scales;   // INT8: f32 [N]
  float scale_A;
  int apply_scale_A;     // INT4 with int8 activations
  int c_dt;
  int ldc;
  int M, N, K;
  int gs;                // INT4 group size
  int ksteps;
  int n_tiles, m_tiles;
  int spin;       // 1: single-thread waits spin on test_wait
  int tma_store;  // 1: 16-bit C written by TMA stores from shared memory
  int* err;
  // Work units: tiles 0 .. whole-1 whole, then each remaining tile as two k
  // halves (units whole .. units-1), which two CTAs of the last round compute.
  int whole, units;
  unsigned* tickets;  // [tiles - whole], zero between calls
  float* partials;    // [tiles - whole][2][BT tokens][128 columns] fp32
};

// Unit u of the launch: a whole tile, or one k half of a tile of the last
// round.  Both halves write their fp32 sums to the scratch; the one that
// finishes second adds the other's and writes C.  The two-term sum does not
// depend on which half finished first, so results are the same on every run.
struct Unit {
  int tile, k0, k1;
  int slot;  // split tile index (-1: whole tile)
  int half;
};
__device__ __forceinline__ Unit unit_of(const GArgs& a, int u) {
  Unit r;
  if (u < a.whole) {
    r.tile = u;
    r.k0 = 0;
    r.k1 = a.ksteps;
    r.slot = -1;
    r.half = 0;
  } else {
    const int v = u - a.whole, kh = a.ksteps >> 1;
    r.slot = v >> 1;
    r.half = v & 1;
    r.tile = a.whole + r.slot;
    r.k0 = r.half ? kh : 0;
    r.k1 = r.half ? a.ksteps : kh;
  }
  return r;
}

// ---------------------------------------------------------------- CTA pairs
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of both CTAs; orders shared-memory writes (barrier inits) before what follows.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of CTA 0 of the pair (address from cluster_addr).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait (as mbar_wait) on a barrier that CTAs of the pair arrive on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      record_error(err, kErrWaitTimeout);
      return false;
    }
  }
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (+)= A * B over the pair: M = 256 (A: 128 rows in each CTA's TMEM), B's N
// columns split between the two CTAs' shared memory at the same address.
__device__ __forceinline__ void umma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at this offset in both CTAs of the pair when the MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

// Bulk copy global -> this CTA's shared memory, completing on an mbarrier.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t lop3_and_or_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
  return d;
}
__device__ __forceinline__ uint32_t lop3_xor_or_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xBE;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a ^ b) | c
  return d;
}
__device__ __forceinline__ uint32_t h2_as_u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ uint32_t ld_shared_u8(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t ld_shared_u16(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// 32 finished values (tokens) of one output column -> C rows base, base + ldc, ...
template <int DT>
__device__ __forceinline__ void epi_store(const uint32_t (&r)[32], int cnt, const GArgs& a, int64_t base) {
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < cnt) store_from_float<DT>(a.C, base + (int64_t)j * a.ldc, __uint_as_float(r[j]));
}

// Bounded wait by every lane of a warp, then reconvergence.  A lane whose
// wait times out raises the CTA abort flag; the warp still finishes the
// current step (its results are then invalid and the device error word says
// so) and leaves at the next step, where all lanes read the flag together.
// Every lane waits itself: electing one lane and broadcasting its result
// costs about three times as much per wait.
__device__ __forceinline__ void warp_wait(uint64_t* bar, uint32_t parity, int* err, int spin,
                                          volatile int* abort_flag) {
  const bool ok = spin ? mbar_wait_spin(bar, parity, err) : mbar_wait(bar, parity, err);
  if (!ok) *abort_flag = 1;
  __syncwarp();
}

// Named barrier of the 128 epilogue threads; returns the OR of pred over them.
__device__ __forceinline__ bool epi_bar_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n"
      " barrier.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(kEpiBarrier), "n"(kEpiWarps * 32)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("barrier.sync %0, %1;" ::"n"(kEpiBarrier), "n"(kEpiWarps * 32) : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(smem_src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_le1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint16_t to_out16(float v, int dt) {
  if (dt == SG_DT_BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  return __half_as_ushort(__float2half_rn(v));
}

// BT tokens per tile; WK weight kind; BF16_OP: operand type (INT8 with bf16 activations); HAS_Z: INT4 zeros;
// PAIR: clusters of two CTAs share each MMA (tiles of 256 weight columns; a.n_tiles counts those).
template <int BT, int WK, bool BF16_OP, bool HAS_Z, int PAR, bool PAIR>
__global__ void __launch_bounds__(threads_of(PAR), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmAct, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmZ,
                   const __grid_constant__ CUtensorMap tmC, GArgs a) {
  using C_ = Cfg<BT, WK, PAIR>;
  constexpr int kTileCols = PAIR ? 2 * kWCols : kWCols;  // weight columns per tile
  constexpr int S = C_::kStages, J = C_::kSlots, kAcc = C_::kAcc;
  constexpr int kWarpAct = warp_tma_act(PAR), kWarpW = warp_tma_w(PAR), kWarpS = warp_tma_s(PAR);
  constexpr int kWarpMma = warp_mma(PAR);
  constexpr int kProducers = WK == kW4Grouped ? 3 : 2;  // INT8 weights have no scale rows to stage
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = sgd::align_smem_1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_::kBarOff);
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;
  uint64_t* aempty = afull + J;
  uint64_t* accfull = aempty + J;
  uint64_t* accempty = accfull + 2;
  uint64_t* done = accempty + 2;
  uint64_t* pfull = done + 1;  // the other half's partial of a split tile has arrived
  uint32_t* tslot = reinterpret_cast<uint32_t*>(pfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  volatile int* last_half = abort_flag + 1;  // epilogue: this CTA finishes its split tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // In a pair, CTA 0 issues the MMAs: the dequant and epilogue warps of both CTAs
  // arrive on its afull / accempty, and its commits reach the barriers of both.
  const uint32_t rank = PAIR ? cluster_rank() : 0;
  const int cta0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;   // this CTA's (pair's) index
  const int nctas = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], kProducers);  // one expect_tx arrival per producer
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < J; ++j) {
      mbar_init(&afull[j], kStepWarps * (PAIR ? 2 : 1));
      mbar_init(&aempty[j], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], kEpiWarps * (PAIR ? 2 : 1));
    }
    mbar_init(done, 1);
    mbar_init(pfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMma) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tslot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tslot, kTmemCols);
      tmem_relinquish();
    }
  }
  if (warp == kWarpAct && lane == 0) tma_prefetch_desc(&tmAct);
  if (warp == kWarpW && lane == 0) tma_prefetch_desc(&tmW);
  if (warp == kWarpS && lane == 0 && WK == kW4Grouped) {
    tma_prefetch_desc(&tmS);
    if (HAS_Z) tma_prefetch_desc(&tmZ);
  }
  if (warp == 0 && lane == 0 && a.tma_store) tma_prefetch_desc(&tmC);
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // both CTAs' barriers exist before either arrives on the other's
  tc_fence_after();
  const uint32_t tbase = *tslot;
  // Inputs written by the preceding kernel on the stream are visible after this.
  pdl_wait();

  if (warp == kWarpAct || warp == kWarpW || warp == kWarpS) {
    // ------------------------------------------------------------ TMA producers
    if (lane == 0 && (warp != kWarpS || WK == kW4Grouped)) {
      const bool is_act = warp == kWarpAct, is_w = warp == kWarpW;
      uint32_t issued[S];
      for (int s = 0; s < S; ++s) issued[s] = 0;
      const int gs = a.gs;
      const int srows = gs >= kKStep ? 1 : kKStep / gs;
      const uint32_t bytes = is_act ? (uint32_t)C_::kActBytes
                             : is_w ? (uint32_t)C_::kWBytes
                                    : (uint32_t)(srows * kWCols * 2 + (HAS_Z ? srows * kWCols : 0));
      uint32_t g = 0;
      bool ok = true;
      for (int u = cta0; u < a.units && ok; u += nctas) {
        const Unit un = unit_of(a, u);
        const int n0 = (un.tile % a.n_tiles) * kTileCols + (int)rank * kWCols;
        const int m0 = (un.tile / a.n_tiles) * BT + (int)rank * C_::kActRows;
        for (int ks = un.k0; ks < un.k1; ++ks, ++g) {
          const int s = g % S;
          const uint32_t use = g / S;
          if (*abort_flag || !(a.spin ? mbar_wait_spin(&empty[s], (use & 1) ^ 1, a.err)
                                      : mbar_wait(&empty[s], (use & 1) ^ 1, a.err))) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          unsigned char* st = smem + s * C_::kStride;
          mbar_arrive_expect_tx(&full[s], bytes);
          if (is_act) {
            tma_load_2d(st, &tmAct, ks * kKStep, m0, &full[s]);
          } else if (is_w) {
            tma_load_2d(st + C_::kActBytes, &tmW, n0, WK == kW4Grouped ? ks * (kKStep / 2) : ks * kKStep, &full[s]);
          } else {
            const int grow = (ks * kKStep) / gs;
            tma_load_2d(st + C_::kActBytes + C_::kWBytes, &tmS, n0, grow, &full[s]);
            if (HAS_Z) tma_load_2d(st + C_::kActBytes + C_::kWBytes + C_::kSBytes, &tmZ, n0, grow, &full[s]);
          }
          issued[s] = use + 1;
        }
      }
      // Drain: every copy issued into this CTA's shared memory completes before exit.
      for (int s = 0; s < S; ++s)
        if (issued[s]) mbar_wait(&full[s], (issued[s] - 1) & 1, a.err);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = umma_idesc_f16(PAIR ? 2 * kWCols : kWCols, BT, BF16_OP ? 1 : 0, 0, 0);
      uint32_t g = 0;
      int lt = 0;
      bool ok = true;
      for (int u = cta0; u < a.units && ok; u += nctas, ++lt) {
        const Unit un = unit_of(a, u);
        const int acc = lt % kAcc;
        const uint32_t ause = lt / kAcc;
        if (*abort_flag || !(PAIR ? mbar_wait_cluster(&accempty[acc], (ause & 1) ^ 1, a.err)
                                  : mbar_wait(&accempty[acc], (ause & 1) ^ 1, a.err))) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dt = tbase + acc * BT;
        for (int ks = un.k0; ks < un.k1; ++ks, ++g) {
          const int s = g % S, j = g % J;
          const uint32_t juse = g / J;
          // The dequant warps (in a pair: of both CTAs) arrive on afull[j] only after they
          // observed full[s], which also covers the activation tile of this stage.
          if (*abort_flag || !(PAIR     ? mbar_wait_cluster(&afull[j], juse & 1, a.err)
                               : a.spin ? mbar_wait_spin(&afull[j], juse & 1, a.err)
                                        : mbar_wait(&afull[j], juse & 1, a.err))) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = umma_smem_desc(smem_u32(smem + s * C_::kStride), 16, 1024, kSwizzle128B);
          const uint32_t at = tbase + kAcc * BT + j * 32;
          if constexpr (PAIR) {
#pragma unroll
            for (int kk = 0; kk < kKStep / 16; ++kk)
              umma_f16_ts_pair(dt, at + kk * 8, bdesc + (uint64_t)(kk * 2), idesc,
                               (ks != un.k0 || kk != 0) ? 1u : 0u);
            umma_commit_pair(&empty[s]);
            umma_commit_pair(&aempty[j]);
          } else {
#pragma unroll
            for (int kk = 0; kk < kKStep / 16; ++kk)
              umma_f16_ts(dt, at + kk * 8, bdesc + (uint64_t)(kk * 2), idesc, (ks != un.k0 || kk != 0) ? 1u : 0u);
            umma_commit(&empty[s]);
            umma_commit(&aempty[j]);
          }
        }
        if (ok) {
          if constexpr (PAIR)
            umma_commit_pair(&accfull[acc]);
          else
            umma_commit(&accfull[acc]);
        }
      }
      if constexpr (PAIR)
        umma_commit_pair(done);
      else
        umma_commit(done);
    }
    // Every MMA (which in a pair also writes the other CTA's TMEM) is complete before TMEM is freed.
    if (lane == 0) mbar_wait(done, 0, a.err);
  } else if (warp >= kEpiWarps) {
    // ------------------------------------------------------------ dequant warps
    const int pw = warp - kEpiWarps;
    const int q = warp & 3, h = (pw >> 2) & 1, par = pw >> 3;
    const int col = q * 32 + lane;  // column within the tile = TMEM lane
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    uint32_t g = 0;
    bool ok = true;
    for (int u = cta0; u < a.units && ok; u += nctas) {
      const Unit un = unit_of(a, u);
      for (int ks = un.k0; ks < un.k1; ++ks, ++g) {
        if (PAR > 1 && (int)(g % PAR) != par) continue;
        __syncwarp();
        if (*abort_flag) {  // one shared load of a converged warp: the same value in every lane
          ok = false;
          break;
        }
        const int s = g % S, j = g % J;
        const uint32_t use = g / S, juse = g / J;
        warp_wait(&full[s], use & 1, a.err, a.spin, abort_flag);
        warp_wait(&aempty[j], (juse & 1) ^ 1, a.err, a.spin, abort_flag);
        tc_fence_after();
        const uint32_t wbase = smem_u32(smem + s * C_::kStride + C_::kActBytes);
        if (WK == kW4Grouped) {
          // rows 16h .. 16h+15 of the packed tile: k = 32h .. 32h+31 of this step
          uint32_t w[16];
          const uint32_t sbase = wbase + C_::kWBytes;
          const uint32_t zbase = sbase + C_::kSBytes;
          const int gs = a.gs;
          // scale rows of this half: rows 0..7 and 8..15 (differ only for groups of 16)
          const int g0 = gs >= kKStep ? 0 : (32 * h) / gs;
          const int g1 = gs >= kKStep ? 0 : (32 * h + 16) / gs;
          const __half2 s0 = __half2half2(__ushort_as_half((unsigned short)ld_shared_u16(sbase + (g0 * kWCols + col) * 2)));
          const __half2 s1 = __half2half2(__ushort_as_half((unsigned short)ld_shared_u16(sbase + (g1 * kWCols + col) * 2)));
          int z0 = 0, z1 = 0;
          if (HAS_Z) {
            z0 = (int)(int8_t)ld_shared_u8(zbase + g0 * kWCols + col);
            z1 = (int)(int8_t)ld_shared_u8(zbase + g1 * kWCols + col);
          }
          const __half2 c0 = __half2half2(__int2half_rn(1032 + z0));
          const __half2 c1 = __half2half2(__int2half_rn(1032 + z1));
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint32_t b = ld_shared_u8(wbase + (16 * h + i) * kWCols + col);
            // (1024 + low nibble, 1024 + high nibble) as fp16x2
            const uint32_t x = lop3_and_or_u(b | (b << 12), 0x000F000Fu, 0x64006400u);
            const __half2 t = __hsub2(u_as_h2(x), i < 8 ? c0 : c1);  // q - 8 - zero, exact
            w[i] = h2_as_u(__hmul2(t, i < 8 ? s0 : s1));              // fp16(scale * (q - 8 - zero))
          }
          tmem_st_32x32b_x16(tbase + lane_addr + kAcc * BT + j * 32 + 16 * h, w);
        } else {
          // rows 32h .. 32h+31 of the int8 tile: k = 32h .. 32h+31 of this step, in two passes of 16
#pragma unroll 1
          for (int o = 0; o < 2; ++o) {
            uint32_t w8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 32 * h + 16 * o + 2 * i;
              const uint32_t b0 = ld_shared_u8(wbase + r * kWCols + col);
              const uint32_t b1 = ld_shared_u8(wbase + (r + 1) * kWCols + col);
              if (BF16_OP) {
                __nv_bfloat162 v = __floats2bfloat162_rn((float)(int)(int8_t)b0, (float)(int)(int8_t)b1);
                w8[i] = *reinterpret_cast<uint32_t*>(&v);  // integers: exact
              } else {
                // (1024 + (q + 128)) - 1152 = q, exact in fp16
                const uint32_t x = lop3_xor_or_u(b0 | (b1 << 16), 0x00800080u, 0x64006400u);
                w8[i] = h2_as_u(__hsub2(u_as_h2(x), __half2half2(__int2half_rn(1152))));
              }
            }
            tmem_st_32x32b_x8(tbase + lane_addr + kAcc * BT + j * 32 + 16 * h + 8 * o, w8);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR && rank != 0)
            mbar_arrive_remote(cluster_addr(&afull[j], 0));
          else
            mbar_arrive(&afull[j]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int q = warp;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const int col = q * 32 + lane;
    unsigned char* out_ring = smem + C_::kOutOff;
    uint32_t chunk = 0;  // chunks stored so far: staging buffer = chunk % kOutBufs
    int lt = 0;
    for (int u = cta0; u < a.units; u += nctas, ++lt) {
      const Unit un = unit_of(a, u);
      const int acc = lt % kAcc;
      const uint32_t ause = lt / kAcc;
      const bool ok = *abort_flag == 0 && mbar_wait_sleep(&accfull[acc], ause & 1, a.err);
      // The four epilogue warps leave together (they share a named barrier below).
      if (epi_bar_or(!ok)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const float* other = nullptr;  // split tile, second half to finish: the first half's sums (shared memory)
      if (un.slot >= 0) {
        // Both halves store their raw fp32 sums, token-major ([token][128 columns], coalesced), then
        // take a ticket; the second to arrive adds the other's sums below.  A split tile is the
        // last unit of its CTA, so its accumulator is not reused and the stage ring is idle.
        float* mine = a.partials + (size_t)(un.slot * 2 + un.half) * BT * kWCols;
#pragma unroll 1
        for (int c = 0; c < BT / kOutChunk; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + lane_addr + acc * BT + c * kOutChunk, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) mine[(size_t)(c * kOutChunk + j) * kWCols + col] = __uint_as_float(r[j]);
        }
        __threadfence();
        epi_bar_sync();
        if (threadIdx.x == 0) {
          const unsigned prev = atomicAdd(&a.tickets[un.slot], 1u);
          *last_half = prev == 1u;
          if (prev == 1u) a.tickets[un.slot] = 0;  // zero again for the next call
        }
        epi_bar_sync();
        if (!*last_half) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[acc]);
          continue;
        }
        const float* theirs = a.partials + (size_t)(un.slot * 2 + (un.half ^ 1)) * BT * kWCols;
        float* ring = reinterpret_cast<float*>(smem);
        if (threadIdx.x == 0) {
          __threadfence();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(pfull, (uint32_t)(BT * kWCols * 4));
          for (int c = 0; c < BT / kOutChunk; ++c)
            bulk_load(ring + c * kOutChunk * kWCols, theirs + (size_t)c * kOutChunk * kWCols,
                      (uint32_t)(kOutChunk * kWCols * 4), pfull);
        }
        const bool got = mbar_wait_sleep(pfull, 0, a.err);
        if (epi_bar_or(!got)) {
          *abort_flag = 1;
          break;
        }
        other = ring;
      }
      const int n0 = (un.tile % a.n_tiles) * kTileCols + (int)rank * kWCols;
      const int n = n0 + col;
      const int m0 = (un.tile / a.n_tiles) * BT;
      const bool nvalid = n < a.N;
      float mul = 1.f, add = 0.f;
      if (nvalid) {
        if (WK == kW8Channel) mul = a.scales[n];
        if (WK == kW4Grouped && a.bias) add = __half2float(a.bias[n]);
      }
      const int mrows = min(BT, a.M - m0);
#pragma unroll 1
      for (int c = 0; c < BT / kOutChunk; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + lane_addr + acc * BT + c * kOutChunk, r);
        tmem_ld_wait();
        if (c == BT / kOutChunk - 1) {  // accumulator read out: the MMA may reuse it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (PAIR && rank != 0)
              mbar_arrive_remote(cluster_addr(&accempty[acc], 0));
            else
              mbar_arrive(&accempty[acc]);
          }
        }
        if (c * kOutChunk >= mrows) continue;  // uniform over the epilogue warps
        if (other != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), other[(c * kOutChunk + j) * kWCols + col]));
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float v = __uint_as_float(r[j]);
          if (WK == kW4Grouped) {
            if (a.apply_scale_A) v = __fmul_rn(v, a.scale_A);
            v = __fadd_rn(v, add);
          } else {
            v = __fmul_rn(v, mul);
          }
          r[j] = __float_as_uint(v);
        }
        if (a.tma_store) {
          // [32 tokens x 128 columns] 16-bit tile, then one TMA store (clipped at M and N).
          // The buffer written now was last read by the store of chunk - 3, which thread 0
          // waited for before it arrived at the previous chunk's barrier.
          unsigned char* buf = out_ring + (chunk % kOutBufs) * kOutBuf;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            *reinterpret_cast<uint16_t*>(buf + j * 256 + col * 2) = to_out16(__uint_as_float(r[j]), a.c_dt);
          fence_proxy_async_smem();
          epi_bar_sync();
          if (threadIdx.x == 0) {
            tma_store_2d(&tmC, buf, n0, m0 + c * kOutChunk);
            bulk_commit();
            bulk_wait_read_le1();
          }
          ++chunk;
        } else if (nvalid) {
          const int cnt = min(32, mrows - c * kOutChunk);
          const int64_t base = (int64_t)(m0 + c * kOutChunk) * a.ldc + n;
          switch (a.c_dt) {
            case SG_DT_F32: epi_store<SG_DT_F32>(r, cnt, a, base); break;
            case SG_DT_BF16: epi_store<SG_DT_BF16>(r, cnt, a, base); break;
            default: epi_store<SG_DT_F16>(r, cnt, a, base); break;
          }
        }
      }
    }
    if (threadIdx.x == 0 && a.tma_store) bulk_wait_all();  // stores done before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  // A pair leaves together: no CTA exits while the other may still arrive on its barriers.
  if constexpr (PAIR) cluster_sync_all();
  if (warp == kWarpMma) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tbase, kTmemCols);
    else
      tmem_dealloc(tbase, kTmemCols);
  }
}

// Activations -> 16-bit operand type, rows padded to ld_out (zero-filled
// beyond K).  Grid: x over 8-element chunks of a row, y over rows.
template <bool TO_BF16>
__global__ void act_convert_kernel(const void* A, int a_dt, int lda, int M, int K, int ld_out, void* out) {
  const int k0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (k0 >= ld_out) return;
  for (int m = blockIdx.y; m < M; m += gridDim.y) {
    const int64_t j = (int64_t)m * lda + k0;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[e] = 0.f;
      if (k0 + e < K) {
        switch (a_dt) {
          case SG_DT_F32: v[e] = load_as_float<SG_DT_F32>(A, j + e); break;
          case SG_DT_F16: v[e] = load_as_float<SG_DT_F16>(A, j + e); break;
          case SG_DT_BF16: v[e] = load_as_float<SG_DT_BF16>(A, j + e); break;
          default: v[e] = load_as_float<SG_DT_I8>(A, j + e); break;
        }
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (TO_BF16) {
        __nv_bfloat162 t = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
        ow[e] = *reinterpret_cast<uint32_t*>(&t);
      } else {
        __half2 t = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
        ow[e] = *reinterpret_cast<uint32_t*>(&t);
      }
    }
    *reinterpret_cast<uint4*>(static_cast<unsigned char*>(out) + ((int64_t)m * ld_out + k0) * 2) = o;
  }
}

// The converted activations start this far into the scratch, so that a
// caller's workspace keeps the zeroed ticket counters of the GEMV kernels at
// its start.
constexpr size_t kConvOffset = 64 * 1024;

std::atomic<int> g_tune_bt{0};        // 0 = automatic
std::atomic<int> g_tune_min_rows{5};  // smallest M sent to the tensor-core GEMM (4 rows and fewer: GEMV kernels)
std::atomic<int> g_tune_par{2};        // dequant warp groups working on alternate k steps
std::atomic<int> g_tune_spin{0};       // single-thread waits spin on test_wait
std::atomic<int> g_tune_tma_store{1};  // 16-bit outputs through TMA stores
std::atomic<int> g_tune_split{1};      // split the tiles of a partial last round into k halves
std::atomic<int> g_tune_pair{0};       // 256-token tiles on CTA pairs (tcgen05 cta_group::2)

struct GPlan {
  bool ok = false;
  int bt = 128;
  bool convert = false;
  bool bf16_op = false;
  int ld_act = 0;
  size_t conv_bytes = 0;
};

int pick_bt(int M, int N, int sms) {
  const int tune = g_tune_bt.load();
  if (tune == 128 || tune == 192 || tune == 256) return tune;
  // Each activation tile is re-read from L2 for every 128 weight columns, so
  // the widest token tile moves the fewest bytes per MMA; a narrower one only
  // pays off when it needs fewer rounds of tiles over the SMs.
  const int n_tiles = (N + kWCols - 1) / kWCols;
  auto rounds = [&](int bt) { return (n_tiles * ((M + bt - 1) / bt) + sms - 1) / sms; };
  if (M > 192 && rounds(256) <= rounds(192)) return 256;
  if (M > 128 && rounds(192) <= rounds(128)) return 192;
  return M > 128 ? 256 : 128;
}

// Split of the last round: when the tiles leave a last round that fills at
// most half of the SMs, each of its tiles becomes two k halves on two SMs
// (fp32 partial sums in the scratch, after a ticket prefix), which halves the
// round's length for a few hundred KB of L2 traffic per tile.  Short k
// ranges gain too little to pay for that.
struct SplitPlan {
  int whole = 0, rem = 0;   // whole tiles, split tiles
  size_t part_off = 0;      // partial sums' offset in the scratch
  size_t bytes = 0;         // scratch the split needs (conversion included)
};
SplitPlan split_plan(const GPlan& pl, int M, int N, int K, int bt, int sms) {
  SplitPlan sp;
  const int tiles = ((N + kWCols - 1) / kWCols) * ((M + bt - 1) / bt);
  const int ksteps = (K + kKStep - 1) / kKStep;
  sp.whole = tiles;
  sp.bytes = pl.conv_bytes;
  if (!g_tune_split.load() || ksteps < 16 || sms <= 0) return sp;
  const int r = tiles % sms;
  if (r == 0 || 2 * r > sms || r > 1024) return sp;
  sp.whole = tiles - r;
  sp.rem = r;
  sp.part_off = pl.convert ? pl.conv_bytes : kConvOffset;
  sp.bytes = sp.part_off + (size_t)r * 2 * bt * kWCols * 4;
  return sp;
}

// CTA pairs: each MMA covers 256 weight columns, so every CTA stages half as
// many activation bytes per FLOP and holds more pipeline stages; used when the
// 256 x 256 tiles give every pair of SMs at least one.
bool use_pair(int M, int N, int bt, int sms) {
  const int mode = g_tune_pair.load();  // 0 never, 1 when the tiles fill the pairs, 2 whenever bt is 256
  if (mode == 0 || bt != 256) return false;
  const int tiles = ((N + 2 * kWCols - 1) / (2 * kWCols)) * ((M + bt - 1) / bt);
  return mode == 2 || tiles >= sms / 2;
}

GPlan make_plan(const SgMatMulParams* p, int wkind) {
  GPlan pl;
  if (p->M < std::max(2, g_tune_min_rows.load()) || p->K <= 0 || p->N <= 0) return pl;
  if (p->N % 16 != 0 || !sg::aligned16(p->B)) return pl;
  const int a_dt = p->a_dtype == SG_DT_DEFAULT ? (wkind == kW4Grouped ? SG_DT_I8 : SG_DT_F16) : p->a_dtype;
  if (wkind == kW4Grouped) {
    const int gs = p->group_size > 0 ? p->group_size : 128;
    if (!(gs == 16 || gs == 32 || gs % kKStep == 0)) return pl;
    if (!sg::aligned16(p->scales_B) || (p->zeros_B && !sg::aligned16(p->zeros_B))) return pl;
    pl.bf16_op = false;
  } else {
    if (a_dt == SG_DT_I8) return pl;  // exact int32 path stays on the GEMV kernels
    pl.bf16_op = (a_dt == SG_DT_BF16);
  }
  const int lda = p->lda > 0 ? p->lda : p->K;
  const bool direct = ((a_dt == SG_DT_F16 && !pl.bf16_op) || (a_dt == SG_DT_BF16 && pl.bf16_op)) &&
                      (lda % 8 == 0) && sg::aligned16(p->A);
  pl.convert = !direct;
  pl.ld_act = direct ? lda : (int)sg::align_up((size_t)p->K, 8);
  pl.conv_bytes = pl.convert ? kConvOffset + sg::align_up((size_t)p->M * pl.ld_act * 2, 256) : 0;
  pl.ok = true;
  return pl;
}

// grid: CTAs for a.units work units on `sms` SMs; a pair kernel launches
// clusters of two, as many as can be resident at once.
template <int BT, int WK, bool BF16_OP, bool HAS_Z, int PAR, bool PAIR>
SgStatus launch(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tz,
                const CUtensorMap& tc, const GArgs& a, int sms, cudaStream_t cs) {
  using C_ = Cfg<BT, WK, PAIR>;
  auto kfn = gemm_tc_kernel<BT, WK, BF16_OP, HAS_Z, PAR, PAIR>;
  static std::atomic<uint64_t> attr_set{0};  // bit per device ordinal
  static std::atomic<int> max_pairs[64];      // resident clusters of two, per device (0 = not known yet)
  int dev = 0;
  SgStatus dst = sg::current_device(&dev);
  if (dst != SG_OK) return dst;
  const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
  if (!(attr_set.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::kSmem);
    if (e != cudaSuccess) {
      cudaGetLastError();
      sg::set_error("gemm_tc_kernel: cannot reserve %d bytes of shared memory: %s", C_::kSmem,
                    cudaGetErrorString(e));
      return SG_ERR_RUNTIME;
    }
    attr_set.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(threads_of(PAR));
  cfg.dynamicSmemBytes = C_::kSmem;
  cfg.stream = cs;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int grid = std::min(a.units, sms);
  if (PAIR) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    const int slot = dev < 64 ? dev : 63;
    int pairs = max_pairs[slot].load();
    if (pairs <= 0) {
      cfg.gridDim = dim3(2 * std::max(1, sms / 2));
      cudaError_t e = cudaOccupancyMaxActiveClusters(&pairs, kfn, &cfg);
      if (e != cudaSuccess || pairs <= 0) {
        cudaGetLastError();
        sg::set_error("gemm_tc_kernel: no resident CTA pair (%s)", cudaGetErrorString(e));
        return SG_ERR_RUNTIME;
      }
      max_pairs[slot].store(pairs);
    }
    grid = 2 * std::min(a.units, pairs);
  }
  cfg.gridDim = dim3(grid);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, ta, tw, ts, tz, tc, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    sg::set_error("gemm_tc_kernel launch failed: %s", cudaGetErrorString(e));
    return SG_ERR_RUNTIME;
  }
  return SG_OK;
}

template <int WK, bool BF16_OP, bool HAS_Z, int PAR>
SgStatus launch_bt(int bt, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& ts,
                   const CUtensorMap& tz, const CUtensorMap& tc, const GArgs& a, int sms, cudaStream_t cs) {
  switch (bt) {
    case 256: return launch<256, WK, BF16_OP, HAS_Z, PAR, false>(ta, tw, ts, tz, tc, a, sms, cs);
    case 192: return launch<192, WK, BF16_OP, HAS_Z, PAR, false>(ta, tw, ts, tz, tc, a, sms, cs);
    default: return launch<128, WK, BF16_OP, HAS_Z, PAR, false>(ta, tw, ts, tz, tc, a, sms, cs);
  }
}

// pair: 256-token tiles shared by two CTAs (always two dequant groups).
template <int WK, bool BF16_OP, bool HAS_Z>
SgStatus launch_par(bool pair, int par, int bt, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& ts,
                    const CUtensorMap& tz, const CUtensorMap& tc, const GArgs& a, int sms, cudaStream_t cs) {
  if (pair) return launch<256, WK, BF16_OP, HAS_Z, 2, true>(ta, tw, ts, tz, tc, a, sms, cs);
  if (par == 1) return launch_bt<WK, BF16_OP, HAS_Z, 1>(bt, ta, tw, ts, tz, tc, a, sms, cs);
  return launch_bt<WK, BF16_OP, HAS_Z, 2>(bt, ta, tw, ts, tz, tc, a, sms, cs);
}

}  // namespace

namespace sg {

// Scratch bytes the tensor-core GEMM needs for this problem (0 when it takes
// the activations as they are); *ok = false when the problem goes elsewhere.
size_t gemm_tc_scratch_bytes(const SgMatMulParams* p, bool int8_weights, bool* ok, bool minimal) {
  const GPlan pl = make_plan(p, int8_weights ? kW8Channel : kW4Grouped);
  *ok = pl.ok;
  if (!pl.ok) return 0;
  if (minimal) return pl.conv_bytes;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return pl.conv_bytes;
  }
  const int sms = sm_count(dev);
  const int bt = pick_bt(p->M, p->N, sms);
  if (use_pair(p->M, p->N, bt, sms)) return pl.conv_bytes;
  return split_plan(pl, p->M, p->N, p->K, bt, sms).bytes;
}

// Runs the tensor-core GEMM when the problem qualifies (*handled = true).
SgStatus gemm_tc_run(const SgMatMulParams* p, bool int8_weights, cudaStream_t cs, int sms, void* ws,
                     size_t ws_bytes, int* err_word, bool* handled) {
  *handled = false;
  const int wk = int8_weights ? kW8Channel : kW4Grouped;
  const GPlan pl = make_plan(p, wk);
  if (!pl.ok) return SG_OK;
  if (pl.convert) {
    SG_CHECK_ARG(ws != nullptr && ws_bytes >= pl.conv_bytes && aligned16(ws),
                 "tensor-core GEMM: activation scratch too small (%zu < %zu bytes)", ws_bytes, pl.conv_bytes);
  }
  const int a_dt = p->a_dtype == SG_DT_DEFAULT ? (wk == kW4Grouped ? SG_DT_I8 : SG_DT_F16) : p->a_dtype;
  const int lda = p->lda > 0 ? p->lda : p->K;
  const void* act = p->A;
  void* const ws_base = ws;
  if (pl.convert) {
    ws = static_cast<unsigned char*>(ws) + kConvOffset;
    const int chunks = pl.ld_act / 8;
    const dim3 grid((chunks + 127) / 128, std::min(p->M, 65535));
    if (pl.bf16_op)
      act_convert_kernel<true><<<grid, 128, 0, cs>>>(p->A, a_dt, lda, p->M, p->K, pl.ld_act, ws);
    else
      act_convert_kernel<false><<<grid, 128, 0, cs>>>(p->A, a_dt, lda, p->M, p->K, pl.ld_act, ws);
    SgStatus st = check_launch("act_convert_kernel");
    if (st != SG_OK) return st;
    act = ws;
  }
  const int bt = pick_bt(p->M, p->N, sms);
  const bool pair = use_pair(p->M, p->N, bt, sms);
  const int gs = p->group_size > 0 ? p->group_size : 128;
  const int G = (p->K + gs - 1) / gs;

  CUtensorMap ta, tw, ts, tz;
  SgStatus st;
  {
    const uint64_t dims[2] = {(uint64_t)p->K, (uint64_t)p->M};
    const uint64_t str[1] = {(uint64_t)pl.ld_act * 2};
    const uint32_t box[2] = {(uint32_t)kKStep, (uint32_t)(pair ? bt / 2 : bt)};
    st = make_tensor_map(&ta, pl.bf16_op ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                         const_cast<void*>(act), dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SG_OK) return st;
  }
  if (wk == kW4Grouped) {
    const uint64_t dims[2] = {(uint64_t)p->N, (uint64_t)((p->K + 1) / 2)};
    const uint64_t str[1] = {(uint64_t)p->N};
    const uint32_t box[2] = {(uint32_t)kWCols, (uint32_t)(kKStep / 2)};
    st = make_tensor_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(p->B), dims, str, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != SG_OK) return st;
    const uint32_t srows = gs >= kKStep ? 1 : kKStep / gs;
    const uint64_t sdims[2] = {(uint64_t)p->N, (uint64_t)G};
    const uint64_t sstr[1] = {(uint64_t)p->N * 2};
    const uint32_t sbox[2] = {(uint32_t)kWCols, srows};
    st = make_tensor_map(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(p->scales_B), sdims, sstr, sbox,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != SG_OK) return st;
    if (p->zeros_B) {
      const uint64_t zstr[1] = {(uint64_t)p->N};
      st = make_tensor_map(&tz, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(p->zeros_B), sdims, zstr, sbox,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
      if (st != SG_OK) return st;
    } else {
      tz = ts;
    }
  } else {
    const uint64_t dims[2] = {(uint64_t)p->N, (uint64_t)p->K};
    const uint64_t str[1] = {(uint64_t)p->N};
    const uint32_t box[2] = {(uint32_t)kWCols, (uint32_t)kKStep};
    st = make_tensor_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(p->B), dims, str, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != SG_OK) return st;
    ts = tw;
    tz = tw;
  }

  GArgs a{};
  a.C = p->C;
  a.bias = wk == kW4Grouped ? static_cast<const __half*>(p->bias) : nullptr;
  a.scales = wk == kW8Channel ? static_cast<const float*>(p->scales_B) : nullptr;
  a.scale_A = p->scale_A;
  a.apply_scale_A = (wk == kW4Grouped && a_dt == SG_DT_I8) ? 1 : 0;
  a.c_dt = p->c_dtype == SG_DT_DEFAULT ? (wk == kW4Grouped ? SG_DT_F16 : SG_DT_F32) : p->c_dtype;
  a.ldc = p->ldc > 0 ? p->ldc : p->N;
  a.M = p->M;
  a.N = p->N;
  a.K = p->K;
  a.gs = gs;
  a.ksteps = (p->K + kKStep - 1) / kKStep;
  a.n_tiles = pair ? (p->N + 2 * kWCols - 1) / (2 * kWCols) : (p->N + kWCols - 1) / kWCols;
  a.m_tiles = (p->M + bt - 1) / bt;
  a.err = err_word;
  a.spin = g_tune_spin.load() ? 1 : 0;
  // 16-bit C with 16-byte aligned rows: TMA stores from a shared-memory staging tile.
  CUtensorMap tc = ta;
  a.tma_store = 0;
  if ((a.c_dt == SG_DT_F16 || a.c_dt == SG_DT_BF16) && aligned16(p->C) && ((size_t)a.ldc * 2) % 16 == 0 &&
      g_tune_tma_store.load()) {
    const uint64_t dims[2] = {(uint64_t)p->N, (uint64_t)p->M};
    const uint64_t str[1] = {(uint64_t)a.ldc * 2};
    const uint32_t box[2] = {(uint32_t)kWCols, (uint32_t)kOutChunk};
    st = make_tensor_map(&tc, a.c_dt == SG_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, p->C, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != SG_OK) return st;
    a.tma_store = 1;
  }
  const int tiles = a.n_tiles * a.m_tiles;
  // Split of the last round, when the scratch has room for it.  Every CTA then
  // gets at most one split unit, as its last one (the kernel relies on that).
  const SplitPlan sp = pair ? SplitPlan{} : split_plan(pl, p->M, p->N, p->K, bt, sms);
  a.whole = tiles;
  a.units = tiles;
  if (sp.rem > 0 && ws_base != nullptr && ws_bytes >= sp.bytes && aligned16(ws_base)) {
    a.whole = sp.whole;
    a.units = sp.whole + 2 * sp.rem;
    a.tickets = static_cast<unsigned*>(ws_base);
    a.partials = reinterpret_cast<float*>(static_cast<unsigned char*>(ws_base) + sp.part_off);
  }
  *handled = true;
  const int par = g_tune_par.load() == 1 ? 1 : 2;
  if (wk == kW4Grouped) {
    if (p->zeros_B) return launch_par<kW4Grouped, false, true>(pair, par, bt, ta, tw, ts, tz, tc, a, sms, cs);
    return launch_par<kW4Grouped, false, false>(pair, par, bt, ta, tw, ts, tz, tc, a, sms, cs);
  }
  if (pl.bf16_op) return launch_par<kW8Channel, true, false>(pair, par, bt, ta, tw, ts, tz, tc, a, sms, cs);
  return launch_par<kW8Channel, false, false>(pair, par, bt, ta, tw, ts, tz, tc, a, sms, cs);
}

bool gemm_tc_tuning(std::string_view key, int value) {
  if (key == "gemm_tc.bt") {
    g_tune_bt.store(value);
    return true;
  }
  if (key == "gemm_tc.tma_store") {
    g_tune_tma_store.store(value);
    return true;
  }
  if (key == "gemm_tc.spin") {
    g_tune_spin.store(value);
    return true;
  }
  if (key == "gemm_tc.par") {
    g_tune_par.store(value);
    return true;
  }
  if (key == "gemm_tc.pair") {
    g_tune_pair.store(value);
    return true;
  }
  if (key == "gemm_tc.split") {
    g_tune_split.store(value);
    return true;
  }
  if (key == "gemm_tc.min_rows") {
    g_tune_min_rows.store(value);
    return true;
  }
  return false;
}

}  // namespace sg
