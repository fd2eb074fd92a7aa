// Flash attention on the 5th-generation tensor cores for fp16 / bf16 I/O and
// head_dim 64 or 128: the batched, GQA, causal driver of
// flash_attention_fp16 (compiler/kernels/cpu/flash_attention.h:95-144) with
// the per-query online softmax of flash_attn_head (flash_attention.h:49-90).
//
// One CTA per (128-query tile, head, batch).  Per 128-key tile j:
//   S_j = Q K_j^T        tcgen05.mma, A = Q and B = K_j from shared memory
//                        (TMA, 128-byte swizzle, K-major), D = S_j in TMEM
//   softmax              one thread per query row (TMEM lane): its whole score
//                        row is in its registers after tcgen05.ld, so the row
//                        max and sum need no shuffles; P_j is written back
//                        into the first half of S_j's TMEM columns (16-bit)
//   O += P_j V_j         tcgen05.mma with A = P_j from TMEM and B = V_j from
//                        shared memory read MN-major (V rows are keys)
// The running max moves (and O is rescaled) only when a row's max grows by
// more than 2^8 in exp2 units; otherwise P is taken against the old max, at
// most 2^8, which the 16-bit P and fp32 sums hold exactly enough.  The final
// O / l is invariant to the reference point of the max; l sums the fp32
// weights whose 16-bit roundings PV multiplies (within 2^-12 of each other).
//
// Warps: 0..3 softmax + epilogue (TMEM lane quarter = warp), 4: K loader,
// 5: V loader, 6: MMA issuer.  K and V tiles have separate two-stage rings:
// a K tile is free as soon as its QK^T finished, a V tile after its PV.
// TMEM: S/P buffers at columns 0 and 128, O at 256 .. 256 + D.
// All waits are bounded (2 s) and report through the device error word.
#include <algorithm>
#include <atomic>
#include <string_view>
#include <type_traits>

#include "sm100.cuh"

namespace {

using namespace sgd;

constexpr int kQT = 128;  // query rows per CTA = TMEM lanes
constexpr int kKT = 128;  // keys per tile
constexpr int kWarpK = 4, kWarpV = 5, kWarpMma = 6;
constexpr int kThreads = 7 * 32;
constexpr int kTmemCols = 512;
constexpr int kStages = 2;
constexpr int kOCol = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct ACfg {
  static constexpr int kBoxes = D / 64;          // 64-element (128-byte) column blocks per tile
  static constexpr int kBox = 128 * 128;         // one [128 rows x 128 B] block
  static constexpr int kTile = kBoxes * kBox;    // one [128 x D] 16-bit tile
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kTile;
  static constexpr int kVOff = kKOff + kStages * kTile;
  static constexpr int kBarOff = kVOff + kStages * kTile;
  static constexpr int kBars = 1 + 6 * kStages + 2;
  // At least 120 KB so that one CTA holds an SM (and its 512 TMEM columns).
  static constexpr int kSmem0 = kBarOff + kBars * 8 + 16 + 1024;
  static constexpr int kSmem = kSmem0 < 120 * 1024 ? 120 * 1024 : kSmem0;
};

struct TArgs {
  void* O;
  int B, H, G, Sq, Skv;
  float scale_log2;  // softmax scale * log2(e)
  int causal, q_pos0;
  int n_qt;
  int* err;
  // paged KV cache: the K (and, unless copied flat, V) maps are [page][kv head]
  // [16 rows][D] and key j of sequence b lives in page pt[b * pt_bs + (j / 16) * pt_ps]
  const int32_t* pt;
  int64_t pt_bs, pt_ps;
  int npages;
  int paged_k, paged_v;
  // fp32 I/O: Q / K / V were copied to fp16 scaled by powers of two; dscale[0]
  // undoes the Q and K scales on the scores, dscale[1] the V scale on O, which
  // is written as fp32
  int o_f32;
  const float* dscale;
};
constexpr int kPageRows = 16;                // keys per page
constexpr int kPagesPerTile = kKT / kPageRows;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void warp_wait_all(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
  if (!mbar_wait(bar, parity, err)) *abort_flag = 1;
  __syncwarp();
}

// BF16: Q / K / O are bf16 (else fp16).  P and V are always fp16: bf16 inputs
// have their V copied to fp16 first (exact within fp16's range), so that P
// keeps 11 significant bits instead of 8.
template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, TArgs a) {
  using C_ = ACfg<D>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = sgd::align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C_::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + kStages;
  uint64_t* v_full = k_empty + kStages;
  uint64_t* v_empty = v_full + kStages;
  uint64_t* s_full = v_empty + kStages;
  uint64_t* p_full = s_full + kStages;
  uint64_t* o_ready = p_full + kStages;
  uint64_t* done = o_ready + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work item: the heaviest query tiles (most keys under a causal mask) launch first.
  const int hb_count = a.H * a.B;
  const int qt = a.n_qt - 1 - (int)(blockIdx.x / hb_count);
  const int hb = (int)(blockIdx.x % hb_count);
  const int h = hb % a.H, b = hb / a.H;
  const int hkv = h / a.G;
  const int q0 = qt * kQT;
  const int q_last = min(q0 + kQT, a.Sq) - 1;
  const int kv_tiles_all = (a.Skv + kKT - 1) / kKT;
  const int n_kv = a.causal ? min(kv_tiles_all, (a.q_pos0 + q_last) / kKT + 1) : kv_tiles_all;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 4);
    }
    mbar_init(o_ready, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(tslot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kWarpK && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
  }
  if (warp == kWarpV && lane == 0) tma_prefetch_desc(&tmV);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();

  if (warp == kWarpK || warp == kWarpV) {
    // ------------------------------------------------------------ loaders
    // lane 0 issues the copies; with a paged cache lanes 0..7 first look up the
    // tile's eight page ids, one tile ahead of its copies
    const bool is_k = warp == kWarpK;
    const CUtensorMap* map = is_k ? &tmK : &tmV;
    uint64_t* fullb = is_k ? k_full : v_full;
    uint64_t* emptyb = is_k ? k_empty : v_empty;
    unsigned char* base = smem + (is_k ? C_::kKOff : C_::kVOff);
    const bool paged = is_k ? a.paged_k : a.paged_v;
    // physical page of logical page kPagesPerTile * j + lane (page 0, whose rows the
    // mask hides, past the keys; a bad id reads page 0 and is reported)
    auto page_of = [&](int j) -> int {
      const int lp = j * kPagesPerTile + lane;
      int pg = 0;
      if (lane < kPagesPerTile && j < n_kv && lp * kPageRows < a.Skv) {
        pg = __ldg(a.pt + (int64_t)b * a.pt_bs + (int64_t)lp * a.pt_ps);
        if ((unsigned)pg >= (unsigned)a.npages) {
          atomicOr(a.err, 4);
          pg = 0;
        }
      }
      return pg;
    };
    if (is_k && lane == 0) {
      mbar_arrive_expect_tx(q_full, C_::kTile);
      for (int bx = 0; bx < C_::kBoxes; ++bx)
        tma_load_3d(smem + C_::kQOff + bx * C_::kBox, &tmQ, bx * 64, q0, hb, q_full);
    }
    uint32_t issued[kStages] = {0, 0};
    int pg_next = paged ? page_of(0) : 0;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j % kStages;
      const uint32_t use = j / kStages;
      const int pg_cur = pg_next;
      if (paged) pg_next = page_of(j + 1);  // in flight while this tile waits for its stage
      int ok = 1;
      if (lane == 0) ok = (!*abort_flag && mbar_wait(&emptyb[st], (use & 1) ^ 1, a.err)) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      if (paged) {
        int pages[kPagesPerTile];
#pragma unroll
        for (int i = 0; i < kPagesPerTile; ++i) pages[i] = __shfl_sync(0xffffffffu, pg_cur, i);
        if (lane == 0) {
          mbar_arrive_expect_tx(&fullb[st], C_::kTile);
          // a 16-row box lands 2 KB into the 128-row block: the 128-byte swizzle
          // pattern (1 KB period) is that of the whole tile
#pragma unroll
          for (int i = 0; i < kPagesPerTile; ++i)
            for (int bx = 0; bx < C_::kBoxes; ++bx)
              tma_load_4d(base + st * C_::kTile + bx * C_::kBox + i * kPageRows * 128, map, bx * 64, 0, hkv,
                          pages[i], &fullb[st]);
        }
      } else if (lane == 0) {
        mbar_arrive_expect_tx(&fullb[st], C_::kTile);
        for (int bx = 0; bx < C_::kBoxes; ++bx)
          tma_load_4d(base + st * C_::kTile + bx * C_::kBox, map, bx * 64, j * kKT, hkv, b, &fullb[st]);
      }
      issued[st] = use + 1;
    }
    if (lane == 0) {
      for (int st = 0; st < kStages; ++st)
        if (issued[st]) mbar_wait(&fullb[st], (issued[st] - 1) & 1, a.err);
      if (is_k) mbar_wait(q_full, 0, a.err);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = umma_idesc_f16(kQT, kKT, BF16 ? 1 : 0, 0, 0);
      const uint32_t idesc_pv = umma_idesc_f16(kQT, D, 0, 0, 1);  // fp16 P x fp16 V, B (= V) MN-major
      bool ok = mbar_wait(q_full, 0, a.err);
      auto issue_qk = [&](int t) -> bool {
        const int st = t % kStages;
        if (*abort_flag || !mbar_wait(&k_full[st], (t / kStages) & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t d = tbase + (t % 2) * kKT;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int bx = kk / 4, off = (kk % 4) * 32;
          const uint64_t ad = umma_smem_desc(smem_u32(smem + C_::kQOff + bx * C_::kBox + off), 16, 1024, kSwizzle128B);
          const uint64_t bd =
              umma_smem_desc(smem_u32(smem + C_::kKOff + st * C_::kTile + bx * C_::kBox + off), 16, 1024, kSwizzle128B);
          umma_f16_ss(d, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&k_empty[st]);
        umma_commit(&s_full[t % 2]);
        return true;
      };
      if (ok) ok = issue_qk(0);
      if (ok && n_kv > 1) ok = issue_qk(1);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % kStages;
        if (*abort_flag || !mbar_wait(&p_full[j % 2], (j / 2) & 1, a.err) ||
            !mbar_wait(&v_full[st], (j / kStages) & 1, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ap = tbase + (j % 2) * kKT;  // P_j: 128 keys as 64 columns of 16-bit pairs
#pragma unroll
        for (int kk = 0; kk < kKT / 16; ++kk) {
          // 16 keys = two 8-row groups of V: the start moves by 2 x 1024 bytes; LBO steps over
          // 64-column blocks of V (the second TMA box), SBO over 8-row groups.
          const uint64_t bd = umma_smem_desc(smem_u32(smem + C_::kVOff + st * C_::kTile + kk * 2048), C_::kBox, 1024,
                                             kSwizzle128B);
          umma_f16_ts(tbase + kOCol, ap + kk * 8, bd, idesc_pv, (j | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&v_empty[st]);
        umma_commit(o_ready);
        if (j + 2 < n_kv) ok = issue_qk(j + 2);
      }
      if (!ok) *abort_flag = 1;
      umma_commit(done);
      mbar_wait(done, 0, a.err);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const float scale_log2 = a.dscale ? a.scale_log2 * a.dscale[0] : a.scale_log2;
    const int r = warp * 32 + lane;  // query row in the tile = TMEM lane
    const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
    const int q = q0 + r;
    const int q_pos = a.q_pos0 + q;  // keys 0 .. q_pos are visible under the causal mask
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      __syncwarp();
      if (*abort_flag) {
        ok = false;
        break;
      }
      warp_wait_all(&s_full[j % 2], (j / 2) & 1, a.err, abort_flag);
      tc_fence_after();
      const uint32_t scol = tbase + lane_addr + (j % 2) * kKT;
      uint32_t sr[kKT];
#pragma unroll
      for (int c = 0; c < kKT / 32; ++c)
        tmem_ld_32x32b_x32(scol + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_ld_wait();
      const int key0 = j * kKT;
      const int lim = min(a.causal ? q_pos : 0x7fffffff, a.Skv - 1) - key0;  // keys key0 + i, i <= lim
      // Only tiles that reach past some row's last visible key need the mask.
      if (__any_sync(0xffffffffu, lim < kKT - 1)) {
#pragma unroll
        for (int i = 0; i < kKT; ++i)
          if (i > lim) sr[i] = __float_as_uint(-INFINITY);
      }
      // Row max on the raw scores (the scale is positive, so it commutes with max).
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kKT; i += 2) mx = fmax3(mx, __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
      mx *= scale_log2;
      float alpha = 1.f;
      const bool rescale = mx > m + kRescaleThreshold;
      if (rescale) {
        alpha = ex2(m - mx);  // 0 on the first tile (m = -inf)
        m = mx;
        l *= alpha;
      }
      // packed fp32x2 arithmetic for the scale-and-shift and the sum (the softmax is
      // issue-bound); l sums the fp32 weights as two interleaved partial sums (their
      // fp16 roundings, which PV multiplies, differ from them by 2^-12 at most)
      const float2 sl2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(-m, -m), one2 = make_float2(1.f, 1.f);
      float2 sum2v = make_float2(0.f, 0.f);
      uint32_t pk[kKT / 2];
#pragma unroll
      for (int i = 0; i < kKT / 2; ++i) {
        const float2 x = ffma2(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sl2, nm2);
        const float2 p = make_float2(ex2(x.x), ex2(x.y));
        pk[i] = pack2<false>(p.x, p.y);
        sum2v = ffma2(p, one2, sum2v);
      }
      l += sum2v.x + sum2v.y;
      tmem_st_32x32b_x16(scol, *reinterpret_cast<uint32_t(*)[16]>(&pk[0]));
      tmem_st_32x32b_x16(scol + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk[16]));
      tmem_st_32x32b_x16(scol + 32, *reinterpret_cast<uint32_t(*)[16]>(&pk[32]));
      tmem_st_32x32b_x16(scol + 48, *reinterpret_cast<uint32_t(*)[16]>(&pk[48]));
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        // O rows of this warp scale by alpha (1 for rows whose max did not move) once
        // PV_{j-1} has landed; PV_j waits for p_full below.
        warp_wait_all(o_ready, (j - 1) & 1, a.err, abort_flag);
        tc_fence_after();
#pragma unroll 1
        for (int dc = 0; dc < D / 32; ++dc) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tbase + lane_addr + kOCol + dc * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32x32b_x16(tbase + lane_addr + kOCol + dc * 32, *reinterpret_cast<uint32_t(*)[16]>(&o[0]));
          tmem_st_32x32b_x16(tbase + lane_addr + kOCol + dc * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&o[16]));
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j % 2]);
    }
    if (ok && n_kv > 0) {
      warp_wait_all(o_ready, (n_kv - 1) & 1, a.err, abort_flag);
      tc_fence_after();
      const float inv_l = 1.f / l;
      typedef typename std::conditional<BF16, __nv_bfloat16, __half>::type T;
      T* orow = static_cast<T*>(a.O) + ((size_t)hb * a.Sq + q) * D;
      float* orow32 = static_cast<float*>(a.O) + ((size_t)hb * a.Sq + q) * D;
      const float omul = a.dscale ? inv_l * a.dscale[1] : inv_l;
#pragma unroll 1
      for (int dc = 0; dc < D / 32; ++dc) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tbase + lane_addr + kOCol + dc * 32, o);
        tmem_ld_wait();
        if (a.o_f32) {  // (l sums the fp16 weights: the normalisation is that of the 16-bit path)
          if (q < a.Sq) {
            float4* dst = reinterpret_cast<float4*>(orow32 + dc * 32);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(__uint_as_float(o[4 * v]) * omul, __uint_as_float(o[4 * v + 1]) * omul,
                                   __uint_as_float(o[4 * v + 2]) * omul, __uint_as_float(o[4 * v + 3]) * omul);
          }
          continue;
        }
        uint32_t pkd[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pkd[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
        if (q < a.Sq) {
          uint4* dst = reinterpret_cast<uint4*>(orow + dc * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pkd[4 * v], pkd[4 * v + 1], pkd[4 * v + 2], pkd[4 * v + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Two query tiles per CTA (attn_tc2_kernel): tiles A (queries q0 ..) and B
// (q0 + 128 ..) of one head share the K and V tiles; 8 softmax warps (4 per
// tile, two per scheduler) and one MMA issuer that interleaves the tiles,
//   QK_A(0) QK_B(0) | PV_A(j) QK_A(j+1) | PV_B(j) QK_B(j+1) | ...
// so that while one tile's softmax runs, the tensor pipe works on the other
// tile's products.  Each tile has one S/P buffer in TMEM (QK_t(j+1) is issued
// after PV_t(j), and the tensor pipe runs them in order) and its own O:
// tile t at TMEM columns 256 t (S/P) and 256 t + 128 (O).  The arithmetic per
// row is the single-tile kernel's (same softmax, masks, rescaling rule and
// rounding), so both kernels give the same bits.
constexpr int kWarpK2 = 8, kWarpV2 = 9, kWarpMma2 = 10;
constexpr int kThreads2 = 11 * 32;

template <int D>
struct ACfg2 {
  static constexpr int kBoxes = D / 64;
  static constexpr int kBox = 128 * 128;
  static constexpr int kTile = kBoxes * kBox;
  static constexpr int kQOff = 0;  // Q tiles A and B
  static constexpr int kKOff = 2 * kTile;
  static constexpr int kVOff = kKOff + kStages * kTile;
  static constexpr int kBarOff = kVOff + kStages * kTile;
  static constexpr int kBars = 1 + 4 * kStages + 2 + 2 + 2 + 1;
  static constexpr int kSmem0 = kBarOff + kBars * 8 + 16 + 1024;
  static constexpr int kSmem = kSmem0 < 120 * 1024 ? 120 * 1024 : kSmem0;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads2, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, TArgs a) {
  using C_ = ACfg2<D>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = sgd::align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C_::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + kStages;
  uint64_t* v_full = k_empty + kStages;
  uint64_t* v_empty = v_full + kStages;
  uint64_t* s_full = v_empty + kStages;  // [tile]
  uint64_t* p_full = s_full + 2;         // [tile]
  uint64_t* o_ready = p_full + 2;        // [tile]
  uint64_t* done = o_ready + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work item: the heaviest pairs of query tiles (most keys under a causal mask) first.
  const int hb_count = a.H * a.B;
  const int n_pairs = (a.n_qt + 1) / 2;
  const int pr = n_pairs - 1 - (int)(blockIdx.x / hb_count);
  const int hb = (int)(blockIdx.x % hb_count);
  const int h = hb % a.H, b = hb / a.H;
  const int hkv = h / a.G;
  const int q0 = pr * 2 * kQT;
  const int kv_tiles_all = (a.Skv + kKT - 1) / kKT;
  int n_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qa = q0 + t * kQT;
    const int q_last = min(qa + kQT, a.Sq) - 1;
    n_t[t] = qa >= a.Sq ? 0 : (a.causal ? min(kv_tiles_all, (a.q_pos0 + q_last) / kKT + 1) : kv_tiles_all);
  }
  const int n_kv = max(n_t[0], n_t[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_ready[t], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMma2) {
    tmem_alloc(tslot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kWarpK2 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
  }
  if (warp == kWarpV2 && lane == 0) tma_prefetch_desc(&tmV);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();

  if (warp == kWarpK2 || warp == kWarpV2) {
    // ------------------------------------------------------------ loaders (as in attn_tc_kernel)
    const bool is_k = warp == kWarpK2;
    const CUtensorMap* map = is_k ? &tmK : &tmV;
    uint64_t* fullb = is_k ? k_full : v_full;
    uint64_t* emptyb = is_k ? k_empty : v_empty;
    unsigned char* base = smem + (is_k ? C_::kKOff : C_::kVOff);
    const bool paged = is_k ? a.paged_k : a.paged_v;
    auto page_of = [&](int j) -> int {
      const int lp = j * kPagesPerTile + lane;
      int pg = 0;
      if (lane < kPagesPerTile && j < n_kv && lp * kPageRows < a.Skv) {
        pg = __ldg(a.pt + (int64_t)b * a.pt_bs + (int64_t)lp * a.pt_ps);
        if ((unsigned)pg >= (unsigned)a.npages) {
          atomicOr(a.err, 4);
          pg = 0;
        }
      }
      return pg;
    };
    if (is_k && lane == 0) {
      const int nq = n_t[1] > 0 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, nq * C_::kTile);
      for (int t = 0; t < nq; ++t)
        for (int bx = 0; bx < C_::kBoxes; ++bx)
          tma_load_3d(smem + C_::kQOff + t * C_::kTile + bx * C_::kBox, &tmQ, bx * 64, q0 + t * kQT, hb, q_full);
    }
    uint32_t issued[kStages] = {0, 0};
    int pg_next = paged ? page_of(0) : 0;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j % kStages;
      const uint32_t use = j / kStages;
      const int pg_cur = pg_next;
      if (paged) pg_next = page_of(j + 1);
      int ok = 1;
      if (lane == 0) ok = (!*abort_flag && mbar_wait(&emptyb[st], (use & 1) ^ 1, a.err)) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      if (paged) {
        int pages[kPagesPerTile];
#pragma unroll
        for (int i = 0; i < kPagesPerTile; ++i) pages[i] = __shfl_sync(0xffffffffu, pg_cur, i);
        if (lane == 0) {
          mbar_arrive_expect_tx(&fullb[st], C_::kTile);
#pragma unroll
          for (int i = 0; i < kPagesPerTile; ++i)
            for (int bx = 0; bx < C_::kBoxes; ++bx)
              tma_load_4d(base + st * C_::kTile + bx * C_::kBox + i * kPageRows * 128, map, bx * 64, 0, hkv,
                          pages[i], &fullb[st]);
        }
      } else if (lane == 0) {
        mbar_arrive_expect_tx(&fullb[st], C_::kTile);
        for (int bx = 0; bx < C_::kBoxes; ++bx)
          tma_load_4d(base + st * C_::kTile + bx * C_::kBox, map, bx * 64, j * kKT, hkv, b, &fullb[st]);
      }
      issued[st] = use + 1;
    }
    if (lane == 0) {
      for (int st = 0; st < kStages; ++st)
        if (issued[st]) mbar_wait(&fullb[st], (issued[st] - 1) & 1, a.err);
      if (is_k) mbar_wait(q_full, 0, a.err);
    }
  } else if (warp == kWarpMma2) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = umma_idesc_f16(kQT, kKT, BF16 ? 1 : 0, 0, 0);
      const uint32_t idesc_pv = umma_idesc_f16(kQT, D, 0, 0, 1);
      bool ok = mbar_wait(q_full, 0, a.err);
      auto wait_k = [&](int j) -> bool {
        if (*abort_flag || !mbar_wait(&k_full[j % kStages], (j / kStages) & 1, a.err)) return false;
        tc_fence_after();
        return true;
      };
      auto qk = [&](int t, int j) {  // S_t = Q_t K_j^T
        const int st = j % kStages;
        const uint32_t d = tbase + 256 * t;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int bx = kk / 4, off = (kk % 4) * 32;
          const uint64_t ad = umma_smem_desc(smem_u32(smem + C_::kQOff + t * C_::kTile + bx * C_::kBox + off), 16,
                                             1024, kSwizzle128B);
          const uint64_t bd =
              umma_smem_desc(smem_u32(smem + C_::kKOff + st * C_::kTile + bx * C_::kBox + off), 16, 1024, kSwizzle128B);
          umma_f16_ss(d, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto pv = [&](int t, int j) {  // O_t += P_t V_j
        const int st = j % kStages;
        const uint32_t ap = tbase + 256 * t;
#pragma unroll
        for (int kk = 0; kk < kKT / 16; ++kk) {
          const uint64_t bd = umma_smem_desc(smem_u32(smem + C_::kVOff + st * C_::kTile + kk * 2048), C_::kBox, 1024,
                                             kSwizzle128B);
          umma_f16_ts(tbase + 256 * t + 128, ap + kk * 8, bd, idesc_pv, (j | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&o_ready[t]);
      };
      if (ok && n_kv > 0) {
        ok = wait_k(0);
        if (ok) {
          if (n_t[0] > 0) qk(0, 0);
          if (n_t[1] > 0) qk(1, 0);
          umma_commit(&k_empty[0]);
        }
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % kStages;
        bool v_waited = false, k_next = false;
        if (j < n_t[0]) {
          if (*abort_flag || !mbar_wait(&p_full[0], j & 1, a.err) ||
              !mbar_wait(&v_full[st], (j / kStages) & 1, a.err)) {
            ok = false;
            break;
          }
          v_waited = true;
          tc_fence_after();
          pv(0, j);
          if (j + 1 < n_t[0]) {
            if (!(ok = wait_k(j + 1))) break;
            k_next = true;
            qk(0, j + 1);
          }
        }
        if (j < n_t[1]) {
          if (*abort_flag || !mbar_wait(&p_full[1], j & 1, a.err) ||
              (!v_waited && !mbar_wait(&v_full[st], (j / kStages) & 1, a.err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          pv(1, j);
        }
        umma_commit(&v_empty[st]);  // V_j: both products issued
        if (j + 1 < n_t[1]) {
          if (!k_next && !(ok = wait_k(j + 1))) break;
          k_next = true;
          qk(1, j + 1);
        }
        if (k_next) umma_commit(&k_empty[(j + 1) % kStages]);  // K_{j+1}: every product issued
      }
      if (!ok) *abort_flag = 1;
      umma_commit(done);
      mbar_wait(done, 0, a.err);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue, tile warp / 4
    const int t = warp >> 2, quarter = warp & 3;
    const int nt = n_t[t];
    const float scale_log2 = a.dscale ? a.scale_log2 * a.dscale[0] : a.scale_log2;
    const int r = quarter * 32 + lane;  // query row in the tile = TMEM lane
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int q = q0 + t * kQT + r;
    const int q_pos = a.q_pos0 + q;
    const uint32_t scol = tbase + lane_addr + 256 * t;
    const uint32_t ocol = scol + 128;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      __syncwarp();
      if (*abort_flag) {
        ok = false;
        break;
      }
      warp_wait_all(&s_full[t], j & 1, a.err, abort_flag);
      tc_fence_after();
      uint32_t sr[kKT];
#pragma unroll
      for (int c = 0; c < kKT / 32; ++c)
        tmem_ld_32x32b_x32(scol + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_ld_wait();
      const int key0 = j * kKT;
      const int lim = min(a.causal ? q_pos : 0x7fffffff, a.Skv - 1) - key0;
      if (__any_sync(0xffffffffu, lim < kKT - 1)) {
#pragma unroll
        for (int i = 0; i < kKT; ++i)
          if (i > lim) sr[i] = __float_as_uint(-INFINITY);
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kKT; i += 2) mx = fmax3(mx, __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
      mx *= scale_log2;
      float alpha = 1.f;
      const bool rescale = mx > m + kRescaleThreshold;
      if (rescale) {
        alpha = ex2(m - mx);
        m = mx;
        l *= alpha;
      }
      // as in attn_tc_kernel: packed fp32x2 scale-and-shift and sum of the fp32 weights
      const float2 sl2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(-m, -m), one2 = make_float2(1.f, 1.f);
      float2 sum2v = make_float2(0.f, 0.f);
      uint32_t pk[kKT / 2];
#pragma unroll
      for (int i = 0; i < kKT / 2; ++i) {
        const float2 x = ffma2(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sl2, nm2);
        const float2 p = make_float2(ex2(x.x), ex2(x.y));
        pk[i] = pack2<false>(p.x, p.y);
        sum2v = ffma2(p, one2, sum2v);
      }
      l += sum2v.x + sum2v.y;
      tmem_st_32x32b_x16(scol, *reinterpret_cast<uint32_t(*)[16]>(&pk[0]));
      tmem_st_32x32b_x16(scol + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk[16]));
      tmem_st_32x32b_x16(scol + 32, *reinterpret_cast<uint32_t(*)[16]>(&pk[32]));
      tmem_st_32x32b_x16(scol + 48, *reinterpret_cast<uint32_t(*)[16]>(&pk[48]));
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        warp_wait_all(&o_ready[t], (j - 1) & 1, a.err, abort_flag);
        tc_fence_after();
#pragma unroll 1
        for (int dc = 0; dc < D / 32; ++dc) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(ocol + dc * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32x32b_x16(ocol + dc * 32, *reinterpret_cast<uint32_t(*)[16]>(&o[0]));
          tmem_st_32x32b_x16(ocol + dc * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&o[16]));
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (ok && nt > 0) {
      warp_wait_all(&o_ready[t], (nt - 1) & 1, a.err, abort_flag);
      tc_fence_after();
      const float inv_l = 1.f / l;
      typedef typename std::conditional<BF16, __nv_bfloat16, __half>::type T;
      T* orow = static_cast<T*>(a.O) + ((size_t)hb * a.Sq + q) * D;
      float* orow32 = static_cast<float*>(a.O) + ((size_t)hb * a.Sq + q) * D;
      const float omul = a.dscale ? inv_l * a.dscale[1] : inv_l;
#pragma unroll 1
      for (int dc = 0; dc < D / 32; ++dc) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(ocol + dc * 32, o);
        tmem_ld_wait();
        if (a.o_f32) {
          if (q < a.Sq) {
            float4* dst = reinterpret_cast<float4*>(orow32 + dc * 32);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(__uint_as_float(o[4 * v]) * omul, __uint_as_float(o[4 * v + 1]) * omul,
                                   __uint_as_float(o[4 * v + 2]) * omul, __uint_as_float(o[4 * v + 3]) * omul);
          }
          continue;
        }
        uint32_t pkd[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pkd[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
        if (q < a.Sq) {
          uint4* dst = reinterpret_cast<uint4*>(orow + dc * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pkd[4 * v], pkd[4 * v + 1], pkd[4 * v + 2], pkd[4 * v + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma2) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// V [B, Hkv, Skv, D] bf16 (strided) -> contiguous fp16, 8 values per thread.
// bf16 V -> contiguous fp16 [B][Hkv][Skv][D]; from a paged cache when pt != NULL
// (kv_bs is then the page stride).
__global__ void v_to_f16_kernel(const __nv_bfloat16* V, int64_t kv_bs, int64_t kv_hs, int Hkv, int Skv, int D,
                                int64_t total8, __half* out, const int32_t* pt, int64_t pt_bs, int64_t pt_ps,
                                int npages, int* err) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 8;
    const int d = (int)(e % D);
    const int64_t row = e / D;  // (b * Hkv + hk) * Skv + s
    const int s = (int)(row % Skv);
    const int64_t bh = row / Skv;
    const int hk = (int)(bh % Hkv), b = (int)(bh / Hkv);
    int64_t src;
    if (pt) {
      int pg = __ldg(pt + (int64_t)b * pt_bs + (int64_t)(s / kPageRows) * pt_ps);
      if ((unsigned)pg >= (unsigned)npages) {
        atomicOr(err, 4);
        pg = 0;
      }
      src = pg * kv_bs + ((int64_t)hk * kPageRows + s % kPageRows) * D + d;
    } else {
      src = b * kv_bs + hk * kv_hs + (int64_t)s * D + d;
    }
    const uint4 v = *reinterpret_cast<const uint4*>(V + src);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float lo = __uint_as_float(w[k] << 16), hi = __uint_as_float(w[k] & 0xffff0000u);
      __half2 h = __floats2half2_rn(lo, hi);
      ow[k] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(out + e) = o;
  }
}

// A paged K / V read as the flat [B][Hkv][Skv][D] tensor: element e of it
// lives on the page the table gives for its (sequence, key) (a page id outside
// the pool reads page 0 and sets bit 4 of the device error word, as the
// kernels' own lookups do).  table == nullptr: the tensor is flat already.
struct KvGather {
  const int32_t* table = nullptr;
  int npages = 0, Hkv = 1, Skv = 0, D = 0;
  int64_t page_stride = 0, tbs = 0, tps = 0;
  int* err = nullptr;
};

__device__ __forceinline__ int64_t gather_index(const KvGather& g, int64_t e) {
  if (!g.table) return e;
  const int d = (int)(e % g.D);
  const int64_t row = e / g.D;
  const int key = (int)(row % g.Skv);
  const int64_t bh = row / g.Skv;
  const int hk = (int)(bh % g.Hkv), b = (int)(bh / g.Hkv);
  int page = __ldg(g.table + (int64_t)b * g.tbs + (int64_t)(key >> 4) * g.tps);
  if ((unsigned)page >= (unsigned)g.npages) {
    if (g.err) atomicOr(g.err, 4);
    page = 0;
  }
  return (int64_t)page * g.page_stride + ((int64_t)hk * 16 + (key & 15)) * g.D + d;
}

// fp32 I/O: the largest |x| of Q, K and V (as float bits, atomicMax on
// non-negative floats orders like the values), then fp16 copies scaled by
// 2^(14 - e), e the exponent of that largest value, so every value fits fp16
// with the largest in [2^14, 2^15); dscale = {2^-(sq + sk), 2^-sv} undoes them.
// A paged K / V is read through its table (only the live rows count) and
// copied flat.
__global__ void __launch_bounds__(256) absmax3_kernel(const float* q, int64_t nq, const float* k, int64_t nk,
                                                       const float* v, int64_t nv, unsigned* amax, KvGather g) {
  // 16-byte loads (the tensors are 16-byte aligned and D % 4 == 0, so the 4
  // values share a row; n % 4 tails scalar), a block reduction in shared
  // memory, then one atomic per block and tensor
  __shared__ unsigned red[3][8];
  unsigned m[3] = {0u, 0u, 0u};
  const float* src[3] = {q, k, v};
  const int64_t n[3] = {nq, nk, nv};
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const int64_t n4 = n[t] / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
      const int64_t e = t ? gather_index(g, 4 * i) : 4 * i;
      const float4 x = __ldg(reinterpret_cast<const float4*>(src[t] + e));
      m[t] = max(m[t], max(max(__float_as_uint(fabsf(x.x)), __float_as_uint(fabsf(x.y))),
                           max(__float_as_uint(fabsf(x.z)), __float_as_uint(fabsf(x.w)))));
    }
    for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n[t]; i += stride)
      m[t] = max(m[t], __float_as_uint(fabsf(src[t][t ? gather_index(g, i) : i])));
    for (int o = 16; o; o >>= 1) m[t] = max(m[t], __shfl_xor_sync(0xffffffffu, m[t], o));
    if ((threadIdx.x & 31) == 0) red[t][threadIdx.x >> 5] = m[t];
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    unsigned b = 0u;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = max(b, red[threadIdx.x][w]);
    atomicMax(&amax[threadIdx.x], b);
  }
}

__device__ __forceinline__ int scale_shift(unsigned amax_bits) {
  const int e = (int)(amax_bits >> 23) - 127;  // exponent of the largest |x| (denormals and 0: -127)
  return min(14 - max(e, -100), 120);          // power-of-two multiplier, kept inside fp32's range
}

__global__ void __launch_bounds__(256) f32_to_f16_scaled_kernel(const float* q, int64_t nq, const float* k,
                                                                 int64_t nk, const float* v, int64_t nv,
                                                                 const unsigned* amax, __half* q16, __half* k16,
                                                                 __half* v16, float* dscale, KvGather g) {
  const int sq = scale_shift(amax[0]), sk = scale_shift(amax[1]), sv = scale_shift(amax[2]);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    dscale[0] = ldexpf(1.f, -(sq + sk));
    dscale[1] = ldexpf(1.f, -sv);
  }
  const float* src[3] = {q, k, v};
  __half* dst[3] = {q16, k16, v16};
  const int64_t n[3] = {nq, nk, nv};
  const float f[3] = {ldexpf(1.f, sq), ldexpf(1.f, sk), ldexpf(1.f, sv)};
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    uint2* d4 = reinterpret_cast<uint2*>(dst[t]);  // 4 halves
    const int64_t n4 = n[t] / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
      const int64_t e = t ? gather_index(g, 4 * i) : 4 * i;
      const float4 x = __ldg(reinterpret_cast<const float4*>(src[t] + e));
      __half2 lo = __floats2half2_rn(x.x * f[t], x.y * f[t]), hi = __floats2half2_rn(x.z * f[t], x.w * f[t]);
      d4[i] = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    }
    for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n[t]; i += stride)
      dst[t][i] = __float2half_rn(src[t][t ? gather_index(g, i) : i] * f[t]);
  }
}

template <int D, bool BF16, bool PAIR>
SgStatus launch_tc(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const TArgs& a, int grid,
                   cudaStream_t cs) {
  const int smem = PAIR ? ACfg2<D>::kSmem : ACfg<D>::kSmem;
  auto kfn = PAIR ? attn_tc2_kernel<D, BF16> : attn_tc_kernel<D, BF16>;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  SgStatus st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
  if (!(attr_set.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      cudaGetLastError();
      sg::set_error("attn_tc_kernel: cannot reserve %d bytes of shared memory: %s", smem, cudaGetErrorString(e));
      return SG_ERR_RUNTIME;
    }
    attr_set.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(PAIR ? kThreads2 : kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = cs;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, tq, tk, tv, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    sg::set_error("attn_tc_kernel launch failed: %s", cudaGetErrorString(e));
    return SG_ERR_RUNTIME;
  }
  return SG_OK;
}

std::atomic<int> g_tune_attn_tc{1};    // 0: tensor-core attention off
std::atomic<int> g_tune_attn_pair{1};  // 1: two query tiles per CTA (attn_tc2_kernel)
std::atomic<int> g_tune_attn_min_s{256};  // shortest query length sent to it

}  // namespace

namespace sg {

// Runs the tensor-core kernel when the problem qualifies (*handled = true):
// fp16 / bf16 I/O, head_dim 64 or 128, at least 256 queries, 16-byte aligned
// tensors and K / V strides.
namespace {
bool tc_qualifies(const SgFlashAttentionParams* p) {
  if (!g_tune_attn_tc.load() || p->q_pos_device) return false;
  const int io = p->io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->io_dtype;
  const int D = p->head_dim;
  if ((io != SG_DT_F16 && io != SG_DT_BF16 && io != SG_DT_F32) || (D != 64 && D != 128)) return false;
  if (io == SG_DT_F32) {  // copied to flat fp16 first: dense K / V, or pages gathered through the table
    const int Skv0 = p->S_kv > 0 ? p->S_kv : p->S;
    const int64_t dense_hs = (int64_t)Skv0 * D, dense_bs = (int64_t)std::max(1, p->num_kv_heads) * dense_hs;
    if (p->kv_pages) {
      if (p->kv_pages->page_size != kPageRows || !aligned16(p->K) || !aligned16(p->V) ||
          (p->kv_pages->page_stride * 4) % 16 != 0)
        return false;
    } else if ((p->kv_head_stride > 0 && p->kv_head_stride != dense_hs) ||
               (p->kv_batch_stride > 0 && p->kv_batch_stride != dense_bs)) {
      return false;
    }
  }
  if (p->S < g_tune_attn_min_s.load()) return false;
  const int Hkv = std::max(1, p->num_kv_heads);
  const int Skv = p->S_kv > 0 ? p->S_kv : p->S;
  const int64_t kv_hs = p->kv_head_stride > 0 ? p->kv_head_stride : (int64_t)Skv * D;
  const int64_t kv_bs = p->kv_batch_stride > 0 ? p->kv_batch_stride : (int64_t)Hkv * kv_hs;
  if (!aligned16(p->Q) || !aligned16(p->K) || !aligned16(p->V) || !aligned16(p->O)) return false;
  if (p->kv_pages && io != SG_DT_F32) {
    if (p->kv_pages->page_size != kPageRows || (p->kv_pages->page_stride * 2) % 16 != 0) return false;
  } else if (!p->kv_pages && ((kv_hs * 2) % 16 != 0 || (kv_bs * 2) % 16 != 0)) {
    return false;
  }
  const int q_pos0 = p->q_pos0 >= 0 ? p->q_pos0 : Skv - p->S;
  return q_pos0 >= 0;  // queries before the first key: the CUDA-core path reports it
}
}  // namespace

// fp32 I/O scratch: the three absolute maxima and two scales (256 bytes), then
// the scaled fp16 copies of Q, K and V.
size_t f32_scratch_parts(const SgFlashAttentionParams* p, size_t* nq, size_t* nk) {
  const int Skv = p->S_kv > 0 ? p->S_kv : p->S;
  *nq = (size_t)p->B * p->num_heads * p->S * p->head_dim;
  *nk = (size_t)p->B * std::max(1, p->num_kv_heads) * Skv * p->head_dim;
  return 256 + align_up(*nq * 2, 256) + 2 * align_up(*nk * 2, 256);
}

// Scratch of the tensor-core path: the fp16 copy of a bf16 V, or the fp16
// copies of fp32 inputs.
size_t attn_tc_scratch_bytes(const SgFlashAttentionParams* p) {
  if (!tc_qualifies(p)) return 0;
  const int io = p->io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->io_dtype;
  if (io == SG_DT_F32) {
    size_t nq, nk;
    return f32_scratch_parts(p, &nq, &nk);
  }
  if (io != SG_DT_BF16) return 0;
  const int Skv = p->S_kv > 0 ? p->S_kv : p->S;
  return align_up((size_t)p->B * std::max(1, p->num_kv_heads) * Skv * p->head_dim * 2, 256);
}

SgStatus attn_tc_run16(const SgFlashAttentionParams* p, cudaStream_t cs, void* ws, size_t ws_bytes, bool ws_external,
                       bool* handled, const float* dscale, bool o_f32);

// fp32 I/O: Q / K / V copied to fp16 with per-tensor power-of-two scales
// (exact; every value fits fp16 with 11 significant bits, the precision of the
// tensor cores' 16-bit operands), the fp16 kernel run on the copies with the
// scales undone on the scores and on O, and O written as fp32.
SgStatus attn_tc_run(const SgFlashAttentionParams* p, cudaStream_t cs, void* ws, size_t ws_bytes, bool ws_external,
                     bool* handled) {
  *handled = false;
  if (!tc_qualifies(p)) return SG_OK;
  const int io = p->io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->io_dtype;
  if (io != SG_DT_F32) return attn_tc_run16(p, cs, ws, ws_bytes, ws_external, handled, nullptr, false);
  size_t nq, nk;
  const size_t need = f32_scratch_parts(p, &nq, &nk);
  SgStatus st;
  if (ws == nullptr) {
    if (ws_external) {
      set_error("sg_flash_attention: scratch required (%zu bytes)", need);
      return SG_ERR_INVALID;
    }
    st = library_workspace(cs, need, &ws, kWsAttention);
    if (st != SG_OK) return st;
  } else {
    SG_CHECK_ARG(ws_bytes >= need && aligned16(ws), "sg_flash_attention: workspace too small (%zu < %zu bytes)",
                 ws_bytes, need);
  }
  char* w = static_cast<char*>(ws);
  unsigned* amax = reinterpret_cast<unsigned*>(w);
  float* dscale = reinterpret_cast<float*>(w + 16);
  __half* q16 = reinterpret_cast<__half*>(w + 256);
  __half* k16 = reinterpret_cast<__half*>(w + 256 + align_up(nq * 2, 256));
  __half* v16 = reinterpret_cast<__half*>(w + 256 + align_up(nq * 2, 256) + align_up(nk * 2, 256));
  SG_CUDA_TRY(cudaMemsetAsync(amax, 0, 16, cs));
  KvGather g;
  if (p->kv_pages) {
    const SgKvPages* pg = p->kv_pages;
    g.table = pg->table;
    g.npages = pg->num_pages;
    g.Hkv = std::max(1, p->num_kv_heads);
    g.Skv = p->S_kv > 0 ? p->S_kv : p->S;
    g.D = p->head_dim;
    g.page_stride = pg->page_stride;
    g.tbs = pg->table_batch_stride;
    g.tps = pg->table_page_stride;
    st = device_error_word(&g.err);
    if (st != SG_OK) return st;
  }
  const int blocks = (int)std::max<size_t>(1, std::min<size_t>((nq + nk * 2) / 1024, 148 * 4));
  absmax3_kernel<<<blocks, 256, 0, cs>>>(static_cast<const float*>(p->Q), (int64_t)nq,
                                         static_cast<const float*>(p->K), (int64_t)nk,
                                         static_cast<const float*>(p->V), (int64_t)nk, amax, g);
  st = check_launch("absmax3_kernel");
  if (st != SG_OK) return st;
  f32_to_f16_scaled_kernel<<<blocks, 256, 0, cs>>>(static_cast<const float*>(p->Q), (int64_t)nq,
                                                   static_cast<const float*>(p->K), (int64_t)nk,
                                                   static_cast<const float*>(p->V), (int64_t)nk, amax, q16, k16, v16,
                                                   dscale, g);
  st = check_launch("f32_to_f16_scaled_kernel");
  if (st != SG_OK) return st;
  SgFlashAttentionParams c = *p;
  c.Q = q16;
  c.K = k16;
  c.V = v16;
  c.io_dtype = SG_DT_F16;
  c.kv_pages = nullptr;  // the copies are flat
  const int Skv = p->S_kv > 0 ? p->S_kv : p->S;
  c.kv_head_stride = (int64_t)Skv * p->head_dim;
  c.kv_batch_stride = (int64_t)std::max(1, p->num_kv_heads) * c.kv_head_stride;
  return attn_tc_run16(&c, cs, nullptr, 0, true, handled, dscale, true);
}

SgStatus attn_tc_run16(const SgFlashAttentionParams* p, cudaStream_t cs, void* ws, size_t ws_bytes, bool ws_external,
                       bool* handled, const float* dscale, bool o_f32) {
  *handled = false;
  if (!tc_qualifies(p)) return SG_OK;
  const int io = p->io_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->io_dtype;
  const int D = p->head_dim;
  const int Hkv = std::max(1, p->num_kv_heads);
  const int Skv = p->S_kv > 0 ? p->S_kv : p->S;
  int64_t kv_hs = p->kv_head_stride > 0 ? p->kv_head_stride : (int64_t)Skv * D;
  int64_t kv_bs = p->kv_batch_stride > 0 ? p->kv_batch_stride : (int64_t)Hkv * kv_hs;
  int* err = nullptr;
  SgStatus st = device_error_word(&err);
  if (st != SG_OK) return st;
  // bf16 V -> contiguous fp16 copy for the PV product
  const void* vsrc = p->V;
  int64_t v_hs = kv_hs, v_bs = kv_bs;
  if (io == SG_DT_BF16) {
    const size_t need = attn_tc_scratch_bytes(p);
    if (ws == nullptr) {
      if (ws_external) {
        set_error("sg_flash_attention: scratch required (%zu bytes)", need);
        return SG_ERR_INVALID;
      }
      st = library_workspace(cs, need, &ws, kWsAttention);
      if (st != SG_OK) return st;
    } else {
      SG_CHECK_ARG(ws_bytes >= need && aligned16(ws), "sg_flash_attention: workspace too small (%zu < %zu bytes)",
                   ws_bytes, need);
    }
    const int64_t total8 = (int64_t)p->B * Hkv * Skv * D / 8;
    const int blocks = (int)std::min<int64_t>((total8 + 255) / 256, 148 * 16);
    const SgKvPages* pg = p->kv_pages;
    v_to_f16_kernel<<<blocks, 256, 0, cs>>>(static_cast<const __nv_bfloat16*>(p->V), pg ? pg->page_stride : kv_bs,
                                            kv_hs, Hkv, Skv, D, total8, static_cast<__half*>(ws),
                                            pg ? pg->table : nullptr, pg ? pg->table_batch_stride : 0,
                                            pg ? pg->table_page_stride : 0, pg ? pg->num_pages : 0, err);
    st = check_launch("v_to_f16_kernel");
    if (st != SG_OK) return st;
    vsrc = ws;
    v_hs = (int64_t)Skv * D;
    v_bs = (int64_t)Hkv * v_hs;
  }

  const CUtensorMapDataType dt = io == SG_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)p->S, (uint64_t)p->B * p->num_heads};
    const uint64_t str[2] = {(uint64_t)D * 2, (uint64_t)p->S * D * 2};
    const uint32_t box[3] = {64, (uint32_t)kQT, 1};
    st = make_tensor_map(&tq, dt, 3, const_cast<void*>(p->Q), dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SG_OK) return st;
  }
  const SgKvPages* pages = p->kv_pages;
  if (pages) {
    // the pool as [page][kv head][16 rows][D]; one 16-row box per page
    const uint64_t pdims[4] = {(uint64_t)D, (uint64_t)kPageRows, (uint64_t)Hkv, (uint64_t)pages->num_pages};
    const uint64_t pstr[3] = {(uint64_t)D * 2, (uint64_t)kPageRows * D * 2, (uint64_t)pages->page_stride * 2};
    const uint32_t pbox[4] = {64, (uint32_t)kPageRows, 1, 1};
    st = make_tensor_map(&tk, dt, 4, const_cast<void*>(p->K), pdims, pstr, pbox, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SG_OK) return st;
    if (io != SG_DT_BF16) {
      st = make_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(p->V), pdims, pstr, pbox,
                           CU_TENSOR_MAP_SWIZZLE_128B);
      if (st != SG_OK) return st;
    }
  } else {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)Skv, (uint64_t)Hkv, (uint64_t)p->B};
    const uint64_t str[3] = {(uint64_t)D * 2, (uint64_t)kv_hs * 2, (uint64_t)kv_bs * 2};
    const uint32_t box[4] = {64, (uint32_t)kKT, 1, 1};
    st = make_tensor_map(&tk, dt, 4, const_cast<void*>(p->K), dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SG_OK) return st;
  }
  if (!pages || io == SG_DT_BF16) {  // V flat: the caller's, or the fp16 copy of a bf16 V
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)Skv, (uint64_t)Hkv, (uint64_t)p->B};
    const uint32_t box[4] = {64, (uint32_t)kKT, 1, 1};
    const uint64_t vstr[3] = {(uint64_t)D * 2, (uint64_t)v_hs * 2, (uint64_t)v_bs * 2};
    st = make_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(vsrc), dims, vstr, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SG_OK) return st;
  }
  TArgs a{};
  a.O = p->O;
  a.B = p->B;
  a.H = p->num_heads;
  a.G = p->num_heads / Hkv;
  a.Sq = p->S;
  a.Skv = Skv;
  const float scale = p->scale > 0.f ? p->scale : 1.0f / sqrtf((float)D);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal = p->causal != 0;
  a.q_pos0 = p->q_pos0 >= 0 ? p->q_pos0 : Skv - p->S;
  a.n_qt = (p->S + kQT - 1) / kQT;
  a.err = err;
  a.o_f32 = o_f32 ? 1 : 0;
  a.dscale = dscale;
  if (pages) {
    a.pt = pages->table;
    a.pt_bs = pages->table_batch_stride;
    a.pt_ps = pages->table_page_stride;
    a.npages = pages->num_pages;
    a.paged_k = 1;
    a.paged_v = io != SG_DT_BF16;
  }
  *handled = true;
  // two query tiles per CTA when the pairs still fill the GPU (small problems keep
  // the wider grid of one tile per CTA)
  int dev = 0;
  st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  if (g_tune_attn_pair.load() && (int64_t)((a.n_qt + 1) / 2) * a.H * a.B >= sg::sm_count(dev)) {
    const int grid = ((a.n_qt + 1) / 2) * a.H * a.B;
    if (D == 64) return io == SG_DT_BF16 ? launch_tc<64, true, true>(tq, tk, tv, a, grid, cs)
                                         : launch_tc<64, false, true>(tq, tk, tv, a, grid, cs);
    return io == SG_DT_BF16 ? launch_tc<128, true, true>(tq, tk, tv, a, grid, cs)
                            : launch_tc<128, false, true>(tq, tk, tv, a, grid, cs);
  }
  const int grid = a.n_qt * a.H * a.B;
  if (D == 64) return io == SG_DT_BF16 ? launch_tc<64, true, false>(tq, tk, tv, a, grid, cs)
                                       : launch_tc<64, false, false>(tq, tk, tv, a, grid, cs);
  return io == SG_DT_BF16 ? launch_tc<128, true, false>(tq, tk, tv, a, grid, cs)
                          : launch_tc<128, false, false>(tq, tk, tv, a, grid, cs);
}

bool attn_tc_tuning(std::string_view key, int value) {
  if (key == "attn_tc.pair") {
    g_tune_attn_pair.store(value);
    return true;
  }
  if (key == "attn_tc.enable") {
    g_tune_attn_tc.store(value);
    return true;
  }
  if (key == "attn_tc.min_s") {
    g_tune_attn_min_s.store(value);
    return true;
  }
  return false;
}

}  // namespace sg
