// One decode token of a Llama-style INT4 decoder (one sequence, one GPU) as a
// single persistent kernel (sm_100a): the SDK's decode step (armsess_decode)
// without a kernel boundary between its dependent projections and attentions.
//
// Semantics are those of the per-op fused step (each op computes what its own
// kernel computes, with the reference's composition: INT4 GEMV
// compiler/kernels/cpu/matmul_neon.h:113-143, RMSNorm :154-190, RoPE
// :262-275, attention flash_attention.h:95-144, SwiGLU and the residual adds
// rounded to fp16 after every op); only the order of the fp32 sums inside a
// projection differs.
//
// Structure:
//   * one CTA per SM, all resident (cooperative launch): 16 consumer warps and
//     one producer warp;
//   * the producer streams every weight chunk this CTA uses in the whole step
//     (64 k x 128 columns of packed INT4 with its scale and zero-point rows:
//     three TMA loads, the same tiles and 128-byte swizzle as the one-row GEMV
//     kernel) through a ring of shared-memory slots (full / empty mbarriers),
//     in the order the consumers take them.  Weights do not depend on the
//     activations, so the stream runs ahead across phase boundaries as far as
//     the ring allows;
//   * the consumers run the step as phases separated by grid barriers (a
//     counter in global memory, bounded waits): per layer q|k|v, attention,
//     o, gate|up, down; then the LM head and the greedy pick.  A projection
//     phase splits its (128-column strip, k range) units over the CTAs; k-split
//     partial sums go to global scratch and the NEXT phase adds them in a fixed
//     order while it stages its activation, so a reduction costs no barrier;
//   * every CTA forms the residual row it needs (the norm needs all of it):
//     h = round(h_prev + round(sum of partials)); CTA 0 stores it for later;
//   * attention units are (kv head, key split); a unit forms its q, k, v from
//     the q|k|v partials and applies the rotary embedding, the unit holding the
//     new position appends k and v to the cache, and the key groups (which do
//     not depend on this step, except the new row, patched in from shared
//     memory) are fetched before the barrier.  The o phase merges the splits
//     (running max, sum) while staging its activation.
// Activation staging and the tensor-core reduction are the one-row GEMV's:
// 24-bit fixed point per 32 k (x = 2^(E-21) x_q, x_q = 65536 hi + 256 mid +
// lo) against the unsigned weight nibbles on mma.sync m16n8k32 u8 x s8.
// Every wait is bounded (sgd::kWaitLimitNs); a wait that gives up records
// error 1 in the library's device error word and raises the abort word, on
// which every CTA leaves.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <vector>

#include "decode_step.h"
#include "rownorm.cuh"
#include "sm100.cuh"

namespace {

constexpr int kRows = 32;                    // k-pair rows per chunk (64 k)
constexpr int kWBytes = 128 * kRows;         // 4096
constexpr int kSBytes = 128 * 2 * 2;         // two scale rows x 128 fp16
constexpr int kZBytes = 128 * 2;             // two zero-point rows x 128 int8
constexpr int kSZBytes = kSBytes + kZBytes;  // 768
constexpr int kCW = 16;                      // consumer warps
constexpr int kCT = kCW * 32;                // consumer threads
constexpr int kThreads = kCT + 32;           // + the producer warp (the last)
constexpr int kAW = 8;                       // attention warps
constexpr int kKG = 16;                      // keys per attention group (one page)
constexpr int kXSlotBytes = kRows * 8 + 2 * 16;
constexpr int kMaxLmUnits = 16;              // LM-head strips per CTA
constexpr int kKinds = 4;                    // projections per layer
constexpr int kTraceEvents = 512;

struct Gemv {
  int K = 0, N = 0, strips = 0, cpt = 0, P = 1, units = 0;
};

struct DArgs {
  const CUtensorMap* maps;  // [(layer * 4 + kind) * 3 + {W, S, Z}], then the LM head's three
  Gemv g[5];                // q|k|v, o, gate|up, down, LM head
  int layers, H, heads, kvh, D, F, vocab, nct, nspl, grp, gs, gs_shift, has_z;
  float rope_base, eps, qscale;
  const __half* embed;
  int vocab_rows;
  const __half* final_norm;
  const __half* const* in_norm;
  const __half* const* post_norm;
  __half* const* kc;
  __half* const* vc;
  int64_t kv_hs;
  const SgKvPages* pages;  // [layers] or null (flat cache)
  const int32_t* pos;
  int32_t* next;
  float* logprob;
  float* logits;
  float* part_qkv;   // [P][N_qkv]
  float* part_o;     // [P][H]
  __half* gu;        // [2 F]
  float* part_down;  // [P][H]
  float* part_attn;  // [kvh][nspl][grp][D + 2]: O, max, sum
  __half* r0;        // residual row after the down projection
  __half* r1;        // ... after the o projection
  float* argp;       // [nct][3]
  unsigned* sync;    // [0] barrier arrivals, [1] pick ticket, [2] abort
  int* err;
  // optional timeline (null: off), per CTA [kTraceEvents] (ns): [0] start;
  // [1 + 2 k] / [2 + 2 k] arrival at / release from grid barrier k, then the
  // end; [200 + p] activation staged in phase p; [300 + p] warp 0's wait for
  // weight chunks in phase p; [400] the producer's wait for free slots, [401]
  // its last issue; [420 + 4 l + kind] the producer's first issue of a projection
  uint64_t* trace;
  int ns, x_slots;
  // shared-memory layout (bytes from the 1024-aligned base)
  int off_sz, off_bars, off_x, off_xf, off_misc, off_a, off_q, off_lm;
};

// Barrier of the consumer warps only (the producer warp never joins it); the
// non-aligned form, so a warp whose lane 0 ran a spin loop may arrive diverged.
__device__ __forceinline__ void cbar() { asm volatile("barrier.sync 1, %0;" ::"n"(kCT) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int group_of(const DArgs& a, int k) {
  return a.gs_shift >= 0 ? (k >> a.gs_shift) : k / a.gs;
}

__device__ __forceinline__ void unit_chunks(const Gemv& g, int u, int& strip, int& piece, int& c0, int& c1) {
  strip = u / g.P;
  piece = u - strip * g.P;
  c0 = (g.cpt * piece) / g.P;
  c1 = (g.cpt * (piece + 1)) / g.P;
}

__device__ __forceinline__ const CUtensorMap* maps_of(const DArgs& a, int l, int kind) {
  return a.maps + ((size_t)l * kKinds + kind) * 3;
}

// ------------------------------------------------------------------ producer
__device__ void producer(const DArgs& a, uint8_t* smem, uint64_t* full, uint64_t* empty) {
  if ((threadIdx.x & 31) != 0) return;
  const int b = blockIdx.x;
  const uint32_t ns = (uint32_t)a.ns;
  const uint32_t tx = kWBytes + kSBytes + (a.has_z ? kZBytes : 0);
  uint32_t ci = 0;
  bool ok = true;
  uint64_t* tr = a.trace ? a.trace + (size_t)b * kTraceEvents : nullptr;
  uint64_t waited_ns = 0;
  for (int l = 0; l <= a.layers && ok; ++l) {
    for (int kind = 0; kind < (l < a.layers ? kKinds : 1) && ok; ++kind) {
      if (tr && 420 + l * kKinds + kind < kTraceEvents) tr[420 + l * kKinds + kind] = sgd::global_timer_ns();
      const Gemv& g = a.g[l < a.layers ? kind : 4];
      const CUtensorMap* m = maps_of(a, l, kind);
      // the next projection's descriptors, ahead of their first use
      const int nl = kind + 1 < kKinds ? l : l + 1, nk = kind + 1 < kKinds ? kind + 1 : 0;
      if (nl <= a.layers) {
        const CUtensorMap* mn = maps_of(a, nl, nk);
        for (int j = 0; j < 3; ++j) sgd::tma_prefetch_desc(mn + j);
      }
      for (int u = b; u < g.units && ok; u += a.nct) {
        int strip, piece, c0, c1;
        unit_chunks(g, u, strip, piece, c0, c1);
        for (int c = c0; c < c1; ++c) {
          const uint32_t slot = ci % ns;
          const uint64_t tw = tr ? sgd::global_timer_ns() : 0;
          if (ci >= ns && !sgd::mbar_wait(&empty[slot], ((ci / ns) - 1) & 1, a.err)) {
            atomicExch(a.sync + 2, 1u);
            ok = false;
            break;
          }
          if (tr) waited_ns += sgd::global_timer_ns() - tw;
          const int x0 = strip * 128, row0 = c * kRows;
          const int gA = group_of(a, 2 * row0);
          uint8_t* wdst = smem + (size_t)slot * kWBytes;
          uint8_t* szdst = smem + a.off_sz + (size_t)slot * kSZBytes;
          sgd::mbar_arrive_expect_tx(&full[slot], tx);
          sgd::tma_load_2d(wdst, m, x0, row0, &full[slot]);
          sgd::tma_load_2d(szdst, m + 1, x0, gA, &full[slot]);
          if (a.has_z) sgd::tma_load_2d(szdst + kSBytes, m + 2, x0, gA, &full[slot]);
          ++ci;
        }
      }
    }
  }
  if (tr) {
    tr[400] = waited_ns;
    tr[401] = sgd::global_timer_ns();
  }
  // copies still in flight land before the CTA may exit
  for (uint32_t j = ci > ns ? ci - ns : 0; j < ci; ++j) sgd::mbar_wait(&full[j % ns], (j / ns) & 1, a.err);
}

// ------------------------------------------------------------------ consumer helpers
// Grid barrier number nb (0-based) of this launch: every CTA's consumers have
// arrived nb + 1 times.  Bounded; false when this CTA or another gave up.
__device__ __forceinline__ void trace_at(const DArgs& a, int ev) {
  if (a.trace && threadIdx.x == 0 && ev < kTraceEvents)
    a.trace[(size_t)blockIdx.x * kTraceEvents + ev] = sgd::global_timer_ns();
}

__device__ bool grid_barrier(const DArgs& a, unsigned& nb, int* s_abort) {
  cbar();  // this CTA's writes of the phase are done
  trace_at(a, 1 + 2 * (int)nb);
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(a.sync, 1u);
    const unsigned target = (nb + 1) * (unsigned)a.nct;
    const uint64_t t0 = sgd::global_timer_ns();
    for (int spin = 0;; ++spin) {
      if (ld_acquire(a.sync) >= target) break;
      if ((spin & 31) == 31) {
        if (ld_acquire(a.sync + 2) != 0u) {
          *s_abort = 1;
          break;
        }
        if (sgd::global_timer_ns() - t0 > sgd::kWaitLimitNs) {
          sgd::record_error(a.err, sgd::kErrWaitTimeout);
          atomicExch(a.sync + 2, 1u);
          *s_abort = 1;
          break;
        }
      }
    }
    __threadfence();
  }
  trace_at(a, 2 + 2 * (int)nb);
  ++nb;
  cbar();
  if (*s_abort == 0) return true;
  sgd::cp_async_wait<0>();  // the CTA leaves: no copy into its shared memory may still be in flight
  return false;
}

// Sum of P k-split partials in p order, the loads batched 8 at a time so that
// they are in flight together (a loop with a runtime trip count would wait for
// each in turn).
__device__ __forceinline__ float sum_parts(const float* p0, size_t stride, int P) {
  float s = 0.f;
  for (int p = 0; p < P; p += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = p + j < P ? __ldcg(p0 + (size_t)(p + j) * stride) : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (p + j < P) s += v[j];
  }
  return s;
}

// The residual row h and its RMSNorm, for a norm phase:
//   h[k] = round(base[k] + round(sum_p part[p][k]))   (or base itself: the embedding)
//   xn[k] = round(h[k] * rms_inv * w[k])              (shared memory, fp16)
// with rms_inv summed in the order of sgn::row_rms_inv (threads 0..255 take the
// 16-byte vectors tid, tid + 256, ... and add their squares in element order,
// then a butterfly per warp and over the warps' sums), so it equals the norm
// kernel's bit for bit.  CTA 0 stores h to dst.  Vector loads of the partials,
// the residual and the norm weight are issued together.
__device__ void norm_row(const DArgs& a, __half* xn, const __half* base, const float* part, int P, __half* dst,
                         const __half* w, float* red32) {
  const int nv = a.H / 8;
  float ss = 0.f;
  if (threadIdx.x < sgn::kNormThreads) {
#pragma unroll 1
    for (int j = 0; j < sgn::kNormVecPerThread; ++j) {
      const int v = threadIdx.x + j * sgn::kNormThreads;
      if (v >= nv) break;
      float b8[8];
      sgn::unpack8<__half>(__ldcg(reinterpret_cast<const uint4*>(base) + v), b8);
      if (part) {
        float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int p = 0; p < P; p += 4) {
          float4 q[4][2];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float4* src = reinterpret_cast<const float4*>(part + (size_t)(p + t) * a.H) + 2 * v;
            q[t][0] = p + t < P ? __ldcg(src) : make_float4(0.f, 0.f, 0.f, 0.f);
            q[t][1] = p + t < P ? __ldcg(src + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            if (p + t >= P) continue;
            s8[0] += q[t][0].x;
            s8[1] += q[t][0].y;
            s8[2] += q[t][0].z;
            s8[3] += q[t][0].w;
            s8[4] += q[t][1].x;
            s8[5] += q[t][1].y;
            s8[6] += q[t][1].z;
            s8[7] += q[t][1].w;
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) b8[e] = __half2float(__float2half_rn(__half2float(__float2half_rn(s8[e])) + b8[e]));
      }
      ss = sgn::sumsq8(b8, ss);
      const uint4 hv = sgn::pack8<__half>(b8);
      reinterpret_cast<uint4*>(xn)[v] = hv;
      if (dst && blockIdx.x == 0) reinterpret_cast<uint4*>(dst)[v] = hv;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  cbar();  // red32 may still be read by a previous reduction
  if (lane == 0) red32[wp] = ss;
  cbar();
  float t = lane < kCW ? red32[lane] : 0.f;
#pragma unroll
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  const float rms = 1.0f / sqrtf(t / (float)a.H + a.eps);
  // the same thread rewrites the vectors it wrote: no barrier needed in between
  if (threadIdx.x < sgn::kNormThreads) {
#pragma unroll 1
    for (int j = 0; j < sgn::kNormVecPerThread; ++j) {
      const int v = threadIdx.x + j * sgn::kNormThreads;
      if (v >= nv) break;
      float h8[8], w8[8], y[8];
      sgn::unpack8<__half>(reinterpret_cast<const uint4*>(xn)[v], h8);
      sgn::unpack8<__half>(__ldg(reinterpret_cast<const uint4*>(w) + v), w8);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = __half2float(__float2half_rn(h8[e] * rms * w8[e]));
      reinterpret_cast<uint4*>(xn)[v] = sgn::pack8<__half>(y);
    }
  }
  cbar();
}

// Stages x over k-pair rows [lo * 32, hi * 32) as 24-bit fixed point with one
// power-of-two scale per 32 k (the one-row GEMV's staging, w4_gemv_mma.cu);
// fn(k) gives x at k (0 past the end).
template <class F>
__device__ __forceinline__ void stage_rows(uint2* xst, int4* xgrp, int lo, int hi, F fn) {
  const int lane = threadIdx.x & 31;
  const int n = (hi - lo) * kRows;
  for (int idx = threadIdx.x; idx < n; idx += kCT) {
    const int k = 2 * (lo * kRows + idx);
    const float xe = fn(k), xo = fn(k + 1);
    float m = fmaxf(fabsf(xe), fabsf(xo));
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int E = max((__float_as_int(m) >> 23) - 127, -100);
    const float inv = __int_as_float((127 + 21 - E) << 23);
    const float sxv = __int_as_float((127 - 21 + E) << 23);
    const int qe = __float2int_rn(xe * inv), qo = __float2int_rn(xo * inv);
    const int le = ((qe + 128) & 255) - 128, lo8 = ((qo + 128) & 255) - 128;
    const int re = (qe - le) >> 8, ro = (qo - lo8) >> 8;
    const int me = ((re + 128) & 255) - 128, mo = ((ro + 128) & 255) - 128;
    const int he = (re - me) >> 8, ho = (ro - mo) >> 8;
    xst[idx] = make_uint2((uint32_t)(he & 255) | ((uint32_t)(ho & 255) << 8) | ((uint32_t)(me & 255) << 16) |
                              ((uint32_t)(mo & 255) << 24),
                          (uint32_t)(le & 255) | ((uint32_t)(lo8 & 255) << 8));
    int shm = re + ro, slo = le + lo8;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
      shm += __shfl_xor_sync(0xffffffffu, shm, o);
      slo += __shfl_xor_sync(0xffffffffu, slo, o);
    }
    if ((lane & 15) == 0) xgrp[idx >> 4] = make_int4(__float_as_int(sxv), shm, slo, 0);
  }
}

// One chunk (64 k x 128 columns) of one warp: the one-row GEMV's tensor-core
// step and epilogue (lane owns columns 16 g + t + 4 i of the strip).
template <bool HAS_Z>
__device__ __forceinline__ void chunk_mma(const DArgs& a, const uint8_t* wst, const uint8_t* szs, const uint2* xs,
                                          const int4* xg, int k0, float (&acc)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int be = g >> 1, bv = g & 1;
  const uint32_t sel_e = (0x4444u & ~(0xFu << (4 * be))) | ((uint32_t)(2 * bv) << (4 * be));
  const uint32_t sel_o = (0x4444u & ~(0xFu << (4 * be))) | ((uint32_t)(2 * bv + 1) << (4 * be));
  const uint32_t woff0 = 256u * t + ((uint32_t)(g ^ (2 * t)) << 4);
  const uint32_t woff1 = 256u * t + ((uint32_t)(g ^ (2 * t + 1)) << 4);
  const uint8_t* xr = reinterpret_cast<const uint8_t*>(xs) + 16 * t;
  int d[2][2][4], e[2][2][4];
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
  const int gA = group_of(a, k0), gB = group_of(a, k0 + 32);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int srow = h ? (gB - gA) : 0;
    const int4 x4 = xg[h];
    const float sxh = __int_as_float(x4.x);
    const __half* sc_row = reinterpret_cast<const __half*>(szs + srow * 256) + 16 * g + t;
    const int8_t* z_row = reinterpret_cast<const int8_t*>(szs + kSBytes + srow * 128) + 16 * g + t;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int jm = i >> 1, fr = (i & 1) * 2;
      const int z8 = HAS_Z ? 8 + (int)z_row[4 * i] : 8;
      const int hm = d[h][jm][fr] * 256 + d[h][jm][fr + 1] - z8 * x4.y;
      const int lw = e[h][jm][fr] - z8 * x4.z;
      acc[i] = fmaf(__half2float(sc_row[4 * i]) * sxh, fmaf(256.f, (float)hm, (float)lw), acc[i]);
    }
  }
}

// The chunk stream of one projection phase: stage x over the union of this
// CTA's units, then per unit its chunks round-robin over the consumer warps
// (chunk ci of the CTA's stream -> warp ci % 16), the warps' column sums added
// in warp order, out(piece, col, value, unit index) for every column < N.
template <bool HAS_Z, class X, class OUT>
__device__ bool gemv_phase(const DArgs& a, const Gemv& g, uint8_t* smem, uint64_t* full, uint64_t* empty,
                           uint32_t& ci, int* s_abort, unsigned ph, X xfn, OUT out) {
  const int b = blockIdx.x;
  if (b >= g.units) return true;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint2* xst = reinterpret_cast<uint2*>(smem + a.off_x);
  int4* xgrp = reinterpret_cast<int4*>(xst + (size_t)a.x_slots * kRows);
  float* red = reinterpret_cast<float*>(smem + a.off_a);
  int lo = g.cpt, hi = 0;
  for (int u = b; u < g.units; u += a.nct) {
    int strip, piece, c0, c1;
    unit_chunks(g, u, strip, piece, c0, c1);
    lo = min(lo, c0);
    hi = max(hi, c1);
  }
  stage_rows(xst, xgrp, lo, hi, xfn);
  cbar();
  const uint32_t ns = (uint32_t)a.ns;
  uint64_t wait0 = 0;  // warp 0's time waiting for weight chunks (timeline only)
  if (a.trace && threadIdx.x == 0 && 200 + ph < (unsigned)kTraceEvents)
    a.trace[(size_t)b * kTraceEvents + 200 + ph] = sgd::global_timer_ns();  // staging done
  int j = 0;
  for (int u = b; u < g.units; u += a.nct, ++j) {
    int strip, piece, c0, c1;
    unit_chunks(g, u, strip, piece, c0, c1);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = c0; c < c1; ++c, ++ci) {
      if ((int)(ci % kCW) != warp) continue;
      const uint32_t slot = ci % ns;
      const uint64_t tw = (a.trace && warp == 0) ? sgd::global_timer_ns() : 0;
      const bool waited = sgd::mbar_wait(&full[slot], (ci / ns) & 1, a.err);
      if (a.trace && warp == 0) wait0 += sgd::global_timer_ns() - tw;
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) {
          *s_abort = 1;
          atomicExch(a.sync + 2, 1u);
        }
        continue;
      }
      chunk_mma<HAS_Z>(a, smem + (size_t)slot * kWBytes, smem + a.off_sz + (size_t)slot * kSZBytes,
                       xst + (size_t)(c - lo) * kRows, xgrp + (size_t)(c - lo) * 2, 64 * c, acc);
      __syncwarp();
      if (lane == 0) sgd::mbar_arrive(&empty[slot]);
    }
    float* r0 = red + warp * 128 + 16 * (lane >> 2) + (lane & 3);
#pragma unroll
    for (int i = 0; i < 4; ++i) r0[4 * i] = acc[i];
    cbar();
    if (threadIdx.x < 128) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) v += red[w * 128 + threadIdx.x];
      const int col = strip * 128 + threadIdx.x;
      if (col < g.N) out(piece, col, v, j);
    }
    cbar();
    if (*s_abort) return false;
  }
  if (a.trace && threadIdx.x == 0 && 300 + ph < (unsigned)kTraceEvents)
    a.trace[(size_t)b * kTraceEvents + 300 + ph] = wait0;
  return true;
}

// ------------------------------------------------------------------ attention
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, const void* smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(sgd::smem_u32(smem_row)));
}

// Element offset of key `key`, head hk, in layer l's K (or V) cache.  A page
// id outside the pool sets bit 4 of the device error word and reads page 0
// (*valid = false: a write there is dropped), as the per-op kernels do.
__device__ __forceinline__ int64_t kv_row(const DArgs& a, int l, int hk, int key, bool* valid = nullptr) {
  if (valid) *valid = true;
  if (!a.pages) return (int64_t)hk * a.kv_hs + (int64_t)key * a.D;
  const SgKvPages& pg = a.pages[l];
  int page = __ldg(pg.table + (int64_t)(key >> 4) * pg.table_page_stride);
  if ((unsigned)page >= (unsigned)pg.num_pages) {
    atomicOr(a.err, 4);
    page = 0;
    if (valid) *valid = false;
  }
  return (int64_t)page * pg.page_stride + ((int64_t)hk * kKG + (key & 15)) * a.D;
}

template <int D>
struct AttnUnit {
  int hk, sp, j0, j1, ngroups;
};

// Fetches group gi (16 keys from j0 + 16 gi) of a unit into this warp's buffer
// (cp.async, zeros past j1).
template <int D>
__device__ __forceinline__ void attn_fetch(const DArgs& a, int l, const AttnUnit<D>& u, int gi, __half* kd) {
  constexpr int KP = D + 8, NP = kKG * D / 8 / 32;
  const int lane = threadIdx.x & 31;
  const int key0 = u.j0 + gi * kKG;
  const int64_t gbase = kv_row(a, l, u.hk, key0);
  __half* vd = kd + kKG * KP;
#pragma unroll
  for (int q = 0; q < NP; ++q) {
    const int pc = lane + 32 * q;
    const int kl = pc / (D / 8), part = pc % (D / 8);
    const bool live = key0 + kl < u.j1;
    const int64_t e0 = gbase + (int64_t)(live ? kl : 0) * D + part * 8;
    sgd::cp_async_16(kd + kl * KP + part * 8, a.kc[l] + e0, live);
    sgd::cp_async_16(vd + kl * KP + part * 8, a.vc[l] + e0, live);
  }
}

template <int D>
__device__ __forceinline__ AttnUnit<D> attn_unit(const DArgs& a, int u, int live, int kps) {
  AttnUnit<D> r;
  r.hk = u / a.nspl;
  r.sp = u - r.hk * a.nspl;
  r.j0 = r.sp * kps;
  r.j1 = min(live, r.j0 + kps);
  r.ngroups = r.j1 > r.j0 ? (r.j1 - r.j0 + kKG - 1) / kKG : 0;
  return r;
}

// One attention unit: q, k, v of kv head hk from the q|k|v partials (rounded
// as the q|k|v projection stores them, rotated as sg_qkv_rope_append does),
// the KV append if the unit holds the new position, then the warp-split
// online softmax over its keys (the decode attention kernel's per-warp step)
// and the merge of the warps in warp order into part_attn.
template <int D>
__device__ bool attn_do_unit(const DArgs& a, int l, const AttnUnit<D>& u, int pos, bool prefetched, uint8_t* smem,
                             int* s_abort) {
  constexpr int KP = D + 8, NT = D / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int grp = a.grp, nq = a.g[0].N;
  float* qs = reinterpret_cast<float*>(smem + a.off_q);  // [grp][D], then k [D], v [D]
  float* kn = qs + grp * D;
  float* vn = kn + D;
  __half* abuf = reinterpret_cast<__half*>(smem + a.off_a);
  // ---- q (grp heads), k, v: sums of the partials in p order, rounded to fp16
  const int P = a.g[0].P;
  const int nv = (grp + 2) * D;
  for (int i = threadIdx.x; i < nv; i += kCT) {
    int col;
    if (i < grp * D) col = (u.hk * grp) * D + i;
    else if (i < (grp + 1) * D) col = (a.heads + u.hk) * D + (i - grp * D);
    else col = (a.heads + a.kvh + u.hk) * D + (i - (grp + 1) * D);
    qs[i] = __half2float(__float2half_rn(sum_parts(a.part_qkv + col, nq, P)));
  }
  cbar();
  // ---- rotary pairs (i, i + D/2) of q and k
  const int half = D / 2;
  for (int pi = threadIdx.x; pi < (grp + 1) * half; pi += kCT) {
    const int r = pi / half, i = pi - r * half;
    float* row = qs + r * D;  // r == grp: the k row
    float y0, y1;
    sgd::rope_pair(row[i], row[i + half], pos, i, D, a.rope_base, &y0, &y1);
    row[i] = __half2float(__float2half_rn(y0));
    row[i + half] = __half2float(__float2half_rn(y1));
  }
  cbar();
  // ---- the new row into the cache (the unit whose range holds the position)
  if (pos >= u.j0 && pos < u.j1 && threadIdx.x < D) {
    bool valid;
    const int64_t off = kv_row(a, l, u.hk, pos, &valid) + threadIdx.x;
    if (valid) {
      a.kc[l][off] = __float2half_rn(kn[threadIdx.x]);
      a.vc[l][off] = __float2half_rn(vn[threadIdx.x]);
    }
  }
  // ---- warp-split attention over the unit's keys
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int q = 0; q < 4; ++q) o[n][q] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  if (warp < kAW) {
    __half* ks = abuf + (size_t)warp * 2 * kKG * KP;
    __half* vs = ks + kKG * KP;
    auto q_at = [&](int r, int d) -> float { return r < grp ? qs[r * D + d] * a.qscale : 0.f; };
    uint32_t qf[D / 16][4];
#pragma unroll
    for (int s2 = 0; s2 < D / 16; ++s2) {
      const int d0 = 16 * s2 + 2 * t;
      qf[s2][0] = pack_half2(q_at(g, d0), q_at(g, d0 + 1));
      qf[s2][1] = pack_half2(q_at(g + 8, d0), q_at(g + 8, d0 + 1));
      qf[s2][2] = pack_half2(q_at(g, d0 + 8), q_at(g, d0 + 9));
      qf[s2][3] = pack_half2(q_at(g + 8, d0 + 8), q_at(g + 8, d0 + 9));
    }
    for (int gi = warp; gi < u.ngroups; gi += kAW) {
      if (!(prefetched && gi == warp)) {
        attn_fetch<D>(a, l, u, gi, ks);
        sgd::cp_async_commit();
      }
      sgd::cp_async_wait<0>();
      const int key0 = u.j0 + gi * kKG;
      if (pos >= key0 && pos < key0 + kKG) {  // the new row: from shared memory, not the cache
        const int kl = pos - key0;
        for (int d = lane; d < D; d += 32) {
          ks[kl * KP + d] = __float2half_rn(kn[d]);
          vs[kl * KP + d] = __float2half_rn(vn[d]);
        }
      }
      __syncwarp();
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
      float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int key = key0 + 8 * h + 2 * t + (q & 1);
          sc[h][q] = key < u.j1 ? sc[h][q] : -INFINITY;
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
      const uint32_t pa0 = pack_half2(p[0][0], p[0][1]), pa1 = pack_half2(p[0][2], p[0][3]);
      const uint32_t pa2 = pack_half2(p[1][0], p[1][1]), pa3 = pack_half2(p[1][2], p[1][3]);
      const __half* vrow = vs + (lane & 15) * KP;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        uint32_t b0, b1;
        ldmatrix_x2_trans(b0, b1, vrow + 8 * n);
        sgd::mma_f16_16816(o[n], pa0, pa1, pa2, pa3, b0, b1);
      }
      __syncwarp();  // the buffer is refilled by the warp's next group
    }
  }
  sgd::cp_async_wait<0>();
  cbar();  // every warp is done with its buffer: the merge area reuses it
  float* wm = reinterpret_cast<float*>(abuf);  // [warp][16][D + 2]
  if (warp < kAW) {
    float* mine = wm + (size_t)warp * 16 * (D + 2);
    const int r_lo = g, r_hi = g + 8;
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
  }
  cbar();
  float* dst = a.part_attn + ((size_t)u.hk * a.nspl + u.sp) * grp * (D + 2);
  for (int i = threadIdx.x; i < grp * (D + 2); i += kCT) {
    const int r = i / (D + 2), d = i - r * (D + 2);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAW; ++w) M = fmaxf(M, wm[((size_t)w * 16 + r) * (D + 2) + D]);
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kAW; ++w) {
      const float* pr = wm + ((size_t)w * 16 + r) * (D + 2);
      if (pr[D] == -INFINITY) continue;
      const float wt = exp2f(pr[D] - M);
      acc = fmaf(d == D ? 0.f : (d == D + 1 ? pr[D + 1] : pr[d]), wt, acc);
    }
    dst[i] = d == D ? M : acc;
  }
  cbar();
  return *s_abort == 0;
}

// ------------------------------------------------------------------ the kernel
template <int D, bool HAS_Z>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(DArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = sgd::align_smem_1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bars);
  uint64_t* empty = full + a.ns;
  __shared__ int s_abort;
  __shared__ float s_red[32];
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.ns; ++i) {
      sgd::mbar_init(&full[i], 1);
      sgd::mbar_init(&empty[i], 1);
    }
    sgd::fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  if (threadIdx.x >= kCT) {
    producer(a, smem, full, empty);
    return;
  }
  const int b = blockIdx.x, warp = threadIdx.x >> 5;
  trace_at(a, 0);
  const int pos = *a.pos;
  const int token = *a.next;
  const int live = pos + 1;
  int kps = (live + a.nspl - 1) / a.nspl;
  kps = max(kKG, (kps + kKG - 1) / kKG * kKG);
  __half* xf = reinterpret_cast<__half*>(smem + a.off_xf);
  float* xa = reinterpret_cast<float*>(smem + a.off_xf);  // the o phase's merged attention values
  float* misc = reinterpret_cast<float*>(smem + a.off_misc);
  float* lmv = reinterpret_cast<float*>(smem + a.off_lm);
  uint32_t ci = 0;
  unsigned nb = 0;
  const int H = a.H;
  const __half* emb = a.embed + (int64_t)min(max(token, 0), a.vocab_rows - 1) * H;

  for (int l = 0; l < a.layers; ++l) {
    // ---- q|k|v of RMSNorm(h): h is the embedding row or h1 + down partials
    if (l > 0 && !grid_barrier(a, nb, &s_abort)) return;
    if (l == 0) norm_row(a, xf, emb, nullptr, 0, a.r0, a.in_norm[l], s_red);
    else norm_row(a, xf, a.r1, a.part_down, a.g[3].P, a.r0, a.in_norm[l], s_red);
    {
      auto xfn = [&](int k) -> float { return k < H ? __half2float(xf[k]) : 0.f; };
      const int nq = a.g[0].N;
      auto out = [&](int piece, int col, float v, int) { a.part_qkv[(size_t)piece * nq + col] = v; };
      if (!gemv_phase<HAS_Z>(a, a.g[0], smem, full, empty, ci, &s_abort, nb, xfn, out)) return;
    }
    // ---- attention: key groups that do not depend on this step first
    const int nunits = a.kvh * a.nspl;
    if (b < nunits && warp < kAW) {
      const AttnUnit<D> u = attn_unit<D>(a, b, live, kps);
      if (warp < u.ngroups) {
        __half* ks = reinterpret_cast<__half*>(smem + a.off_a) + (size_t)warp * 2 * kKG * (D + 8);
        attn_fetch<D>(a, l, u, warp, ks);
      }
      sgd::cp_async_commit();
    }
    if (!grid_barrier(a, nb, &s_abort)) return;
    for (int uu = b; uu < nunits; uu += a.nct) {
      const AttnUnit<D> u = attn_unit<D>(a, uu, live, kps);
      if (!attn_do_unit<D>(a, l, u, pos, uu == b, smem, &s_abort)) return;
    }
    // ---- o: the splits merged per head while staging
    if (!grid_barrier(a, nb, &s_abort)) return;
    {
      const Gemv& g = a.g[1];
      if (b < g.units) {
        int strip, piece, c0, c1;
        unit_chunks(g, b, strip, piece, c0, c1);  // one unit per CTA (the plan keeps units <= CTAs)
        const int k_lo = c0 * 64, k_hi = min(H, c1 * 64);
        const int h0 = k_lo / D, h1 = (k_hi + D - 1) / D;
        const int nsp = a.nspl;
        // per head: the splits' (max, sum) into shared memory, their weights
        // exp2(m_sp - M) and the sum L = sum_sp l_sp w_sp in split order
        const int nh = h1 - h0;
        const size_t sstride = (size_t)a.grp * (D + 2);
        float* wts = misc;                        // [nh][nsp + 1]: weights, then L
        float* mls = misc + nh * (nsp + 1);       // [nh][nsp][2]: max, sum
        for (int i = threadIdx.x; i < nh * nsp; i += kCT) {
          const int hh = i / nsp, sp = i - hh * nsp;
          const int h = h0 + hh, hk = h / a.grp, r = h - hk * a.grp;
          const float* pr = a.part_attn + ((size_t)hk * nsp * a.grp + r) * (D + 2) + sp * sstride;
          mls[2 * i] = __ldcg(pr + D);
          mls[2 * i + 1] = __ldcg(pr + D + 1);
        }
        cbar();
        for (int hh = warp; hh < nh; hh += kCW) {
          const int lane = threadIdx.x & 31;
          float M = -INFINITY;
          for (int sp = lane; sp < nsp; sp += 32) M = fmaxf(M, mls[2 * (hh * nsp + sp)]);
#pragma unroll
          for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
          for (int sp = lane; sp < nsp; sp += 32) {
            const float m = mls[2 * (hh * nsp + sp)];
            wts[hh * (nsp + 1) + sp] = m == -INFINITY ? 0.f : exp2f(m - M);
          }
          __syncwarp();
          if (lane == 0) {  // in split order; empty splits (weight 0) add nothing
            float L = 0.f;
            for (int sp = 0; sp < nsp; ++sp) {
              const float wt = wts[hh * (nsp + 1) + sp];
              if (wt != 0.f) L = fmaf(mls[2 * (hh * nsp + sp) + 1], wt, L);
            }
            wts[hh * (nsp + 1) + nsp] = L;
          }
        }
        cbar();
        for (int k = k_lo + threadIdx.x; k < k_hi; k += kCT) {
          const int h = k / D, d = k - h * D, hh = h - h0;
          const int hk = h / a.grp, r = h - hk * a.grp;
          const float* pr = a.part_attn + ((size_t)hk * nsp * a.grp + r) * (D + 2) + d;
          const float* wt = wts + hh * (nsp + 1);
          float acc = 0.f;
          for (int sp = 0; sp < nsp; sp += 8) {  // loads batched; an empty split holds O = 0 and weight 0
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = sp + j < nsp ? __ldcg(pr + (sp + j) * sstride) : 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (sp + j < nsp && wt[sp + j] != 0.f) acc = fmaf(v[j], wt[sp + j], acc);
          }
          const float L = wt[nsp];
          xa[k - k_lo] = __half2float(__float2half_rn(L > 0.f ? acc / L : 0.f));
        }
        cbar();
        auto xfn = [&](int k) -> float { return k < k_hi ? xa[k - k_lo] : 0.f; };
        auto out = [&](int piece2, int col, float v, int) { a.part_o[(size_t)piece2 * H + col] = v; };
        if (!gemv_phase<HAS_Z>(a, g, smem, full, empty, ci, &s_abort, nb, xfn, out)) return;
      }
    }
    // ---- gate|up of RMSNorm(h1), h1 = h + o
    if (!grid_barrier(a, nb, &s_abort)) return;
    norm_row(a, xf, a.r0, a.part_o, a.g[1].P, a.r1, a.post_norm[l], s_red);
    {
      auto xfn = [&](int k) -> float { return k < H ? __half2float(xf[k]) : 0.f; };
      auto out = [&](int, int col, float v, int) { a.gu[col] = __float2half_rn(v); };
      if (!gemv_phase<HAS_Z>(a, a.g[2], smem, full, empty, ci, &s_abort, nb, xfn, out)) return;
    }
    // ---- down of SwiGLU(gate, up)
    if (!grid_barrier(a, nb, &s_abort)) return;
    {
      const int F = a.F;
      const Gemv& g = a.g[3];
      int k_lo = 0, k_hi = 0;
      if (b < g.units) {  // one unit per CTA
        int strip, piece, c0, c1;
        unit_chunks(g, b, strip, piece, c0, c1);
        k_lo = c0 * 64;
        k_hi = min(F, c1 * 64);
        for (int v = threadIdx.x; v < (k_hi - k_lo) / 8; v += kCT) {  // k_lo, k_hi: multiples of 8
          float g8[8], u8[8];
          sgn::unpack8<__half>(__ldcg(reinterpret_cast<const uint4*>(a.gu + k_lo) + v), g8);
          sgn::unpack8<__half>(__ldcg(reinterpret_cast<const uint4*>(a.gu + F + k_lo) + v), u8);
          __half y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = sgd::swiglu_value<__half>(g8[e], u8[e]);
          reinterpret_cast<uint4*>(xf)[v] = *reinterpret_cast<const uint4*>(y);
        }
        cbar();
      }
      auto xfn = [&](int k) -> float { return k < k_hi ? __half2float(xf[k - k_lo]) : 0.f; };
      auto out = [&](int piece, int col, float v, int) { a.part_down[(size_t)piece * H + col] = v; };
      if (!gemv_phase<HAS_Z>(a, a.g[3], smem, full, empty, ci, &s_abort, nb, xfn, out)) return;
    }
  }
  // ---- final norm, LM head, greedy pick
  if (!grid_barrier(a, nb, &s_abort)) return;
  norm_row(a, xf, a.r1, a.part_down, a.g[3].P, nullptr, a.final_norm, s_red);
  {
    auto xfn = [&](int k) -> float { return k < H ? __half2float(xf[k]) : 0.f; };
    auto out = [&](int, int col, float v, int j) {
      a.logits[col] = v;
      lmv[j * 128 + (col & 127)] = v;
    };
    if (!gemv_phase<HAS_Z>(a, a.g[4], smem, full, empty, ci, &s_abort, nb, xfn, out)) return;
  }
  // this CTA's (max, first index of the max, sum of exp(x - max)) over its columns
  const Gemv& gl = a.g[4];
  float best = -INFINITY;
  int bi = 0x7fffffff;
  int nval = 0;
  for (int u = b; u < gl.units; u += a.nct) ++nval;
  for (int i = threadIdx.x; i < nval * 128; i += kCT) {
    const int j = i >> 7, col = (b + j * a.nct) * 128 + (i & 127);
    if (col >= a.vocab) continue;
    const float v = lmv[i];
    if (v > best || (v == best && col < bi)) {
      best = v;
      bi = col;
    }
  }
  float* sv = misc;  // [16] max, [16] index, [16] sum
  int* si = reinterpret_cast<int*>(misc + 16);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  cbar();
  best = sv[0];
  bi = si[0];
  for (int w = 1; w < kCW; ++w)
    if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
      best = sv[w];
      bi = si[w];
    }
  float sum = 0.f;
  if (best != -INFINITY)
    for (int i = threadIdx.x; i < nval * 128; i += kCT) {
      const int j = i >> 7, col = (b + j * a.nct) * 128 + (i & 127);
      if (col < a.vocab) sum += expf(lmv[i] - best);
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  cbar();
  if (lane == 0) sv[32 + warp] = sum;
  cbar();
  __shared__ int s_last;
  trace_at(a, 1 + 2 * (int)nb);
  if (threadIdx.x == 0) {
    float tsum = 0.f;
    for (int w = 0; w < kCW; ++w) tsum += sv[32 + w];
    a.argp[3 * b] = best;
    a.argp[3 * b + 1] = __int_as_float(bi);
    a.argp[3 * b + 2] = tsum;
    __threadfence();
    s_last = atomicAdd(a.sync + 1, 1u) == (unsigned)a.nct - 1 ? 1 : 0;
    __threadfence();
  }
  cbar();
  if (!s_last) return;
  // the last CTA: merge the CTAs' triples (equal maxima keep the lowest index)
  float* pm = misc + 64;                 // [nct] max
  int* pi = reinterpret_cast<int*>(pm + a.nct);
  float* ps = pm + 2 * a.nct;
  for (int c = threadIdx.x; c < a.nct; c += kCT) {
    pm[c] = __ldcg(a.argp + 3 * c);
    pi[c] = __float_as_int(__ldcg(a.argp + 3 * c + 1));
    ps[c] = __ldcg(a.argp + 3 * c + 2);
  }
  cbar();
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    int idx = 0x7fffffff;
    for (int c = 0; c < a.nct; ++c)
      if (pm[c] > M || (pm[c] == M && pi[c] < idx)) {
        M = pm[c];
        idx = pi[c];
      }
    float L = 0.f;
    if (M != -INFINITY)
      for (int c = 0; c < a.nct; ++c)
        if (pm[c] != -INFINITY) L += ps[c] * expf(pm[c] - M);
    const int r = idx == 0x7fffffff ? 0 : idx;
    *a.next = r;
    *a.logprob = __ldcg(a.logits + r) - M - logf(L);
  }
}

}  // namespace

// ------------------------------------------------------------------ host side
namespace sg {

struct DecodeStep {
  uint64_t* trace = nullptr;  // [nct][kTraceEvents] when tracing
  int dev = 0;
  int D = 0;
  bool has_z = true;
  DArgs a{};
  size_t smem = 0;
  char* mem = nullptr;  // one allocation: tensor maps, pointer tables, scratch
  size_t mem_bytes = 0;
};

namespace {

Gemv plan_gemv(int K, int N, int nct, bool split) {
  Gemv g;
  g.K = K;
  g.N = N;
  g.strips = (N + 127) / 128;
  g.cpt = ((K + 1) / 2 + kRows - 1) / kRows;
  // k-split projections keep one unit per CTA (the o phase relies on it)
  g.P = split ? std::max(1, std::min(g.cpt, nct / g.strips)) : 1;
  g.units = g.strips * g.P;
  return g;
}

template <int D, bool Z>
void* kernel_ptr() {
  return reinterpret_cast<void*>(decode_step_kernel<D, Z>);
}

void* pick_kernel(int D, bool z) {
  if (D == 64) return z ? kernel_ptr<64, true>() : kernel_ptr<64, false>();
  return z ? kernel_ptr<128, true>() : kernel_ptr<128, false>();
}

}  // namespace

const char* decode_step_unsupported(const DsModel& m, int dev) {
  if (m.layers < 1 || m.hidden < 64 || m.heads < 1 || m.kv_heads < 1) return "model shape";
  if (m.head_dim != 64 && m.head_dim != 128) return "head_dim other than 64 or 128";
  if (m.heads % m.kv_heads != 0 || m.heads / m.kv_heads > 16) return "query heads per kv head";
  if (m.hidden % 8 != 0 || m.hidden > sgn::kNormMaxN) return "hidden size";
  if (m.ffn % 8 != 0) return "SwiGLU width";
  if (m.group_size <= 0 || m.group_size % 32 != 0) return "group size";
  if (!m.lm.qw) return "an fp16 LM head";
  const DsLinear* all[4] = {nullptr, nullptr, nullptr, nullptr};
  for (int l = 0; l < m.layers; ++l) {
    all[0] = &m.qkv[l];
    all[1] = &m.o[l];
    all[2] = &m.gu[l];
    all[3] = &m.down[l];
    for (const DsLinear* L : all)
      if (!L->qw || !L->scales || L->N % 16 != 0 || (L->zeros == nullptr) != (m.qkv[0].zeros == nullptr))
        return "a projection's layout";
  }
  if ((m.lm.zeros == nullptr) != (m.qkv[0].zeros == nullptr) || m.lm.N % 16 != 0) return "the LM head's layout";
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return "device query";
  }
  if ((m.lm.N + 127) / 128 > sms * kMaxLmUnits) return "vocabulary too large for one wave of LM-head strips";
  if (m.kv_heads > sms) return "more kv heads than SMs";
  return nullptr;
}

size_t decode_step_device_bytes(const DecodeStep* ds) { return ds ? ds->mem_bytes : 0; }

SgStatus decode_step_trace(DecodeStep* ds, bool on, uint64_t* host, size_t cap, size_t* n, int* ctas) {
  SG_CHECK_ARG(ds, "decode step trace: no step kernel");
  *ctas = ds->a.nct;
  *n = 0;
  if (on && !ds->trace) {
    const size_t bytes = (size_t)ds->a.nct * kTraceEvents * 8;
    SG_CUDA_TRY(cudaMalloc(&ds->trace, bytes));
    SG_CUDA_TRY(cudaMemset(ds->trace, 0, bytes));
  }
  if (!on && ds->trace) {
    cudaFree(ds->trace);
    ds->trace = nullptr;
  }
  if (host && ds->trace) {
    const size_t total = (size_t)ds->a.nct * kTraceEvents;
    *n = std::min(cap, total);
    SG_CUDA_TRY(cudaMemcpy(host, ds->trace, *n * 8, cudaMemcpyDeviceToHost));
  }
  return SG_OK;
}

void decode_step_destroy(DecodeStep* ds) {
  if (!ds) return;
  if (ds->trace) cudaFree(ds->trace);
  if (ds->mem) cudaFree(ds->mem);
  delete ds;
}

SgStatus decode_step_create(const DsModel& m, int dev, DecodeStep** out) {
  *out = nullptr;
  if (const char* why = decode_step_unsupported(m, dev)) {
    set_error("decode step kernel: unsupported %s", why);
    return SG_ERR_UNSUPPORTED;
  }
  int sms = 0;
  SG_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  auto* ds = new DecodeStep();
  ds->dev = dev;
  ds->D = m.head_dim;
  ds->has_z = m.qkv[0].zeros != nullptr;
  DArgs& a = ds->a;
  const int L = m.layers, H = m.hidden, D = m.head_dim;
  a.layers = L;
  a.H = H;
  a.heads = m.heads;
  a.kvh = m.kv_heads;
  a.D = D;
  a.F = m.ffn;
  a.vocab = m.lm.N;
  a.nct = sms;
  a.grp = m.heads / m.kv_heads;
  a.nspl = std::max(1, sms / m.kv_heads);
  a.gs = m.group_size;
  a.gs_shift = (m.group_size & (m.group_size - 1)) == 0 ? __builtin_ctz((unsigned)m.group_size) : -1;
  a.has_z = ds->has_z ? 1 : 0;
  a.rope_base = m.rope_theta;
  a.eps = m.rms_eps;
  a.qscale = (1.0f / sqrtf((float)D)) * 1.4426950408889634f;
  a.g[0] = plan_gemv(m.qkv[0].K, m.qkv[0].N, sms, true);
  a.g[1] = plan_gemv(m.o[0].K, m.o[0].N, sms, true);
  a.g[2] = plan_gemv(m.gu[0].K, m.gu[0].N, sms, false);
  a.g[3] = plan_gemv(m.down[0].K, m.down[0].N, sms, true);
  a.g[4] = plan_gemv(m.lm.K, m.lm.N, sms, false);
  if (a.g[0].N != (m.heads + 2 * m.kv_heads) * D || a.g[1].N != H || a.g[2].N != 2 * m.ffn || a.g[3].N != H ||
      a.g[1].K != m.heads * D || a.g[3].K != m.ffn || a.g[0].K != H || a.g[2].K != H || a.g[4].K != H ||
      a.g[1].units > sms) {
    decode_step_destroy(ds);
    set_error("decode step kernel: projection shapes do not match the model");
    return SG_ERR_INVALID;
  }
  // ---- shared-memory layout
  int x_slots = 0;
  for (int k = 0; k < 5; ++k) {
    const Gemv& g = a.g[k];
    x_slots = std::max(x_slots, g.P == 1 ? g.cpt : (g.cpt + g.P - 1) / g.P + 1);
  }
  a.x_slots = x_slots;
  const int lm_units = (a.g[4].units + sms - 1) / sms;
  const size_t attn_bytes = std::max((size_t)kAW * 2 * kKG * (D + 8) * 2, (size_t)kAW * 16 * (D + 2) * 4);
  const size_t red_bytes = (size_t)kCW * 128 * 4;
  const size_t a_bytes = align_up(std::max(attn_bytes, red_bytes), 128);
  const size_t q_bytes = align_up((size_t)(a.grp + 2) * D * 4, 128);
  const size_t lm_bytes = align_up((size_t)lm_units * 128 * 4, 128);
  const size_t x_bytes = align_up((size_t)x_slots * kXSlotBytes, 128);
  // xf: the normed row (H fp16), the o phase's merged attention (its k range, fp32)
  // or the down phase's SwiGLU values (its k range, fp16)
  const int o_range = (a.g[1].cpt + a.g[1].P - 1) / a.g[1].P + 1;
  const int d_range = (a.g[3].cpt + a.g[3].P - 1) / a.g[3].P + 1;
  const size_t xf_bytes =
      align_up(std::max({(size_t)H * 2, (size_t)o_range * 64 * 4, (size_t)d_range * 64 * 2}), 128);
  // misc: the o phase's per-head split weights and (max, sum) pairs, or the greedy pick's scratch
  const int o_heads = o_range * 64 / D + 2;
  const size_t misc_bytes =
      align_up(std::max({(size_t)o_heads * (3 * a.nspl + 1) * 4, (size_t)(64 + 3 * sms) * 4, (size_t)64 * 4}), 128);
  const size_t fixed = a_bytes + q_bytes + lm_bytes + x_bytes + xf_bytes + misc_bytes;
  int max_optin = 0;
  SG_CUDA_TRY(cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  const size_t budget = (size_t)max_optin - 1024 /* alignment */ - 1024 /* static */;
  const size_t per_slot = kWBytes + kSZBytes + 16;
  if (fixed + 8 * per_slot > budget || lm_units > kMaxLmUnits) {
    decode_step_destroy(ds);
    set_error("decode step kernel: the model's staging does not fit in shared memory");
    return SG_ERR_UNSUPPORTED;
  }
  a.ns = (int)std::min<size_t>(64, (budget - fixed) / per_slot);
  size_t off = 0;
  off += (size_t)a.ns * kWBytes;
  a.off_sz = (int)off;
  off += (size_t)a.ns * kSZBytes;
  a.off_bars = (int)off;
  off = align_up(off + (size_t)a.ns * 16, 128);
  a.off_x = (int)off;
  off += x_bytes;
  a.off_xf = (int)off;
  off += xf_bytes;
  a.off_misc = (int)off;
  off += misc_bytes;
  a.off_a = (int)off;
  off += a_bytes;
  a.off_q = (int)off;
  off += q_bytes;
  a.off_lm = (int)off;
  off += lm_bytes;
  ds->smem = off + 1024;
  // ---- device memory: tensor maps, pointer tables, scratch
  const int nmaps = (L * kKinds + 1) * 3;
  const int Pq = a.g[0].P, Po = a.g[1].P, Pd = a.g[3].P;
  size_t mo = 0;
  auto take = [&](size_t bytes) {
    const size_t at = mo;
    mo = align_up(mo + bytes, 256);
    return at;
  };
  const size_t o_maps = take((size_t)nmaps * sizeof(CUtensorMap));
  const size_t o_ptrs = take((size_t)L * 4 * sizeof(void*));
  const size_t o_pages = take((size_t)L * sizeof(SgKvPages));
  const size_t o_pq = take((size_t)Pq * a.g[0].N * 4);
  const size_t o_po = take((size_t)Po * H * 4);
  const size_t o_gu = take((size_t)2 * m.ffn * 2);
  const size_t o_pd = take((size_t)Pd * H * 4);
  const size_t o_pa = take((size_t)m.kv_heads * a.nspl * a.grp * (D + 2) * 4);
  const size_t o_r0 = take((size_t)H * 2);
  const size_t o_r1 = take((size_t)H * 2);
  const size_t o_ap = take((size_t)sms * 3 * 4);
  const size_t o_sync = take(64);
  ds->mem_bytes = mo;
  if (cudaMalloc(&ds->mem, mo) != cudaSuccess) {
    cudaGetLastError();
    decode_step_destroy(ds);
    set_error("decode step kernel: out of device memory (%zu bytes)", mo);
    return SG_ERR_OOM;
  }
  std::vector<CUtensorMap> maps(nmaps);
  auto make = [&](const DsLinear& lin, CUtensorMap* tm) -> SgStatus {
    const int KP = (lin.K + 1) / 2, G = (lin.K + m.group_size - 1) / m.group_size;
    const uint64_t wd[2] = {(uint64_t)lin.N, (uint64_t)KP};
    const uint64_t ws[1] = {(uint64_t)lin.N};
    const uint32_t wb[2] = {128, (uint32_t)kRows};
    SgStatus st = make_tensor_map(&tm[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(lin.qw), wd, ws, wb,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SG_OK) return st;
    const uint64_t sd[2] = {(uint64_t)lin.N, (uint64_t)G};
    const uint64_t ss[1] = {(uint64_t)lin.N * 2};
    const uint32_t sb[2] = {128, 2};
    st = make_tensor_map(&tm[1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(lin.scales), sd, ss, sb,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != SG_OK) return st;
    if (lin.zeros) {
      const uint64_t zs[1] = {(uint64_t)lin.N};
      st = make_tensor_map(&tm[2], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(lin.zeros), sd, zs, sb,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
      tm[2] = tm[1];  // never read
    }
    return st;
  };
  SgStatus st = SG_OK;
  for (int l = 0; l < L && st == SG_OK; ++l) {
    const DsLinear* lins[4] = {&m.qkv[l], &m.o[l], &m.gu[l], &m.down[l]};
    for (int k = 0; k < kKinds && st == SG_OK; ++k) st = make(*lins[k], &maps[((size_t)l * kKinds + k) * 3]);
  }
  if (st == SG_OK) st = make(m.lm, &maps[(size_t)L * kKinds * 3]);
  if (st != SG_OK) {
    decode_step_destroy(ds);
    return st;
  }
  std::vector<const void*> ptrs((size_t)L * 4);
  for (int l = 0; l < L; ++l) {
    ptrs[l] = m.in_norm[l];
    ptrs[L + l] = m.post_norm[l];
    ptrs[2 * L + l] = m.k_cache[l];
    ptrs[3 * L + l] = m.v_cache[l];
  }
  if (cudaMemset(ds->mem, 0, mo) != cudaSuccess ||
      cudaMemcpy(ds->mem + o_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice) !=
          cudaSuccess ||
      cudaMemcpy(ds->mem + o_ptrs, ptrs.data(), ptrs.size() * sizeof(void*), cudaMemcpyHostToDevice) != cudaSuccess ||
      (!m.pages.empty() && cudaMemcpy(ds->mem + o_pages, m.pages.data(), (size_t)L * sizeof(SgKvPages),
                                      cudaMemcpyHostToDevice) != cudaSuccess)) {
    cudaGetLastError();
    decode_step_destroy(ds);
    set_error("decode step kernel: setting up its tables failed");
    return SG_ERR_RUNTIME;
  }
  char* base = ds->mem;
  a.maps = reinterpret_cast<const CUtensorMap*>(base + o_maps);
  const void* const* pt = reinterpret_cast<const void* const*>(base + o_ptrs);
  a.in_norm = reinterpret_cast<const __half* const*>(pt);
  a.post_norm = reinterpret_cast<const __half* const*>(pt + L);
  void* const* ptm = reinterpret_cast<void* const*>(base + o_ptrs);
  a.kc = reinterpret_cast<__half* const*>(ptm + 2 * L);
  a.vc = reinterpret_cast<__half* const*>(ptm + 3 * L);
  a.kv_hs = m.kv_head_stride;
  a.pages = m.pages.empty() ? nullptr : reinterpret_cast<const SgKvPages*>(base + o_pages);
  a.embed = static_cast<const __half*>(m.embed);
  a.vocab_rows = m.vocab_rows;
  a.final_norm = static_cast<const __half*>(m.final_norm);
  a.part_qkv = reinterpret_cast<float*>(base + o_pq);
  a.part_o = reinterpret_cast<float*>(base + o_po);
  a.gu = reinterpret_cast<__half*>(base + o_gu);
  a.part_down = reinterpret_cast<float*>(base + o_pd);
  a.part_attn = reinterpret_cast<float*>(base + o_pa);
  a.r0 = reinterpret_cast<__half*>(base + o_r0);
  a.r1 = reinterpret_cast<__half*>(base + o_r1);
  a.argp = reinterpret_cast<float*>(base + o_ap);
  a.sync = reinterpret_cast<unsigned*>(base + o_sync);
  st = device_error_word(&a.err);
  if (st != SG_OK) {
    decode_step_destroy(ds);
    return st;
  }
  void* kfn = pick_kernel(D, ds->has_z);
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ds->smem) != cudaSuccess) {
    cudaGetLastError();
    decode_step_destroy(ds);
    set_error("decode step kernel: %zu bytes of shared memory refused", ds->smem);
    return SG_ERR_UNSUPPORTED;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kThreads, ds->smem) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    decode_step_destroy(ds);
    set_error("decode step kernel: no SM can hold one block");
    return SG_ERR_UNSUPPORTED;
  }
  *out = ds;
  return SG_OK;
}

SgStatus decode_step_run(DecodeStep* ds, const int32_t* pos, int32_t* next, float* logprob, float* logits,
                         cudaStream_t st) {
  SG_CHECK_ARG(ds && pos && next && logprob && logits, "decode step kernel: null argument");
  DArgs a = ds->a;
  a.trace = ds->trace;
  a.pos = pos;
  a.next = next;
  a.logprob = logprob;
  a.logits = logits;
  SG_CUDA_TRY(cudaMemsetAsync(a.sync, 0, 16, st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nct);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = ds->smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (ds->D == 64)
    e = ds->has_z ? cudaLaunchKernelEx(&cfg, decode_step_kernel<64, true>, a)
                  : cudaLaunchKernelEx(&cfg, decode_step_kernel<64, false>, a);
  else
    e = ds->has_z ? cudaLaunchKernelEx(&cfg, decode_step_kernel<128, true>, a)
                  : cudaLaunchKernelEx(&cfg, decode_step_kernel<128, false>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("decode step kernel: launch failed: %s", cudaGetErrorString(e));
    return SG_ERR_RUNTIME;
  }
  return SG_OK;
}

}  // namespace sg
