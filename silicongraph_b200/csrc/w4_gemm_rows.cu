// INT4 group-quantised GEMM for a few activation rows (2..16: batched decode)
// on the tensor cores (sm_100a).  Same contract and weight layout as
// w4_gemv.cu (compiler/kernels/cpu/matmul_neon.h:113-143); used when
// 2 <= M <= 16, the group size is a power of two >= 32 and N % 16 == 0
// (measured faster than both the tcgen05 GEMM and the GEMV kernels on every
// decoder shape there).
//
//   * Tile = 128 output columns.  Few tiles: a cluster of ksplit blocks shares
//     a tile's K range, and each rank adds the ranks' partials of 1/ksplit of
//     the tile's outputs in rank order from their shared memory
//     (deterministic, no scratch).  Many tiles: persistent blocks (one or two
//     per SM) stage the activations once and take every blocks-th tile, the
//     weight ring running on across tiles.
//   * One producer warp streams chunks of 64 k-pair rows (128 k) x 128
//     columns of packed weights (128-byte swizzled TMA box) plus the chunk's
//     scale and zero-point rows through a ring of 4 to 16 stages.  Two sets of
//     8 consumer warps take alternate chunks; in a set each warp owns 16
//     columns, and the sets' partials are added in set order at the end.
//   * The nibble unpacking is written as explicit prmt + lop3 (one three-input
//     logic op with both constants in registers); the same expression in C
//     compiled to two logic ops per weight pair.
//   * A warp's 16 columns are the 16 rows of the mma.sync m16n8k16 A operand
//     (A row g = column 2g, row g + 8 = column 2g + 1); a lane's byte of two
//     k gives both halves of one A register: (byte & 0x0F) | 0x6400 is
//     1024 + q_lo and (byte & 0xF0) | 0x5400 is 64 + q_hi (the fp16 ulp at 64
//     is 1/16), so subtracting (1032 + zero, 72 + zero) is exact and one
//     multiply by the scale rounds once: the fp16 weight scale * (q - 8 - zero).
//   * The activation rows, staged once per block in fp16, are the B columns
//     (8 rows per n-tile, fetched with ldmatrix); D accumulates in fp32 over
//     the block's whole range.
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string_view>

#include "sm100.cuh"

namespace {

constexpr int kRowsPerChunk = 64;  // k-pair rows per chunk (128 k)
constexpr int kTileCols = 128;
constexpr int kColWarps = 8;                         // warps per chunk: 16 columns each
constexpr int kSets = 2;                             // consumer sets, taking every kSets-th chunk (3 measured slower)
constexpr int kConsumerWarps = kSets * kColWarps;
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // + the producer warp
constexpr int kMinStages = 4;  // ring depth: 4, 8 or 16 chunks (the most that fit shared memory)
constexpr int kMaxStages = 16;
constexpr int kMaxSmem = 227 * 1024 - 2048;  // opt-in limit minus this kernel's static shared memory
constexpr int kWBytes = 128 * kRowsPerChunk;      // 8192
constexpr int kSBytes = 128 * 4 * 2;              // up to 4 scale rows (group 32) x 128 fp16
constexpr int kZBytes = 128 * 4;                  // up to 4 zero rows x 128 int8
constexpr int kSZBytes = kSBytes + kZBytes;       // 1536
constexpr int kStageBytes = kWBytes + kSZBytes;   // weights [stage][8192] (1024-aligned for the swizzle), then [stage][1536]

struct RArgs {
  const void* A;
  const __half* bias;
  void* C;
  int M, K, N, lda, ldc, gs_shift;
  int a_dt, c_dt;
  float scale_A;
  int n_tiles, cpt, ksplit, x_slots;
  int static_w;
  int stage_shift;  // log2 of the ring depth
  int psleep;       // producer backs off with nanosleep while the ring is full
  int x_vec;  // A 16-byte aligned, lda and K multiples of 8: rows staged 8 values at a time
  int swiglu; // A rows are [gate | up]: x = SwiGLU(A[m][k], A[m][K + k]) (SG_MM_A_SWIGLU)
  int* err;
};

__device__ __forceinline__ float load_act(const void* A, int dt, int64_t i) {
  switch (dt) {
    case SG_DT_F32: return static_cast<const float*>(A)[i];
    case SG_DT_F16: return __half2float(static_cast<const __half*>(A)[i]);
    case SG_DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(A)[i]);
    default: return (float)static_cast<const int8_t*>(A)[i];
  }
}

// 8 consecutive activations (fp16) of element i; i % 8 == 0 and A 16-byte aligned
__device__ __forceinline__ uint4 load_act8(const void* A, int dt, int64_t i) {
  uint4 o;
  __half2* oh = reinterpret_cast<__half2*>(&o);
  switch (dt) {
    case SG_DT_F16: return *reinterpret_cast<const uint4*>(static_cast<const __half*>(A) + i);
    case SG_DT_F32: {
      const float4 u = reinterpret_cast<const float4*>(static_cast<const float*>(A) + i)[0];
      const float4 v = reinterpret_cast<const float4*>(static_cast<const float*>(A) + i)[1];
      oh[0] = __floats2half2_rn(u.x, u.y);
      oh[1] = __floats2half2_rn(u.z, u.w);
      oh[2] = __floats2half2_rn(v.x, v.y);
      oh[3] = __floats2half2_rn(v.z, v.w);
      return o;
    }
    case SG_DT_BF16: {
      const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(A) + i);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b[j]);
        oh[j] = __floats2half2_rn(f.x, f.y);
      }
      return o;
    }
    default: {
      const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const int8_t*>(A) + i);
      const int8_t* b = reinterpret_cast<const int8_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) oh[j] = __floats2half2_rn((float)b[2 * j], (float)b[2 * j + 1]);
      return o;
    }
  }
}

// A constant the compiler keeps in a register (opaque to constant folding).
__device__ __forceinline__ uint32_t opaque_u32(uint32_t v) {
  uint32_t r;
  asm volatile("mov.b32 %0, %1;" : "=r"(r) : "r"(v));
  return r;
}

// SwiGLU of gate element i and up element i + K, rounded to A's type, as fp32.
__device__ __forceinline__ float load_swiglu(const void* A, int dt, int64_t i, int K) {
  if (dt == SG_DT_BF16) {
    const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(A);
    return __bfloat162float(sgd::swiglu_value<__nv_bfloat16>(__bfloat162float(p[i]), __bfloat162float(p[i + K])));
  }
  const __half* p = static_cast<const __half*>(A);
  return __half2float(sgd::swiglu_value<__half>(__half2float(p[i]), __half2float(p[i + K])));
}

// 8 SwiGLU activations (fp16) from gate elements i.. and up elements i + K..; 16-byte aligned
__device__ __forceinline__ uint4 load_swiglu8(const void* A, int dt, int64_t i, int K) {
  uint4 o;
  __half* oh = reinterpret_cast<__half*>(&o);
  if (dt == SG_DT_BF16) {
    const uint4 g = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(A) + i);
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(A) + i + K);
    const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&g);
    const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      oh[j] = __float2half_rn(__bfloat162float(
          sgd::swiglu_value<__nv_bfloat16>(__bfloat162float(gb[j]), __bfloat162float(ub[j]))));
  } else {
    const uint4 g = *reinterpret_cast<const uint4*>(static_cast<const __half*>(A) + i);
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __half*>(A) + i + K);
    const __half* gh = reinterpret_cast<const __half*>(&g);
    const __half* uh = reinterpret_cast<const __half*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) oh[j] = sgd::swiglu_value<__half>(__half2float(gh[j]), __half2float(uh[j]));
  }
  return o;
}

// (1024 + q_lo, 64 + q_hi) of the byte at `sel` (0x4040: byte 0, 0x4141: byte 1)
// of w: one byte permute and one three-input logic op, (x & mask) | magic with
// mask = 0x00F0000F and magic = 0x54006400 in registers.
template <uint32_t SEL>
__device__ __forceinline__ __half2 nibble_pair(uint32_t w, uint32_t mask, uint32_t magic) {
  uint32_t v;
  asm("{\n .reg .b32 t;\n prmt.b32 t, %1, 0, %2;\n lop3.b32 %0, t, %3, %4, 0xEA;\n}"
      : "=r"(v)
      : "r"(w), "n"(SEL), "r"(mask), "r"(magic));
  return *reinterpret_cast<const __half2*>(&v);
}

// fp16 pair (1152 + z, 1152 + z) of the signed zero byte z at `sel` of zz:
// ((z, 0, z, 0) ^ flip) | magic with flip = 0x00800080, magic = 0x64006400.
template <uint32_t SEL>
__device__ __forceinline__ uint32_t zero_pair(uint32_t zz, uint32_t flip, uint32_t magic) {
  uint32_t v;
  asm("{\n .reg .b32 t;\n prmt.b32 t, %1, 0, %2;\n lop3.b32 %0, t, %3, %4, 0xBE;\n}"
      : "=r"(v)
      : "r"(zz), "n"(SEL), "r"(flip), "r"(magic));
  return v;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }

// GPC: groups per chunk (128 k): 4 for group 32, 2 for group 64, 1 for larger groups.
template <bool HAS_Z, int MT, int GPC>
__global__ void __launch_bounds__(kThreads, 1)
    w4_rows_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                   const __grid_constant__ CUtensorMap tmZ, RArgs a) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = sgd::align_smem_1024(smem_raw);
  const int nst = 1 << a.stage_shift;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + nst * kStageBytes);
  uint64_t* empty = full + nst;
  const int XP = a.x_slots * 128 + 8;  // staged k per row, padded (bank spread)
  __half* xs = reinterpret_cast<__half*>(empty + nst);  // [MT][XP]
  float* red = reinterpret_cast<float*>(xs + MT * XP);      // [kSets][MT][128] this block's partials
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sp = blockIdx.x;
  const bool split = a.ksplit > 1;  // then gridDim.y == n_tiles: one tile per cluster
  const int cr0 = (a.cpt * sp) / a.ksplit;                // first chunk (of every tile) of this block
  const int nch = (a.cpt * (sp + 1)) / a.ksplit - cr0;    // chunks per tile
  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i) {
      sgd::mbar_init(&full[i], 1);
      sgd::mbar_init(&empty[i], kColWarps);
    }
    sgd::fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  if (split) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  sgd::pdl_launch_dependents();

  if (warp == kConsumerWarps) {
    // ---- producer: weights that no earlier kernel writes stream before the dependency wait
    if (!a.static_w) sgd::pdl_wait();
    if (lane == 0) {
      constexpr uint32_t tx = kWBytes + GPC * (256 + (HAS_Z ? 128 : 0));
      int it = 0;  // chunks issued, over all tiles of this block
      bool stop = false;
      for (int tile = blockIdx.y; tile < a.n_tiles && !stop; tile += gridDim.y) {
        for (int i = 0; i < nch; ++i, ++it) {
          const int s = it & (nst - 1);
          // the ring is usually full: a sleeping poll keeps this warp's issue slots for the consumers
          if (it >= nst && !(a.psleep ? sgd::mbar_wait_sleep(&empty[s], ((it >> a.stage_shift) - 1) & 1, a.err)
                                      : sgd::mbar_wait(&empty[s], ((it >> a.stage_shift) - 1) & 1, a.err))) {
            s_abort = 1;
            stop = true;
            break;
          }
          const int row0 = (cr0 + i) * kRowsPerChunk;
          const int gA = (2 * row0) >> a.gs_shift;
          uint8_t* wst = smem + s * kWBytes;
          uint8_t* szst = smem + nst * kWBytes + s * kSZBytes;
          sgd::mbar_arrive_expect_tx(&full[s], tx);
          sgd::tma_load_2d(wst, &tmW, tile * kTileCols, row0, &full[s]);
          sgd::tma_load_2d(szst, &tmS, tile * kTileCols, gA, &full[s]);
          if (HAS_Z) sgd::tma_load_2d(szst + kSBytes, &tmZ, tile * kTileCols, gA, &full[s]);
        }
      }
    }
  } else {
    // ---- consumers: stage the activation rows once (fp16, zero past M and K), then the chunks
    sgd::pdl_wait();
    const int span = nch * 128;
    if (a.x_vec) {
      // 8 values per thread and access, 4 accesses in flight per thread
      constexpr int kU = 4, kT = kConsumerWarps * 32;
      const int nv = span / 8, total = MT * nv;
      for (int base = threadIdx.x; base < total; base += kU * kT) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int idx = base + u * kT;
          const int m = idx / nv, k = cr0 * 128 + 8 * (idx - m * nv);
          v[u] = make_uint4(0u, 0u, 0u, 0u);
          if (idx < total && m < a.M && k < a.K)
            v[u] = a.swiglu ? load_swiglu8(a.A, a.a_dt, (int64_t)m * a.lda + k, a.K)
                            : load_act8(a.A, a.a_dt, (int64_t)m * a.lda + k);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int idx = base + u * kT;
          if (idx < total) {
            const int m = idx / nv;
            *reinterpret_cast<uint4*>(xs + m * XP + 8 * (idx - m * nv)) = v[u];
          }
        }
      }
    } else {
      for (int idx = threadIdx.x; idx < MT * span; idx += kConsumerWarps * 32) {
        const int m = idx / span, kk = idx - m * span;
        const int k = cr0 * 128 + kk;
        const int64_t e = (int64_t)m * a.lda + k;
        const float v = (m < a.M && k < a.K) ? (a.swiglu ? load_swiglu(a.A, a.a_dt, e, a.K) : load_act(a.A, a.a_dt, e))
                                             : 0.f;
        xs[m * XP + kk] = __float2half_rn(v);
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
    const int cw = warp % kColWarps, cp = warp / kColWarps;  // column group; chunk parity of this set
    const int g = lane >> 2, t = lane & 3;
    const int c0 = 16 * cw + 2 * g;  // A row g: column c0; row g + 8: column c0 + 1
    // ldmatrix row of this lane: MT 16: matrices (n-tile j / 2, k half j % 2) of one 16-k step;
    // MT 8: matrices (k half j % 2) of steps 2p + j / 2
    const int lj = lane >> 3, lr = lane & 7;
    const __half* xrow = MT == 16 ? xs + (8 * (lj >> 1) + lr) * XP + 8 * (lj & 1) : xs + lr * XP + 8 * lj;
    // this lane's weight bytes in a stage: k-pair rows 8 st + t (+ 4), 16-byte column group cw (swizzled)
    const int wl0 = t * 128 + ((cw ^ t) << 4) + 2 * g, wl1 = (t + 4) * 128 + ((cw ^ (t + 4)) << 4) + 2 * g;
    float* myred = red + cp * MT * kTileCols;
    const uint32_t kMaskW = opaque_u32(0x00F0000Fu), kMagicW = opaque_u32(0x54006400u);
    const uint32_t kFlipZ = opaque_u32(0x00800080u), kMagicZ = opaque_u32(0x64006400u);
    bool dead = false;  // a wait of this warp ran out: skip the rest, keep to the barriers
    int it0 = 0;
    for (int tile = blockIdx.y; tile < a.n_tiles; tile += gridDim.y) {
      float acc[MT / 8][4];
#pragma unroll
      for (int n = 0; n < MT / 8; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[n][q] = 0.f;
      for (int i = ((cp - it0) % kSets + kSets) % kSets; i < nch && !dead; i += kSets) {
        const int it = it0 + i;
        const int s = it & (nst - 1);
        const bool ok = sgd::mbar_wait(&full[s], (it >> a.stage_shift) & 1, a.err);
        if (!__all_sync(0xffffffffu, ok)) {
          s_abort = 1;
          dead = true;
          break;
        }
        const uint8_t* W = smem + s * kWBytes;
        const uint8_t* SZ = smem + nst * kWBytes + s * kSZBytes;
        const __half* xi = xrow + i * 128;
#pragma unroll
        for (int gi = 0; gi < GPC; ++gi) {
          // scale and zero of columns c0, c0 + 1 for group gi of the chunk
          const uint32_t s2 = *reinterpret_cast<const uint32_t*>(SZ + (gi * 128 + c0) * 2);
          const uint32_t sd0 = __byte_perm(s2, 0u, 0x1010u), sd1 = __byte_perm(s2, 0u, 0x3232u);
          const __half2 sc0 = *reinterpret_cast<const __half2*>(&sd0), sc1 = *reinterpret_cast<const __half2*>(&sd1);
          __half2 off0, off1;
          if (HAS_Z) {
            // zero byte z -> fp16 pair (1152 + z, 1152 + z) by bits, minus (120, 1080): (1032 + z, 72 + z), exact
            const uint32_t zz = *reinterpret_cast<const uint16_t*>(SZ + kSBytes + gi * 128 + c0);
            const __half2 bias = __halves2half2(__ushort_as_half(0x5780), __ushort_as_half(0x6438));  // 120, 1080
            const uint32_t m0 = zero_pair<0x4040u>(zz, kFlipZ, kMagicZ);
            const uint32_t m1 = zero_pair<0x4141u>(zz, kFlipZ, kMagicZ);
            off0 = __hsub2(*reinterpret_cast<const __half2*>(&m0), bias);
            off1 = __hsub2(*reinterpret_cast<const __half2*>(&m1), bias);
          } else {
            off0 = off1 = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x5480));  // 1032, 72
          }
          constexpr int kSteps = 8 / GPC;  // 16-k steps in the group's part of the chunk
#pragma unroll
          for (int j = 0; j < kSteps; j += (MT == 16 ? 1 : 2)) {
            const int st0 = gi * kSteps + j;
            uint32_t bx[2][2][2];  // [step][n-tile][k half]
            {
              uint32_t r0, r1, r2, r3;
              sgd::ldmatrix_x4(r0, r1, r2, r3, xi + 16 * st0);
              if (MT == 16) {
                bx[0][0][0] = r0;
                bx[0][0][1] = r1;
                bx[0][1][0] = r2;
                bx[0][1][1] = r3;
              } else {
                bx[0][0][0] = r0;
                bx[0][0][1] = r1;
                bx[1][0][0] = r2;
                bx[1][0][1] = r3;
              }
            }
#pragma unroll
            for (int u = 0; u < (MT == 16 ? 1 : 2); ++u) {
              const int st = st0 + u;
              const uint32_t w0 = *reinterpret_cast<const uint16_t*>(W + st * 1024 + wl0);
              const uint32_t w1 = *reinterpret_cast<const uint16_t*>(W + st * 1024 + wl1);
              const uint32_t a0 = h2_bits(__hmul2(__hsub2(nibble_pair<0x4040u>(w0, kMaskW, kMagicW), off0), sc0));
              const uint32_t a1 = h2_bits(__hmul2(__hsub2(nibble_pair<0x4141u>(w0, kMaskW, kMagicW), off1), sc1));
              const uint32_t a2 = h2_bits(__hmul2(__hsub2(nibble_pair<0x4040u>(w1, kMaskW, kMagicW), off0), sc0));
              const uint32_t a3 = h2_bits(__hmul2(__hsub2(nibble_pair<0x4141u>(w1, kMaskW, kMagicW), off1), sc1));
#pragma unroll
              for (int n = 0; n < MT / 8; ++n)
                sgd::mma_f16_16816(acc[n], a0, a1, a2, a3, bx[MT == 16 ? 0 : u][n][0], bx[MT == 16 ? 0 : u][n][1]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) sgd::mbar_arrive(&empty[s]);
      }
      it0 += nch;
      // D: [n][0] row 8n + 2t, column c0; [1] row 8n + 2t + 1, c0; [2] row 8n + 2t, c0 + 1; [3] row 8n + 2t + 1, c0 + 1
#pragma unroll
      for (int n = 0; n < MT / 8; ++n) {
        const int m = 8 * n + 2 * t;
        myred[m * kTileCols + c0] = acc[n][0];
        myred[(m + 1) * kTileCols + c0] = acc[n][1];
        myred[m * kTileCols + c0 + 1] = acc[n][2];
        myred[(m + 1) * kTileCols + c0 + 1] = acc[n][3];
      }
      if (!split) {
        // the sets' partials of this tile, added in set order, go out coalesced
        asm volatile("bar.sync 2, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        if (!s_abort) {
          for (int idx = threadIdx.x; idx < a.M * kTileCols; idx += kConsumerWarps * 32) {
            const int m = idx / kTileCols, cc = idx - m * kTileCols;
            const int col = tile * kTileCols + cc;
            if (col >= a.N) continue;
            float v = red[idx];
#pragma unroll
            for (int q = 1; q < kSets; ++q) v += red[q * MT * kTileCols + idx];
            if (a.a_dt == SG_DT_I8) v *= a.scale_A;
            if (a.bias) v += __half2float(a.bias[col]);
            const int64_t o = (int64_t)m * a.ldc + col;
            switch (a.c_dt) {
              case SG_DT_F32: sgd::store_from_float<SG_DT_F32>(a.C, o, v); break;
              case SG_DT_BF16: sgd::store_from_float<SG_DT_BF16>(a.C, o, v); break;
              default: sgd::store_from_float<SG_DT_F16>(a.C, o, v); break;
            }
          }
        }
        asm volatile("bar.sync 2, %0;" ::"n"(kConsumerWarps * 32) : "memory");  // red is free for the next tile
      }
    }
  }
  if (!split) return;
  __syncthreads();
  // ---- split K: rank r adds the ranks' partials (in rank order) of its 1/ksplit of the tile's outputs
  cg::cluster_group cluster = cg::this_cluster();
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  cluster.sync();
  int aborted = 0;
  for (int r = 0; r < a.ksplit; ++r) aborted |= *cluster.map_shared_rank(&s_abort, r);
  if (!aborted) {
    const float* parts[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) parts[q] = cluster.map_shared_rank(red, q < a.ksplit ? q : 0);
    const int tile = blockIdx.y;
    const int tot = a.M * kTileCols, per = (tot + a.ksplit - 1) / a.ksplit;
    const int hi = min(tot, (sp + 1) * per);
    for (int idx = sp * per + threadIdx.x; idx < hi; idx += kThreads) {
      const int m = idx / kTileCols, cc = idx - m * kTileCols;
      const int col = tile * kTileCols + cc;
      if (col >= a.N) continue;
      float pv[8][kSets];
#pragma unroll
      for (int q = 0; q < 8; ++q)
#pragma unroll
        for (int c = 0; c < kSets; ++c) pv[q][c] = q < a.ksplit ? parts[q][c * MT * kTileCols + idx] : 0.f;
      float v = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q < a.ksplit) {
          float t = pv[q][0];
#pragma unroll
          for (int c = 1; c < kSets; ++c) t += pv[q][c];
          v += t;
        }
      if (a.a_dt == SG_DT_I8) v *= a.scale_A;
      if (a.bias) v += __half2float(a.bias[col]);
      const int64_t o = (int64_t)m * a.ldc + col;
      switch (a.c_dt) {
        case SG_DT_F32: sgd::store_from_float<SG_DT_F32>(a.C, o, v); break;
        case SG_DT_BF16: sgd::store_from_float<SG_DT_BF16>(a.C, o, v); break;
        default: sgd::store_from_float<SG_DT_F16>(a.C, o, v); break;
      }
    }
  }
  cluster.sync();  // peers keep their shared memory until every rank has read it
}

struct RPlan {
  bool ok = false;
  int mt = 8, n_tiles = 0, cpt = 0, ksplit = 1, x_slots = 0;
  int blocks = 0;  // ksplit == 1: persistent blocks, each taking every blocks-th tile
  int stages = kMinStages;
  size_t smem = 0;
};

size_t rows_smem(int mt, int x_slots, int stages) {
  return 1024 + (size_t)stages * kStageBytes + 2 * stages * 8 + (size_t)mt * (x_slots * 128 + 8) * 2 +
         (size_t)kSets * mt * kTileCols * 4;
}

// Blocks of this kernel (at the given shared memory, no cluster) resident per SM.
// This cache and the next are process-wide, not per device: they assume every
// GPU of the process is the same model (true of one B200 node).
int rows_blocks_per_sm(size_t smem) {
  static std::mutex mu;
  static int cache[8] = {};  // [smem bucket of 32 KB]
  const int bucket = (int)std::min<size_t>(7, smem / (32 * 1024));
  std::lock_guard<std::mutex> lk(mu);
  if (cache[bucket] != 0) return cache[bucket];
  int n = 0;
  auto kfn = w4_rows_kernel<true, 16, 4>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kfn, kThreads, (size_t)(bucket + 1) * 32 * 1024) !=
          cudaSuccess) {
    cudaGetLastError();
    n = -1;
  }
  cache[bucket] = n;
  return n;
}

// Clusters of k blocks of this kernel (at the given shared memory) resident at once.
int rows_active_clusters(int k, size_t smem) {
  static std::mutex mu;
  static int cache[9][8] = {};  // [k][smem bucket of 32 KB]
  const int bucket = (int)std::min<size_t>(7, smem / (32 * 1024));
  std::lock_guard<std::mutex> lk(mu);
  if (k < 1 || k > 8) return 0;
  if (cache[k][bucket] != 0) return cache[k][bucket];
  const int bytes = (int)((size_t)(bucket + 1) * 32 * 1024);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(k, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = bytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = k;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  auto kfn = w4_rows_kernel<true, 16, 4>;
  // the attribute only ever grows (a launch may already rely on a larger value)
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) != cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = -1;
  }
  cache[k][bucket] = n;
  return n;
}

std::atomic<int> g_rows_enable{1};
std::atomic<int> g_rows_max_tiles{1 << 30};  // widest output (in 128-column tiles) taken
std::atomic<int> g_rows_stages{0};  // 0: deepest ring that fits
std::atomic<int> g_rows_psleep{1};

RPlan make_rplan(const SgMatMulParams* p, int sms) {
  RPlan pl;
  const int gs = p->group_size > 0 ? p->group_size : 128;
  if (p->M < 2 || p->M > 16 || p->K <= 0 || p->N <= 0 || (p->N % 16) != 0 || gs < 32 || (gs & (gs - 1)) != 0)
    return pl;
  if ((p->N + kTileCols - 1) / kTileCols > g_rows_max_tiles.load()) return pl;
  if (!sg::aligned16(p->B) || !sg::aligned16(p->scales_B) || (p->zeros_B && !sg::aligned16(p->zeros_B))) return pl;
  pl.mt = p->M <= 8 ? 8 : 16;
  pl.n_tiles = (p->N + kTileCols - 1) / kTileCols;
  pl.cpt = ((p->K + 1) / 2 + kRowsPerChunk - 1) / kRowsPerChunk;
  // the largest split that keeps every cluster resident in one wave; many tiles: one block each
  int ks = 1;
  for (int k = std::min({8, pl.cpt, std::max(1, (2 * sms) / pl.n_tiles)}); k >= 2; --k) {
    const size_t smem = rows_smem(pl.mt, (pl.cpt + k - 1) / k, kMinStages);
    if (smem <= (size_t)kMaxSmem && rows_active_clusters(k, smem) >= pl.n_tiles) {
      ks = k;
      break;
    }
  }
  pl.ksplit = ks;
  pl.x_slots = (pl.cpt + ks - 1) / ks;
  // the deepest ring that fits (more weight bytes in flight per SM)
  // (no deeper than the chunks one block streams)
  const int want = g_rows_stages.load();
  const long chunks = (long)pl.x_slots * (ks > 1 ? 1 : (pl.n_tiles + sms - 1) / sms);
  pl.stages = kMinStages;
  for (int st = kMinStages * 2; st <= kMaxStages; st *= 2)
    if ((want == 0 ? st / 2 < chunks : st <= want) && rows_smem(pl.mt, pl.x_slots, st) <= (size_t)kMaxSmem)
      pl.stages = st;
  while (ks > 1 && pl.stages > kMinStages && rows_active_clusters(ks, rows_smem(pl.mt, pl.x_slots, pl.stages)) < pl.n_tiles)
    pl.stages /= 2;
  pl.smem = rows_smem(pl.mt, pl.x_slots, pl.stages);
  if (pl.smem > (size_t)kMaxSmem) return pl;
  if (ks > 1) {
    pl.blocks = pl.n_tiles;
  } else {
    // persistent blocks stage the activations once; one per SM unless two per
    // SM finish the tiles in fewer rounds (two blocks share an SM's issue slots)
    const int bps = rows_blocks_per_sm(pl.smem);
    if (bps < 1) return pl;
    const int r1 = (pl.n_tiles + sms - 1) / sms;
    const int r2 = bps >= 2 ? 2 * ((pl.n_tiles + 2 * sms - 1) / (2 * sms)) : 1 << 30;
    pl.blocks = std::min(pl.n_tiles, r2 <= r1 ? 2 * sms : sms);
  }
  pl.ok = true;
  return pl;
}

}  // namespace

namespace sg {

bool w4_rows_tuning(std::string_view key, int value) {
  if (key == "w4_rows.enable") {
    g_rows_enable.store(value);
    return true;
  }
  if (key == "w4_rows.producer_sleep") {
    g_rows_psleep.store(value);
    return true;
  }
  if (key == "w4_rows.stages") {
    g_rows_stages.store(value);
    return true;
  }
  if (key == "w4_rows.max_tiles") {
    g_rows_max_tiles.store(std::max(1, value));
    return true;
  }
  return false;
}

SgStatus w4_rows_run(const SgMatMulParams* p, cudaStream_t cs, int sms, int* err_word, bool* handled) {
  *handled = false;
  if (!g_rows_enable.load()) return SG_OK;
  const RPlan pl = make_rplan(p, sms);
  if (!pl.ok) return SG_OK;
  *handled = true;
  const int gs = p->group_size > 0 ? p->group_size : 128;
  const int KP = (p->K + 1) / 2;
  const int G = (p->K + gs - 1) / gs;
  const int gpc = gs == 32 ? 4 : gs == 64 ? 2 : 1;  // groups per 128-k chunk
  CUtensorMap tw, ts, tz;
  SgStatus st;
  {
    const uint64_t dims[2] = {(uint64_t)p->N, (uint64_t)KP};
    const uint64_t strides[1] = {(uint64_t)p->N};
    const uint32_t box[2] = {128, (uint32_t)kRowsPerChunk};  // 64 k-pair rows
    st = make_tensor_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(p->B), dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != SG_OK) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)p->N, (uint64_t)G};
    const uint64_t sstr[1] = {(uint64_t)p->N * 2};
    const uint32_t box[2] = {128, (uint32_t)gpc};  // the chunk's group rows
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
  RArgs a{};
  a.A = p->A;
  a.bias = static_cast<const __half*>(p->bias);
  a.C = p->C;
  a.M = p->M;
  a.K = p->K;
  a.N = p->N;
  a.swiglu = (p->flags & SG_MM_A_SWIGLU) ? 1 : 0;
  a.lda = p->lda > 0 ? p->lda : (a.swiglu ? 2 * p->K : p->K);
  a.ldc = p->ldc > 0 ? p->ldc : p->N;
  a.gs_shift = __builtin_ctz((unsigned)gs);
  a.a_dt = p->a_dtype == SG_DT_DEFAULT ? SG_DT_I8 : p->a_dtype;
  a.c_dt = p->c_dtype == SG_DT_DEFAULT ? SG_DT_F16 : p->c_dtype;
  a.scale_A = p->scale_A;
  a.n_tiles = pl.n_tiles;
  a.cpt = pl.cpt;
  a.ksplit = pl.ksplit;
  a.x_slots = pl.x_slots;
  a.static_w = (p->flags & SG_MM_STATIC_WEIGHTS) ? 1 : 0;
  a.stage_shift = __builtin_ctz((unsigned)pl.stages);
  a.psleep = g_rows_psleep.load() ? 1 : 0;
  a.x_vec = sg::aligned16(p->A) && a.lda % 8 == 0 && p->K % 8 == 0;
  a.err = err_word;
  using KFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, RArgs);
  static const KFn kfns[2][2][3] = {
      {{w4_rows_kernel<false, 8, 4>, w4_rows_kernel<false, 8, 2>, w4_rows_kernel<false, 8, 1>},
       {w4_rows_kernel<false, 16, 4>, w4_rows_kernel<false, 16, 2>, w4_rows_kernel<false, 16, 1>}},
      {{w4_rows_kernel<true, 8, 4>, w4_rows_kernel<true, 8, 2>, w4_rows_kernel<true, 8, 1>},
       {w4_rows_kernel<true, 16, 4>, w4_rows_kernel<true, 16, 2>, w4_rows_kernel<true, 16, 1>}}};
  const int zi = p->zeros_B ? 1 : 0, mi = pl.mt == 8 ? 0 : 1, gi = gpc == 4 ? 0 : gpc == 2 ? 1 : 2;
  const KFn kfn = kfns[zi][mi][gi];
  // every instantiation gets the largest shared-memory opt-in once per device
  // (the attribute belongs to the device's copy of the kernel); the occupancy
  // query above relies on the same value
  static std::atomic<uint64_t> attr_set[2][2][3] = {};
  int dev = 0;
  st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
  if (!(attr_set[zi][mi][gi].load() & bit)) {
    const cudaError_t ae = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (ae != cudaSuccess) {
      cudaGetLastError();
      set_error("w4_rows: cudaFuncSetAttribute(%d) failed: %s", kMaxSmem, cudaGetErrorString(ae));
      return SG_ERR_RUNTIME;
    }
    attr_set[zi][mi][gi].fetch_or(bit);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.ksplit, pl.blocks);
  cfg.blockDim = dim3(kThreads);
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
  cfg.numAttrs = pl.ksplit > 1 ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, tw, ts, tz, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("w4_rows_kernel launch failed: %s", cudaGetErrorString(e));
    return SG_ERR_RUNTIME;
  }
  return SG_OK;
}

}  // namespace sg
