// INT8 per-channel GEMV for one float activation row on the int8 tensor pipe
// (sm_100a): C[n] = scales[n] * sum_k x[k] * W[k, n], the float-activation
// form of sg_matmul_int8_channel (the GLSL gemm_int8 shader's layout,
// compiler/kernels/gpu/vulkan_shaders.h:53-82 / opencl_kernels.h:36-52, with
// float activations).  Used for M == 1 when a cluster split fills the GPU;
// other shapes keep dense_gemv.cu.
//
// Memory side (HBM-bound): the structure of the INT4 GEMV (w4_gemv_mma.cu):
//   * work unit = a chunk of 32 k rows x one tile of 1, 2 or 4 128-column
//     strips; 16 warps per block = strips x phases, warp (strip, phase) takes
//     every phases-th chunk of the block's k range for its strip through its
//     own 2-stage TMA ring of 128-byte x 32-row boxes (128-byte swizzle);
//   * tiles split over thread-block clusters of k <= 8 blocks that reduce
//     through distributed shared memory (each rank pushes the columns another
//     rank owns with st.async; the owner adds the ranks in order).
// Math side:
//   * x is staged once per block as 24-bit fixed point with one power-of-two
//     scale per 32 k (x = 2^(E-21) x_q, |x_q| <= 2^22, x_q = 65536 hi + 256 mid
//     + lo in signed bytes; one word [hi, mid, lo, 0] per k);
//   * the weights are signed bytes, so a 32-bit word of a weight row (4
//     columns at one k) is directly an A fragment register of mma.sync
//     m16n8k32 s8 x s8: A row m is the word of 4 columns, A k-slot 4 s + e its
//     column e at the step's s-th k row.  The 8 k rows of a step are taken in
//     the order 0, 2, 4, 6, 1, 3, 5, 7 and lane (g, t) owns words 4g .. 4g+3,
//     so its A registers are two 16-byte loads (k rows 2t and 2t+1), and with
//     the 128-byte swizzle the 8 lanes of a quarter warp hit 8 distinct 16-byte
//     bank groups;
//   * B column 2e + v carries byte v (hi, mid) of x at column slot e, zero
//     elsewhere; a second MMA on the same A registers takes lo.  Every D entry
//     is one column's exact int32 partial, every lane owns 4 columns, and per
//     chunk acc += 2^(E-21) (256 (256 D_hi + D_mid) + D_lo).
// No zero points and no group scales: per chunk about 11 instructions per
// 1024 weights in the MMA loop against the INT4 kernel's 18 per 2048 nibbles,
// i.e. ~40 % fewer per byte streamed.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <string_view>

#include "sm100.cuh"

namespace {

constexpr int kRows = 32;             // k rows per chunk: one 24-bit scale group
constexpr int kWBytes = 128 * kRows;  // 4096
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 2;
constexpr int kRingBytes = kWarps * kStages * kWBytes;
constexpr int kStaticSmemReserve = 2048;

struct W8Args {
  const void* A;
  const float* scales;
  void* C;
  int K, N;
  int a_dt, c_dt;
  int n_tiles, cpt, ksplit, x_slots;
  int static_w;
  int* err;
};

__device__ __forceinline__ float load_act(const void* A, int dt, int i) {
  switch (dt) {
    case SG_DT_F32: return static_cast<const float*>(A)[i];
    case SG_DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(A)[i]);
    default: return __half2float(static_cast<const __half*>(A)[i]);
  }
}

__device__ __forceinline__ void store_out(void* C, int dt, int64_t i, float v) {
  switch (dt) {
    case SG_DT_F32: sgd::store_from_float<SG_DT_F32>(C, i, v); break;
    case SG_DT_BF16: sgd::store_from_float<SG_DT_BF16>(C, i, v); break;
    default: sgd::store_from_float<SG_DT_F16>(C, i, v); break;
  }
}

// mma.sync m16n8k32, A and B signed 8-bit, exact int32 accumulation.
__device__ __forceinline__ void mma_s8s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared memory after the ring: the staged x ([slot][32] words, then [slot]
// scales), the stage barriers, the cluster's [rank][column] partials, the
// per-phase partials.
inline size_t w8_tail_bytes(int strips, int x_slots, int ksplit) {
  const size_t cols = (size_t)strips * 128;
  return (size_t)x_slots * kRows * 4 + (size_t)x_slots * 4 + 16 + (size_t)kWarps * kStages * 8 +
         (size_t)ksplit * cols * 4 + (size_t)(kWarps / strips) * cols * 4;
}

// grid (ksplit, n_tiles), clusters of ksplit blocks per tile of STRIPS x 128 columns
template <int STRIPS>
__global__ void __launch_bounds__(kThreads, 1)
    w8_gemv_mma_kernel(const __grid_constant__ CUtensorMap tmW, W8Args a) {
  constexpr int kPhases = kWarps / STRIPS, kTC = STRIPS * 128;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = sgd::align_smem_1024(smem_raw);
  uint32_t* xst = reinterpret_cast<uint32_t*>(smem + kRingBytes);  // [slot][32]: [hi, mid, lo, 0]
  float* xsc = reinterpret_cast<float*>(xst + (size_t)a.x_slots * kRows);  // [slot]: 2^(E-21)
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      reinterpret_cast<uint8_t*>(xsc) + (((size_t)a.x_slots * 4 + 15) & ~(size_t)15));
  float* csum = reinterpret_cast<float*>(bars + kWarps * kStages);  // [rank][kTC]
  float* red = csum + (size_t)a.ksplit * kTC;                        // [phase][kTC]
  __shared__ int s_abort;
  __shared__ int s_aborts[16];
  __shared__ __align__(8) uint64_t s_rbar;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int strip = warp % STRIPS, phase = warp / STRIPS;
  const int tile = blockIdx.y, rank = blockIdx.x;
  const int cs = (a.cpt * rank) / a.ksplit, ce = (a.cpt * (rank + 1)) / a.ksplit;
  const int per = ((kTC + a.ksplit - 1) / a.ksplit + 3) & ~3;
  const int own_lo = min(kTC, rank * per);
  const int own = min(kTC, own_lo + per) - own_lo;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kWarps * kStages; ++i) sgd::mbar_init(&bars[i], 1);
    if (a.ksplit > 1) {
      sgd::mbar_init(&s_rbar, 1);
      sgd::mbar_arrive_expect_tx(&s_rbar, (uint32_t)((a.ksplit - 1) * (own * 4 + 4)));
    }
    sgd::fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  sgd::pdl_launch_dependents();

  uint64_t* my_bars = bars + warp * kStages;
  const int c_first = cs + phase;
  const int n_my = c_first < ce ? (ce - c_first + kPhases - 1) / kPhases : 0;
  const int x0 = tile * kTC + strip * 128;
  auto issue = [&](int i) {
    const int c = c_first + i * kPhases;
    const int s = i % kStages;
    uint64_t* bar = &my_bars[s];
    sgd::mbar_arrive_expect_tx(bar, kWBytes);
    sgd::tma_load_2d(smem + (size_t)(warp * kStages + s) * kWBytes, &tmW, x0, c * kRows, bar);
  };
  // Weights that no earlier kernel writes stream before the dependency wait.
  if (a.static_w && lane == 0)
    for (int i = 0; i < min(kStages, n_my); ++i) issue(i);
  sgd::pdl_wait();
  if (!a.static_w && lane == 0)
    for (int i = 0; i < min(kStages, n_my); ++i) issue(i);

  // ---- stage x over k rows [cs * 32, ce * 32): one warp = one 32-k group
  const int nrows = (ce - cs) * kRows;
  for (int idx = threadIdx.x; idx < nrows; idx += kThreads) {
    const int k = cs * kRows + idx;
    const float x = k < a.K ? load_act(a.A, a.a_dt, k) : 0.f;
    float m = fabsf(x);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int E = max((__float_as_int(m) >> 23) - 127, -100);
    const float inv = __int_as_float((127 + 21 - E) << 23);  // 2^(21 - E), exact scaling
    const float sxv = __int_as_float((127 - 21 + E) << 23);  // 2^(E - 21)
    const int q = __float2int_rn(x * inv);
    const int lo = ((q + 128) & 255) - 128;
    const int r = (q - lo) >> 8;  // 256 hi + mid, exact
    const int mid = ((r + 128) & 255) - 128;
    const int hi = (r - mid) >> 8;
    xst[idx] = (uint32_t)(hi & 255) | ((uint32_t)(mid & 255) << 8) | ((uint32_t)(lo & 255) << 16);
    if (lane == 0) xsc[idx >> 5] = sxv;
  }
  __syncthreads();

  // ---- lane roles (see the header): A registers = words 4g .. 4g+3 of k rows
  //      2t and 2t+1 of each 8-row step; B provider: column n = g, i.e. slot
  //      e = g >> 1 and byte v = g & 1 (hi / mid), lo or zero for the second MMA
  const int g = lane >> 2, t = lane & 3;
  const int be = g >> 1, bv = g & 1;
  const uint32_t sel_d = (0x4444u & ~(0xFu << (4 * be))) | ((uint32_t)bv << (4 * be));
  const uint32_t sel_l = (0x4444u & ~(0xFu << (4 * be))) | ((uint32_t)(bv ? 4 : 2) << (4 * be));
  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // columns 16 g + t + 4 i of the warp's strip
  int ok = 1;
  for (int i = 0; i < n_my; ++i) {
    const int c = c_first + i * kPhases;
    const int s = i % kStages;
    const bool waited = sgd::mbar_wait(&my_bars[s], (i / kStages) & 1, a.err);
    if (!__all_sync(0xffffffffu, waited)) {
      ok = 0;
      break;
    }
    const uint8_t* wst = smem + (size_t)(warp * kStages + s) * kWBytes;
    const uint32_t* xr = xst + (size_t)(c - cs) * kRows;
    int d[2][4], e[2][4];
#pragma unroll
    for (int jm = 0; jm < 2; ++jm)
#pragma unroll
      for (int q = 0; q < 4; ++q) d[jm][q] = e[jm][q] = 0;
#pragma unroll
    for (int st = 0; st < 4; ++st) {
      const int r0 = 8 * st + 2 * t, r1 = r0 + 1;
      const uint4 X = *reinterpret_cast<const uint4*>(wst + r0 * 128 + ((g ^ (r0 & 7)) << 4));
      const uint4 Y = *reinterpret_cast<const uint4*>(wst + r1 * 128 + ((g ^ (r1 & 7)) << 4));
      const uint2 xw = *reinterpret_cast<const uint2*>(xr + r0);
      const uint32_t b0 = __byte_perm(xw.x, 0u, sel_d), b1 = __byte_perm(xw.y, 0u, sel_d);
      const uint32_t c0 = __byte_perm(xw.x, 0u, sel_l), c1 = __byte_perm(xw.y, 0u, sel_l);
      mma_s8s8_16832(d[0], X.x, X.y, Y.x, Y.y, b0, b1);
      mma_s8s8_16832(d[1], X.z, X.w, Y.z, Y.w, b0, b1);
      mma_s8s8_16832(e[0], X.x, X.y, Y.x, Y.y, c0, c1);
      mma_s8s8_16832(e[1], X.z, X.w, Y.z, Y.w, c0, c1);
    }
    const float sx = xsc[c - cs];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int jm = q >> 1, fr = (q & 1) * 2;  // q: (jm, row g / g + 8) -> columns 16 g + t + 4 q
      const int hm = d[jm][fr] * 256 + d[jm][fr + 1];
      acc[q] = fmaf(sx, fmaf(256.f, (float)hm, (float)e[jm][fr]), acc[q]);
    }
    __syncwarp();
    if (lane == 0 && i + kStages < n_my) issue(i + kStages);
  }
  if (!ok) s_abort = 1;
  {
    float* r0 = red + (size_t)phase * kTC + strip * 128 + 16 * g + t;
#pragma unroll
    for (int q = 0; q < 4; ++q) r0[4 * q] = acc[q];
  }
  __syncthreads();

  // ---- cluster reduction: each rank adds its phases and pushes the columns
  //      another rank owns into that rank's [rank][column] buffer; the owner
  //      adds the ranks in order and stores scales[n] * sum
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
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
  __syncthreads();
  int aborted = s_abort || !ok_wait;
  for (int r = 0; r < a.ksplit; ++r)
    if (r != rank) aborted |= s_aborts[r];
  if (aborted) return;
  for (int cc = own_lo + threadIdx.x; cc < own_lo + own; cc += kThreads) {
    float v = 0.f;
    for (int r = 0; r < a.ksplit; ++r) v += csum[r * kTC + cc];
    const int col = tile * kTC + cc;
    if (col < a.N) store_out(a.C, a.c_dt, col, v * a.scales[col]);
  }
}

struct W8Plan {
  bool ok = false;
  int strips = 4, ksplit = 1, n_tiles = 0, cpt = 0, x_slots = 0;
  size_t smem = 0;
};

// Clusters of k 16-warp blocks resident at once (shape-only, cached per k).
int w8_active_clusters(int k) {
  static std::mutex mu;
  static int cache[9] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (k < 1 || k > 8) return 0;
  if (cache[k] != 0) return cache[k];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(k, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 200 * 1024;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = k;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  auto kfn = w8_gemv_mma_kernel<4>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = -1;
  }
  cache[k] = n;
  return n;
}

std::atomic<int> g_w8_mma{1};  // 0: keep the dp4a kernel for one-row float activations

W8Plan make_w8_plan(const SgMatMulParams* p, int sms) {
  W8Plan pl;
  const int adt = p->a_dtype;
  if (!g_w8_mma.load() || p->M != 1 || p->K <= 0 || p->N % 16 != 0) return pl;
  if (adt != SG_DT_F32 && adt != SG_DT_F16 && adt != SG_DT_BF16) return pl;
  if (!sg::aligned16(p->B)) return pl;
  pl.cpt = (p->K + kRows - 1) / kRows;
  long long best = 0;
  for (int strips : {4, 2, 1}) {
    const int n_tiles = (p->N + strips * 128 - 1) / (strips * 128);
    if (n_tiles > sms) continue;
    for (int k = std::min({8, pl.cpt, sms / n_tiles}); k >= 1; --k) {
      if (w8_active_clusters(k) < n_tiles) continue;
      const long long score = (long long)n_tiles * k;
      if (score > best) {
        best = score;
        pl.strips = strips;
        pl.ksplit = k;
        pl.n_tiles = n_tiles;
      }
      break;
    }
  }
  if (best == 0 || 2 * best < sms) return pl;  // less than half the SMs: the dp4a kernel
  pl.x_slots = (pl.cpt + pl.ksplit - 1) / pl.ksplit;
  pl.smem = 1024 + kRingBytes + w8_tail_bytes(pl.strips, pl.x_slots, pl.ksplit);
  if (pl.smem > 227 * 1024 - kStaticSmemReserve) return pl;
  pl.ok = true;
  return pl;
}

}  // namespace

namespace sg {

// Runs the tensor-core INT8 GEMV (one float activation row) if it applies; *handled says so.
SgStatus w8_gemv_mma_run(const SgMatMulParams* p, cudaStream_t cs, int sms, int* err_word, bool* handled) {
  *handled = false;
  const W8Plan pl = make_w8_plan(p, sms);
  if (!pl.ok) return SG_OK;
  CUtensorMap tw;
  const uint64_t dims[2] = {(uint64_t)p->N, (uint64_t)p->K};
  const uint64_t strides[1] = {(uint64_t)p->N};
  const uint32_t box[2] = {128, (uint32_t)kRows};
  SgStatus st = make_tensor_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(p->B), dims, strides, box,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != SG_OK) return st;
  W8Args a{};
  a.A = p->A;
  a.scales = static_cast<const float*>(p->scales_B);
  a.C = p->C;
  a.K = p->K;
  a.N = p->N;
  a.a_dt = p->a_dtype;
  a.c_dt = p->c_dtype == SG_DT_DEFAULT ? SG_DT_F32 : p->c_dtype;
  a.n_tiles = pl.n_tiles;
  a.cpt = pl.cpt;
  a.ksplit = pl.ksplit;
  a.x_slots = pl.x_slots;
  a.static_w = (p->flags & SG_MM_STATIC_WEIGHTS) ? 1 : 0;
  a.err = err_word;
  using KFn = void (*)(CUtensorMap, W8Args);
  const KFn kfn = pl.strips == 4 ? w8_gemv_mma_kernel<4> : pl.strips == 2 ? w8_gemv_mma_kernel<2>
                                                                           : w8_gemv_mma_kernel<1>;
  const int ki = pl.strips == 4 ? 2 : pl.strips == 2 ? 1 : 0;
  int dev = 0;
  st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  {
    static std::mutex mu;
    static size_t done[64][3] = {};
    std::lock_guard<std::mutex> lk(mu);
    size_t scratch = 0;
    size_t& d = dev >= 0 && dev < 64 ? done[dev][ki] : scratch;
    if (d < pl.smem) {
      if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) != cudaSuccess) {
        cudaGetLastError();
        set_error("w8_gemv_mma: cudaFuncSetAttribute(%zu) failed", pl.smem);
        return SG_ERR_RUNTIME;
      }
      d = pl.smem;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.ksplit, pl.n_tiles);
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
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, tw, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("w8_gemv_mma_kernel launch failed: %s", cudaGetErrorString(e));
    return SG_ERR_RUNTIME;
  }
  *handled = true;
  return SG_OK;
}

bool w8_gemv_mma_tuning(std::string_view key, int value) {
  if (key == "w8_gemv_mma.enable") {
    g_w8_mma.store(value);
    return true;
  }
  return false;
}

}  // namespace sg
