// One-shot all-reduce of a small fp16 vector across the ranks of a
// tensor-parallel group over NVLink peer memory (the decode-time sum after the
// row-split projections: [tokens, hidden], a few to a few hundred KB).
//
// Every rank owns a region (cudaMalloc, mapped into the other ranks with CUDA
// IPC):  data [2 parities][world][max_n] fp16 | flags [world][kMaxBlocks] u32 |
// epoch u32.  Call k (epoch k, parity k & 1), block b of rank r:
//   1. stores its slice of the local partial into slot [parity][r] of every
//      rank's region (plain 16-byte peer stores), fences at system scope and
//      writes epoch into flag [r][b] of every rank;
//   2. waits (bounded) until flag [q][b] of its own region reaches epoch for
//      every rank q;
//   3. sums the slots of its slice in rank order (fp32, one rounding) into the
//      local vector, so every rank gets the same bits.
// Rank r can only start call k + 2 after every peer has raised its flags of
// call k + 1, which they do after finishing call k: two parities suffice.  A
// wait that runs out records an error in the device error word and leaves the
// vector unreduced (the host reports it); nothing spins forever.  The limit
// is 2 s, or what sg_set_tuning("tp_allreduce.wait_ms", ms) sets.
#include <atomic>
#include <string_view>

#include "sm100.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 32;
constexpr int kThreads = 512;
constexpr int kChunk = 8;  // fp16 per 16-byte vector
std::atomic<int> g_wait_ms{2000};  // bounded wait for the peers' flags

struct Peers {
  uint8_t* region[kMaxRanks];
};

__device__ __forceinline__ void st_flag(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_flag(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// residual != NULL: the sum is not written back to data; instead
// residual = round(residual + round(sum)) (the decoder's residual add, as
// sg_rmsnorm with a residual does it).
__global__ void __launch_bounds__(kThreads) tp_allreduce_kernel(__half* __restrict__ data, int n, int rank, int world,
                                                                Peers peers, int max_n, int* err, uint64_t wait_ns,
                                                                __half* __restrict__ residual) {
  sgd::pdl_wait();  // the partial comes from the previous kernel
  sgd::pdl_launch_dependents();
  uint8_t* mine = peers.region[rank];
  const size_t data_bytes = (size_t)2 * world * max_n * sizeof(__half);
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(mine + data_bytes);
  uint32_t* epoch_word = my_flags + world * kMaxBlocks;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(epoch_word) + 1;
  const int par = epoch & 1;
  // this block's slice, in 16-byte vectors
  const int nvec = n / kChunk;
  const int per = (nvec + gridDim.x - 1) / gridDim.x;
  const int v0 = blockIdx.x * per, v1 = min(nvec, v0 + per);
  const uint4* src = reinterpret_cast<const uint4*>(data);
  for (int q = 0; q < world; ++q) {
    uint4* dst = reinterpret_cast<uint4*>(peers.region[q] + ((size_t)par * world + rank) * max_n * sizeof(__half));
    for (int v = v0 + threadIdx.x; v < v1; v += kThreads) dst[v] = src[v];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) {
    uint32_t* f = reinterpret_cast<uint32_t*>(peers.region[threadIdx.x] + data_bytes);
    st_flag(f + rank * kMaxBlocks + blockIdx.x, epoch);
  }
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < world) {
    const uint32_t* f = my_flags + threadIdx.x * kMaxBlocks + blockIdx.x;
    if (ld_flag(f) < epoch) {
      const uint64_t t0 = sgd::global_timer_ns();
      for (;;) {
        if (ld_flag(f) >= epoch) break;
        if (sgd::global_timer_ns() - t0 > wait_ns) {
          sgd::record_error(err, sgd::kErrWaitTimeout);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (s_ok) {
    const uint4* slots = reinterpret_cast<const uint4*>(mine + (size_t)par * world * max_n * sizeof(__half));
    const int stride = max_n / kChunk;  // vectors per slot
    for (int v = v0 + threadIdx.x; v < v1; v += kThreads) {
      float acc[kChunk] = {};
      for (int q = 0; q < world; ++q) {
        const uint4 x = slots[(size_t)q * stride + v];
        const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          acc[2 * i] += f.x;
          acc[2 * i + 1] += f.y;
        }
      }
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) oh[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
      if (residual) {
        uint4 r = reinterpret_cast<const uint4*>(residual)[v];
        __half2* rh = reinterpret_cast<__half2*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 a = __half22float2(oh[i]), b = __half22float2(rh[i]);
          rh[i] = __floats2half2_rn(a.x + b.x, a.y + b.y);
        }
        reinterpret_cast<uint4*>(residual)[v] = r;
      } else {
        reinterpret_cast<uint4*>(data)[v] = o;
      }
    }
  }
  // the epoch advances once every block has taken it (all blocks read it before any flag of this call)
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(reinterpret_cast<unsigned*>(epoch_word + 1), 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    epoch_word[1] = 0u;
    __threadfence();
    *reinterpret_cast<volatile uint32_t*>(epoch_word) = epoch;
  }
}

}  // namespace

namespace sg {
bool tp_allreduce_tuning(std::string_view key, int value) {
  if (key == "tp_allreduce.wait_ms") {
    g_wait_ms.store(value <= 0 ? 2000 : std::min(value, 2000));
    return true;
  }
  return false;
}
}  // namespace sg

extern "C" {

size_t sg_tp_allreduce_region_bytes(int32_t world, int32_t max_n) {
  if (world < 1 || world > kMaxRanks || max_n < 0) return 0;
  const size_t n = sg::align_up((size_t)max_n, (size_t)kChunk);
  return sg::align_up((size_t)2 * world * n * sizeof(__half) + (size_t)world * kMaxBlocks * 4 + 8, 256);
}

static SgStatus allreduce_run(void* data, int32_t n, int32_t rank, int32_t world, void* const* regions,
                              int32_t max_n, void* residual, void* stream) {
  SG_CHECK_ARG(world >= 1 && world <= kMaxRanks, "sg_tp_allreduce_f16: world %d outside [1, %d]", world, kMaxRanks);
  SG_CHECK_ARG(rank >= 0 && rank < world, "sg_tp_allreduce_f16: rank %d outside the group", rank);
  SG_CHECK_ARG(n >= 0 && n <= max_n && max_n % kChunk == 0 && n % kChunk == 0,
               "sg_tp_allreduce_f16: n %d / max_n %d must be multiples of %d with n <= max_n", n, max_n, kChunk);
  SG_CHECK_ARG(data && regions && sg::aligned16(data), "sg_tp_allreduce_f16: data must be 16-byte aligned");
  if (n == 0) return SG_OK;
  Peers pe{};
  for (int q = 0; q < world; ++q) {
    SG_CHECK_ARG(regions[q] && sg::aligned16(regions[q]), "sg_tp_allreduce_f16: region %d is NULL or unaligned", q);
    pe.region[q] = static_cast<uint8_t*>(regions[q]);
  }
  int* err = nullptr;
  SgStatus st = sg::device_error_word(&err);
  if (st != SG_OK) return st;
  const int nvec = n / kChunk;
  const int blocks = std::max(1, std::min(kMaxBlocks, (nvec + 1023) / 1024));
  SG_CUDA_TRY(sgd::launch_pdl(tp_allreduce_kernel, dim3(blocks), dim3(kThreads), 0, static_cast<cudaStream_t>(stream),
                              static_cast<__half*>(data), (int)n, (int)rank, (int)world, pe, (int)max_n, err,
                              (uint64_t)std::max(1, g_wait_ms.load()) * 1000000ull, static_cast<__half*>(residual)));
  return SG_OK;
}

SgStatus sg_tp_allreduce_f16(void* data, int32_t n, int32_t rank, int32_t world, void* const* regions, int32_t max_n,
                             void* stream) {
  return allreduce_run(data, n, rank, world, regions, max_n, nullptr, stream);
}

SgStatus sg_tp_allreduce_f16_residual(void* data, int32_t n, int32_t rank, int32_t world, void* const* regions,
                                      int32_t max_n, void* residual, void* stream) {
  SG_CHECK_ARG(residual && sg::aligned16(residual), "sg_tp_allreduce_f16_residual: residual NULL or unaligned");
  return allreduce_run(data, n, rank, world, regions, max_n, residual, stream);
}

}  // extern "C"
