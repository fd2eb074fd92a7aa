// The row statistics of the decoder's RMSNorm (rmsnorm_fp16_neon,
// compiler/kernels/cpu/matmul_neon.h:154-190: y = x / sqrt(mean(x^2) + eps) * w),
// shared by the RMSNorm kernel (blockops.cu) and the INT4 GEMV that fuses the
// norm into its activation staging (w4_gemv_mma.cu, SG_MM_A_RMSNORM), so that
// both form the same sum of squares bit for bit: threads 0..kNormThreads-1 each
// take 16-byte vectors tid, tid + kNormThreads, ... of the row and add their
// squares in element order, then one block-wide butterfly sum; any further
// threads of the block add exact zeros, which leaves every partial unchanged.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace sgn {

constexpr int kNormThreads = 256;
constexpr int kNormVecPerThread = 4;  // rows up to 8 * 256 * 4 = 8192 values
constexpr int kNormMaxN = 8 * kNormThreads * kNormVecPerThread;

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int k = 0; k < 8; ++k) f[k] = (float)h[k];
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  T* h = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int k = 0; k < 8; ++k) h[k] = (T)f[k];
  return u;
}

// Sum over the block (every thread gets it); red: 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by a previous reduction
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// Adds the squares of one 8-value vector of h (already rounded to T) to a
// thread's partial, in element order.
__device__ __forceinline__ float sumsq8(const float (&h)[8], float ss) {
#pragma unroll
  for (int e = 0; e < 8; ++e) ss += h[e] * h[e];
  return ss;
}

// 1 / sqrt(mean(h^2) + eps) of a 16-bit row h of n values (n % 8 == 0,
// n <= kNormMaxN, 16-byte aligned); called by every thread of the block.
template <typename T>
__device__ __forceinline__ float row_rms_inv(const T* __restrict__ row, int n, float eps, float* red) {
  float ss = 0.f;
  if (threadIdx.x < kNormThreads) {
    const int nv = n / 8;
#pragma unroll
    for (int k = 0; k < kNormVecPerThread; ++k) {
      const int v = threadIdx.x + k * kNormThreads;
      if (v < nv) {
        float h[8];
        unpack8<T>(reinterpret_cast<const uint4*>(row)[v], h);
        ss = sumsq8(h, ss);
      }
    }
  }
  ss = block_sum(ss, red);
  return 1.0f / sqrtf(ss / (float)n + eps);
}

}  // namespace sgn
