// Shared host/device helpers for the SiliconGraph-B200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "sg_kernels.h"

namespace sg {

// ------------------------------------------------------------------ errors
// Thread-local last-error message (sg_last_error()).
void set_error(const char* fmt, ...);
const char* last_error();

#define SG_CHECK_ARG(cond, ...)          \
  do {                                   \
    if (!(cond)) {                       \
      ::sg::set_error(__VA_ARGS__);      \
      return SG_ERR_INVALID;             \
    }                                    \
  } while (0)

#define SG_CUDA_TRY(expr)                                                               \
  do {                                                                                  \
    cudaError_t e_ = (expr);                                                            \
    if (e_ != cudaSuccess) {                                                            \
      ::sg::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                      __LINE__);                                                        \
      return SG_ERR_RUNTIME;                                                            \
    }                                                                                   \
  } while (0)

// After a launch: report configuration errors (bad grid, smem, ...).
SgStatus check_launch(const char* what);

// Current device ordinal, or error if no usable device.
SgStatus current_device(int* dev);

// Number of SMs of the current device (cached per device).
int sm_count(int dev);

// ---------------------------------------------------------------- workspace
// Library-owned scratch, one buffer per (device, stream, user), grown on
// demand and zero-filled when (re)allocated.  Each entry-point family has its
// own buffer, so ticket counters that a family keeps at zero between calls are
// never overwritten by another family's partial results.  Growth synchronises
// the stream, so the first call with a larger shape must not run under stream
// capture.
enum WorkspaceUser : int { kWsInt4Gemv = 0, kWsDenseGemv = 1, kWsAttention = 2, kWsPrefillGemm = 3, kWsArgmax = 4,
                           kWsUsers = 5 };
SgStatus library_workspace(void* stream, size_t bytes, void** out, int user);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Ticket counters (one per column tile) live in a fixed 4 KB prefix of a
// kernel's scratch (more only beyond 1024 tiles), so partial results of one
// call never land where another call of the same kernels expects zeros.
// Tensor-core prefill GEMM (gemm_tc.cu) for INT4-grouped or INT8-per-channel
// weights.  gemm_tc_scratch_bytes: *ok tells whether the problem qualifies;
// the result is the scratch it needs (0 when activations are used in place).
// minimal: the least scratch it runs with (no split of the last round of tiles).
size_t gemm_tc_scratch_bytes(const SgMatMulParams* p, bool int8_weights, bool* ok, bool minimal = false);
// Tensor-core INT8 GEMV for one float activation row (w8_gemv_mma.cu); *handled says whether it ran.
SgStatus w8_gemv_mma_run(const SgMatMulParams* p, cudaStream_t cs, int sms, int* err_word, bool* handled);
SgStatus gemm_tc_run(const SgMatMulParams* p, bool int8_weights, cudaStream_t cs, int sms, void* ws,
                     size_t ws_bytes, int* err_word, bool* handled);

// Tensor-core flash attention (attn_tc.cu): runs the problem when it
// qualifies (fp16 / bf16, head_dim 64 or 128, long enough), else *handled = false.
SgStatus attn_tc_run(const SgFlashAttentionParams* p, cudaStream_t cs, void* ws, size_t ws_bytes, bool ws_external,
                     bool* handled);
size_t attn_tc_scratch_bytes(const SgFlashAttentionParams* p);

inline size_t ticket_bytes(int n_tiles) {
  const size_t t = align_up((size_t)n_tiles * sizeof(unsigned), 256);
  return t < 4096 ? 4096 : t;
}

// ------------------------------------------------------------------ dtypes
inline int elem_size(int dt) {
  switch (dt) {
    case SG_DT_F32: return 4;
    case SG_DT_F16:
    case SG_DT_BF16: return 2;
    case SG_DT_I8: return 1;
    default: return 0;
  }
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace sg

// ------------------------------------------------------------ device helpers
namespace sgd {

template <int DT>
__device__ __forceinline__ float load_as_float(const void* p, int64_t i);
template <>
__device__ __forceinline__ float load_as_float<SG_DT_F32>(const void* p, int64_t i) {
  return static_cast<const float*>(p)[i];
}
template <>
__device__ __forceinline__ float load_as_float<SG_DT_F16>(const void* p, int64_t i) {
  return __half2float(static_cast<const __half*>(p)[i]);
}
template <>
__device__ __forceinline__ float load_as_float<SG_DT_BF16>(const void* p, int64_t i) {
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
template <>
__device__ __forceinline__ float load_as_float<SG_DT_I8>(const void* p, int64_t i) {
  return (float)static_cast<const int8_t*>(p)[i];
}

template <int DT>
__device__ __forceinline__ void store_from_float(void* p, int64_t i, float v);
template <>
__device__ __forceinline__ void store_from_float<SG_DT_F32>(void* p, int64_t i, float v) {
  static_cast<float*>(p)[i] = v;
}
template <>
__device__ __forceinline__ void store_from_float<SG_DT_F16>(void* p, int64_t i, float v) {
  static_cast<__half*>(p)[i] = __float2half_rn(v);
}
template <>
__device__ __forceinline__ void store_from_float<SG_DT_BF16>(void* p, int64_t i, float v) {
  static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// 128-bit streaming load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t d;
  // (a & mask) | orv  -> immLut = (0xF0 & 0xCC) | 0xAA = 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}

// Packed fp32x2 FMA (sm_100): d = a * b + c, lane-wise, round-to-nearest.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t ra, rb, rc, rd;
  ra = ((uint64_t)__float_as_uint(a.y) << 32) | __float_as_uint(a.x);
  rb = ((uint64_t)__float_as_uint(b.y) << 32) | __float_as_uint(b.x);
  rc = ((uint64_t)__float_as_uint(c.y) << 32) | __float_as_uint(c.x);
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
  return make_float2(__uint_as_float((uint32_t)rd), __uint_as_float((uint32_t)(rd >> 32)));
}

// Element i of a uint4 / fp16 / int8 lane of packed registers, for indices
// that are compile-time constants after unrolling (keeps values in registers).
__device__ __forceinline__ uint32_t u4_get(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
// fp16 number cc (0..15) of 16 packed halves held in (lo: 0..7, hi: 8..15).
__device__ __forceinline__ float half16_at(const uint4& lo, const uint4& hi, int cc) {
  const uint32_t w = u4_get(cc < 8 ? lo : hi, (cc & 7) >> 1);
  return __half2float(__ushort_as_half((unsigned short)(w >> ((cc & 1) * 16))));
}
// int8 number cc (0..15) of 16 packed bytes.
__device__ __forceinline__ int i8x16_at(const uint4& v, int cc) {
  const uint32_t w = u4_get(v, cc >> 2);
  return (int)(int8_t)(w >> ((cc & 3) * 8));
}

}  // namespace sgd
