// Device-side INT4 packer and unpacker for the reference weight layout
// (compiler/kernels/cpu/matmul_neon.h:127-136):
//   B u8 [ceil(K/2), N] (low nibble = even k), scales f16 [ceil(K/gs), N],
//   zeros i8 [ceil(K/gs), N] in [-8, 7].
//
// Asymmetric convention: python/armcc/calibration.py:37-50 applied per
// (group, column), in double precision as Python computes it:
//   scale = (max - min) / 15 ; zp = clamp(round_half_even(-8 - min/scale), -8, 7)
//   (scale = 1, zp = 0 when max == min, the dataclass defaults)
// Symmetric: scale = absmax / 7, no zero points.
// Stored scale s16 = fp16(float(scale)); q = clamp(rint(w / s16) + zp, -8, 7)
// in fp32 with IEEE division; nibble = q + 8.  Every step is correctly
// rounded, so the bytes equal the CPU packer's bit for bit.
#include "sg_common.cuh"

namespace {

// One thread per column: walks the groups of its column in k order, so odd
// group sizes (a byte shared by two groups) need no cross-thread merging.
__global__ void quantize_int4_kernel(const float* __restrict__ W, int K, int N, int gs, int symmetric,
                                     uint8_t* __restrict__ B, __half* __restrict__ scales,
                                     int8_t* __restrict__ zeros) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const int G = (K + gs - 1) / gs;
  uint8_t pending = 0;  // low nibble of the current byte, for odd k
  for (int g = 0; g < G; ++g) {
    const int k0 = g * gs, k1 = min(K, k0 + gs);
    float mn = W[(int64_t)k0 * N + n], mx = mn, amax = 0.f;
    for (int k = k0; k < k1; ++k) {
      const float v = W[(int64_t)k * N + n];
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
      amax = fmaxf(amax, fabsf(v));
    }
    double sd = 1.0;
    int zp = 0;
    if (symmetric) {
      if (amax > 0.f) sd = __ddiv_rn((double)amax, 7.0);
    } else {
      const double range = __dsub_rn((double)mx, (double)mn);
      if (range > 0.0) {
        sd = __ddiv_rn(range, 15.0);
        zp = (int)rint(__dsub_rn(-8.0, __ddiv_rn((double)mn, sd)));
        zp = max(-8, min(7, zp));
      }
    }
    const __half s16 = __float2half_rn(__double2float_rn(sd));
    const float s = __half2float(s16);
    scales[(int64_t)g * N + n] = s16;
    if (zeros) zeros[(int64_t)g * N + n] = (int8_t)zp;
    for (int k = k0; k < k1; ++k) {
      const float r = (s > 0.f) ? rintf(__fdiv_rn(W[(int64_t)k * N + n], s)) : 0.f;
      float qf = __fadd_rn(r, (float)zp);
      qf = fmaxf(-8.f, fminf(7.f, qf));
      const uint8_t nib = (uint8_t)((int)qf + 8) & 0x0F;
      if ((k & 1) == 0) {
        pending = nib;
        if (k + 1 == K) B[(int64_t)(k / 2) * N + n] = pending;
      } else {
        B[(int64_t)(k / 2) * N + n] = (uint8_t)(pending | (nib << 4));
      }
    }
  }
}

__global__ void dequantize_int4_kernel(const uint8_t* __restrict__ B, const __half* __restrict__ scales,
                                       const int8_t* __restrict__ zeros, int K, int N, int gs,
                                       float* __restrict__ W) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)K * N) return;
  const int k = (int)(idx / N), n = (int)(idx % N);
  const int group = (k & ~1) / gs;  // the pair's even k selects the group (:131)
  const uint8_t packed = B[(int64_t)(k / 2) * N + n];
  const int w = (int)((k & 1) ? (packed >> 4) : (packed & 0x0F)) - 8;
  const float scale = __half2float(scales[(int64_t)group * N + n]);
  const int zero = zeros ? (int)zeros[(int64_t)group * N + n] : 0;
  W[idx] = __fmul_rn(scale, (float)(w - zero));
}

}  // namespace

extern "C" {

SgStatus sg_quantize_int4_grouped(const float* W, int32_t K, int32_t N, int32_t group_size,
                                  int32_t symmetric, uint8_t* B, uint16_t* scales, int8_t* zeros,
                                  void* stream) {
  SG_CHECK_ARG(K >= 0 && N >= 0, "sg_quantize_int4_grouped: negative size");
  if (K == 0 || N == 0) return SG_OK;
  SG_CHECK_ARG(W && B && scales, "sg_quantize_int4_grouped: W, B and scales must be non-NULL");
  SG_CHECK_ARG(symmetric || zeros, "sg_quantize_int4_grouped: asymmetric packing needs zeros");
  int dev;
  SgStatus st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  const int gs = group_size > 0 ? group_size : 128;
  quantize_int4_kernel<<<(N + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      W, K, N, gs, symmetric, B, reinterpret_cast<__half*>(scales), symmetric ? nullptr : zeros);
  return sg::check_launch("quantize_int4_kernel");
}

SgStatus sg_dequantize_int4_grouped(const uint8_t* B, const uint16_t* scales, const int8_t* zeros,
                                    int32_t K, int32_t N, int32_t group_size, float* W, void* stream) {
  SG_CHECK_ARG(K >= 0 && N >= 0, "sg_dequantize_int4_grouped: negative size");
  if (K == 0 || N == 0) return SG_OK;
  SG_CHECK_ARG(W && B && scales, "sg_dequantize_int4_grouped: W, B and scales must be non-NULL");
  int dev;
  SgStatus st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  const int gs = group_size > 0 ? group_size : 128;
  const int64_t total = (int64_t)K * N;
  dequantize_int4_kernel<<<(unsigned)((total + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      B, reinterpret_cast<const __half*>(scales), zeros, K, N, gs, W);
  return sg::check_launch("dequantize_int4_kernel");
}

}  // extern "C"
