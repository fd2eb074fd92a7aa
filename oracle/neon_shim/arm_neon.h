// x86 stand-in for <arm_neon.h>, used only to compile the reference's CPU
// kernel headers (compiler/kernels/cpu/matmul_neon.h, flash_attention.h) on
// an x86 host so that their `#ifdef __ARM_NEON` branches run as written.
//
// Why: on non-ARM builds matmul_int4_grouped_neon's `#else` branch is a no-op
// (matmul_neon.h:144-147); the only working INT4 loop is inside the NEON
// branch (matmul_neon.h:114-142).  Defining __ARM_NEON and supplying these
// definitions lets the unmodified reference source execute here.
//
// Semantics follow the Arm ACLE definitions of each intrinsic, lane by lane:
//   * vmlaq_f32 is the NEON non-fused multiply-accumulate (a + b*c, two
//     roundings); the recipe compiles with -ffp-contract=off to keep it so.
//   * vaddvq_f32 is FADDP-based: (v0 + v1) + (v2 + v3).
//   * f16 <-> f32 conversions are IEEE round-to-nearest-even (_Float16).
// Only the intrinsics the reference headers use are provided.
#pragma once
#include <stdint.h>
#include <string.h>

typedef float float32_t;
typedef _Float16 float16_t;
typedef float    float32x4_t __attribute__((vector_size(16)));
typedef _Float16 float16x4_t __attribute__((vector_size(8)));
typedef _Float16 float16x8_t __attribute__((vector_size(16)));

static inline float32x4_t vdupq_n_f32(float v) { float32x4_t r = {v, v, v, v}; return r; }

static inline float16x8_t vld1q_f16(const _Float16* p) { float16x8_t r; memcpy(&r, p, sizeof(r)); return r; }
static inline float16x4_t vld1_f16(const _Float16* p) { float16x4_t r; memcpy(&r, p, sizeof(r)); return r; }
static inline void vst1q_f16(_Float16* p, float16x8_t v) { memcpy(p, &v, sizeof(v)); }
static inline void vst1_f16(_Float16* p, float16x4_t v) { memcpy(p, &v, sizeof(v)); }

static inline float16x4_t vget_low_f16(float16x8_t v) { float16x4_t r = {v[0], v[1], v[2], v[3]}; return r; }
static inline float16x4_t vget_high_f16(float16x8_t v) { float16x4_t r = {v[4], v[5], v[6], v[7]}; return r; }
static inline float16x8_t vcombine_f16(float16x4_t lo, float16x4_t hi) {
  float16x8_t r = {lo[0], lo[1], lo[2], lo[3], hi[0], hi[1], hi[2], hi[3]};
  return r;
}

static inline float32x4_t vcvt_f32_f16(float16x4_t v) {
  float32x4_t r = {(float)v[0], (float)v[1], (float)v[2], (float)v[3]};
  return r;
}
static inline float16x4_t vcvt_f16_f32(float32x4_t v) {
  float16x4_t r = {(_Float16)v[0], (_Float16)v[1], (_Float16)v[2], (_Float16)v[3]};
  return r;
}

static inline float32x4_t vmlaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
  float32x4_t r;
  for (int i = 0; i < 4; ++i) { float p = b[i] * c[i]; r[i] = a[i] + p; }
  return r;
}
static inline float32x4_t vmulq_f32(float32x4_t a, float32x4_t b) {
  float32x4_t r;
  for (int i = 0; i < 4; ++i) r[i] = a[i] * b[i];
  return r;
}
static inline float32x4_t vnegq_f32(float32x4_t a) {
  float32x4_t r;
  for (int i = 0; i < 4; ++i) r[i] = -a[i];
  return r;
}
static inline float vaddvq_f32(float32x4_t a) { return (a[0] + a[1]) + (a[2] + a[3]); }
static inline float16x8_t vaddq_f16(float16x8_t a, float16x8_t b) {
  float16x8_t r;
  for (int i = 0; i < 8; ++i) r[i] = (_Float16)((float)a[i] + (float)b[i]);
  return r;
}
