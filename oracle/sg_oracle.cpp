// ORACLE -- test infrastructure, not product code.
//
// CPU restatement of the reference's quantized-block arithmetic, used only by
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the
// checker.  The product path (silicongraph_b200/) never links or calls it.
//
// Each function cites the reference file:line whose steps it restates.  The
// restatement is pinned against the reference's own kernels compiled from
// their headers (oracle/ref_kernels.cpp -> oracle/_ref/libsg_ref.so) by the
// committed golden vectors under tests/golden/.
//
// Build: oracle/Makefile, with -ffp-contract=off so every `a += b * c` keeps
// the reference's separate multiply and add roundings.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>

namespace {

// dtype codes shared with the product C ABI (include/sg_kernels.h SgDType).
enum { DT_DEFAULT = 0, DT_F32 = 1, DT_F16 = 2, DT_BF16 = 3, DT_I8 = 4 };

inline float h2f(uint16_t h) {
  _Float16 v;
  std::memcpy(&v, &h, 2);
  return (float)v;
}
inline uint16_t f2h(float f) {
  _Float16 v = (_Float16)f;
  uint16_t h;
  std::memcpy(&h, &v, 2);
  return h;
}
inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline uint16_t f2bf(float f) {  // round to nearest even; NaN stays NaN
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

inline float load_act(const void* A, int dt, int64_t i) {
  switch (dt) {
    case DT_F32: return ((const float*)A)[i];
    case DT_F16: return h2f(((const uint16_t*)A)[i]);
    case DT_BF16: return bf2f(((const uint16_t*)A)[i]);
    default: return (float)((const int8_t*)A)[i];  // DT_DEFAULT / DT_I8
  }
}
inline void store_out(void* C, int dt, int64_t i, float v) {
  switch (dt) {
    case DT_F32: ((float*)C)[i] = v; break;
    case DT_BF16: ((uint16_t*)C)[i] = f2bf(v); break;
    default: ((uint16_t*)C)[i] = f2h(v); break;  // DT_DEFAULT / DT_F16
  }
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// INT4 grouped dequant GEMV, restating compiler/kernels/cpu/matmul_neon.h:113-143
// (the body of the __ARM_NEON branch, which is the only branch with a loop).
//   packed = B[(k/2)*N + n]                                   (:127)
//   w0 = (packed & 0xF) - 8 ; w1 = (packed >> 4) - 8          (:128-129)
//   group = k / gs ; scale = fp16 scales[group*N+n]           (:131-132)
//   zero = zeros ? zeros[group*N+n] : 0                       (:133)
//   w0f = scale*(w0-zero) ; w1f = scale*(w1-zero)             (:135-136)
//   acc += A[k]*w0f ; acc += (k+1<K) ? A[k+1]*w1f : 0         (:138-139)
//   C[n] = fp16(acc)                                          (:142)
// gs <= 0 means 128 (:120).  The reference reads only row 0 of A and ignores
// M, lda/ldc, bias and scale_A.  Extensions, all inactive at the reference's
// defaults: rows m < M with strides lda/ldc; int8 A multiplied by scale_A
// after the k loop (scale_A = 1 reproduces the reference bit for bit); an
// fp16 bias added in fp32 before the output rounding; activation dtype
// a_dt (default int8) and output dtype c_dt (default fp16).
// ---------------------------------------------------------------------------
void orc_matmul_int4_grouped(const void* A, int a_dt, const uint8_t* B, const uint16_t* scales,
                             const int8_t* zeros, const uint16_t* bias, void* C, int c_dt,
                             int32_t M, int32_t K, int32_t N, int32_t lda, int32_t ldc,
                             int32_t group_size, float scale_A) {
  const int32_t gs = (group_size > 0) ? group_size : 128;
  if (lda <= 0) lda = K;
  if (ldc <= 0) ldc = N;
  // Every column n gets the reference's sequence of fp32 operations in
  // ascending k (per k pair: acc += a0 * w0f, then acc += a1 * w1f, or + 0.0f
  // past an odd K); the loops only visit the columns side by side (k outer,
  // n inner) so that the oracle streams its rows and vectorises.  Each
  // column's accumulator is independent, so the results are the same bits.
  std::vector<float> acc((size_t)N), sc((size_t)N), zf((size_t)N);
  for (int32_t m = 0; m < M; ++m) {
    std::fill(acc.begin(), acc.end(), 0.0f);
    int32_t cur_group = -1;
    for (int32_t k = 0; k < K; k += 2) {
      const int32_t group = k / gs;
      if (group != cur_group) {
        cur_group = group;
        for (int32_t n = 0; n < N; ++n) {
          sc[n] = h2f(scales[(int64_t)group * N + n]);
          zf[n] = zeros ? (float)zeros[(int64_t)group * N + n] : 0.0f;
        }
      }
      const uint8_t* row = B + (int64_t)(k / 2) * N;
      const float a0 = load_act(A, a_dt, (int64_t)m * lda + k);
      const bool odd = k + 1 < K;
      const float a1 = odd ? load_act(A, a_dt, (int64_t)m * lda + k + 1) : 0.0f;
      float* ac = acc.data();
      const float* scp = sc.data();
      const float* zp = zf.data();
      for (int32_t n = 0; n < N; ++n) {
        const uint8_t packed = row[n];
        // (w - zero) is an exact small integer either way: (float)(int) == float - float
        const float w0f = scp[n] * ((float)((int)(packed & 0x0F) - 8) - zp[n]);
        const float w1f = scp[n] * ((float)((int)(packed >> 4) - 8) - zp[n]);
        float v = ac[n] + a0 * w0f;
        v = v + (odd ? a1 * w1f : 0.0f);
        ac[n] = v;
      }
    }
    for (int32_t n = 0; n < N; ++n) {
      float v = acc[n];
      if (a_dt == DT_DEFAULT || a_dt == DT_I8) v = v * scale_A;
      if (bias) v = v + h2f(bias[n]);
      store_out(C, c_dt, (int64_t)m * ldc + n, v);
    }
  }
}

// Dequantised weight W[k*N + n] exactly as the reference forms w0f/w1f
// (matmul_neon.h:127-136): scale * (float)((nibble - 8) - zero).
void orc_dequant_int4_grouped(const uint8_t* B, const uint16_t* scales, const int8_t* zeros,
                              float* W, int32_t K, int32_t N, int32_t group_size) {
  const int32_t gs = (group_size > 0) ? group_size : 128;
  for (int32_t k = 0; k < K; ++k) {
    const int32_t kk = k & ~1;  // the reference takes the group of the even k of a pair
    const int32_t group = kk / gs;
    for (int32_t n = 0; n < N; ++n) {
      const uint8_t packed = B[(int64_t)(k / 2) * N + n];
      const int8_t w = (int8_t)(((k & 1) ? (packed >> 4) : (packed & 0x0F)) - 8);
      const float scale = h2f(scales[(int64_t)group * N + n]);
      const int8_t zero = zeros ? zeros[(int64_t)group * N + n] : 0;
      W[(int64_t)k * N + n] = scale * (float)(w - zero);
    }
  }
}

// ---------------------------------------------------------------------------
// INT4 quantiser (packer).  The reference has no weight quantiser: its INT4
// pass only records metadata (compiler/lib/passes/quantization/quant_passes.cpp:24-61).
// The one asymmetric INT4 convention it does define is
// python/armcc/calibration.py:37-50 (per tensor, in Python floats):
//   scale = (max - min) / 15
//   zp    = clamp(round(-8 - min/scale), -8, 7)      round = half-to-even
// applied here per (group of gs along K, output column n), in double precision
// as Python does, with scale = 1, zp = 0 when max == min (the dataclass
// defaults, calibration.py:32-33).  Storage: scale as fp16, zp as int8 in
// [-8, 7] (the zeros_B the GEMV subtracts, matmul_neon.h:133).
// Quantised value: q = clamp(rint(w / s16) + zp, -8, 7), s16 = the stored
// fp16 scale in fp32, IEEE division; nibble = q + 8 (matmul_neon.h:128-129
// undoes the +8).  Packing: low nibble = even k, high nibble = odd k,
// byte (k/2)*N + n (matmul_neon.h:127); an odd K leaves the last high nibble 0.
// symmetric != 0: scale = absmax / 7 (no reference formula; our choice),
// zeros omitted (zeros == NULL), q = clamp(rint(w / s16), -8, 7).
// W is [K, N] row-major (W[k*N+n]), i.e. nn.Linear.weight transposed.
// ---------------------------------------------------------------------------
void orc_quantize_int4_grouped(const float* W, int32_t K, int32_t N, int32_t group_size,
                               int32_t symmetric, uint8_t* B, uint16_t* scales, int8_t* zeros) {
  const int32_t gs = (group_size > 0) ? group_size : 128;
  const int32_t G = (K + gs - 1) / gs;
  const int32_t KP = (K + 1) / 2;
  std::memset(B, 0, (size_t)KP * N);
  std::vector<int8_t> q((size_t)K);
  for (int32_t n = 0; n < N; ++n) {
    for (int32_t g = 0; g < G; ++g) {
      const int32_t k0 = g * gs, k1 = std::min(K, k0 + gs);
      float mn = W[(int64_t)k0 * N + n], mx = mn, amax = 0.0f;
      for (int32_t k = k0; k < k1; ++k) {
        const float v = W[(int64_t)k * N + n];
        mn = std::min(mn, v);
        mx = std::max(mx, v);
        amax = std::max(amax, std::fabs(v));
      }
      uint16_t s16;
      int32_t zp = 0;
      if (symmetric) {
        const double sd = (amax > 0.0f) ? (double)amax / 7.0 : 1.0;
        s16 = f2h((float)sd);
      } else {
        const double range = (double)mx - (double)mn;
        double sd = 1.0;
        if (range > 0) {
          sd = range / 15.0;
          zp = (int32_t)std::nearbyint(-8.0 - (double)mn / sd);
          zp = std::max(-8, std::min(7, zp));
        }
        s16 = f2h((float)sd);
      }
      float s = h2f(s16);
      scales[(int64_t)g * N + n] = s16;
      if (zeros) zeros[(int64_t)g * N + n] = (int8_t)zp;
      for (int32_t k = k0; k < k1; ++k) {
        const float r = (s > 0.0f) ? std::nearbyint(W[(int64_t)k * N + n] / s) : 0.0f;
        float qf = r + (float)zp;
        qf = std::max(-8.0f, std::min(7.0f, qf));
        q[k] = (int8_t)qf;
      }
    }
    for (int32_t k = 0; k < K; ++k) {
      const uint8_t nib = (uint8_t)(q[k] + 8) & 0x0F;
      B[(int64_t)(k / 2) * N + n] |= (k & 1) ? (uint8_t)(nib << 4) : nib;
    }
  }
}

// ---------------------------------------------------------------------------
// INT8 per-channel GEMM, restating the GLSL gemm_int8 shader
// compiler/kernels/gpu/vulkan_shaders.h:70-81 (identical to OpenCL gemm_int8_m1,
// opencl_kernels.h:37-51):
//   acc_i32 = sum_k int(A[k]) * int(B[k*N + n])
//   C[n] = float(acc) * scale_A * Scales[n]
// Extension: rows m < M (row m of A at m*lda, of C at m*ldc).
// ---------------------------------------------------------------------------
void orc_gemm_int8_channel(const int8_t* A, const int8_t* B, const float* scales, float* C,
                           int32_t M, int32_t K, int32_t N, int32_t lda, int32_t ldc,
                           float scale_A) {
  if (lda <= 0) lda = K;
  if (ldc <= 0) ldc = N;
  for (int32_t m = 0; m < M; ++m)
    for (int32_t n = 0; n < N; ++n) {
      int32_t acc = 0;
      for (int32_t k = 0; k < K; ++k)
        acc += (int32_t)A[(int64_t)m * lda + k] * (int32_t)B[(int64_t)k * N + n];
      C[(int64_t)m * ldc + n] = (float)acc * scale_A * scales[n];
    }
}

// Weight-only INT8 per-channel (dequant variant of the same shader for
// floating activations): C[m,n] = Scales[n] * sum_k A[m,k] * float(B[k*N+n]),
// fp32 accumulation in ascending k.  The reference has no such kernel; this is
// the shader's per-channel dequantisation applied to a float activation.
void orc_gemm_w8_channel(const void* A, int a_dt, const int8_t* B, const float* scales, void* C,
                         int c_dt, int32_t M, int32_t K, int32_t N, int32_t lda, int32_t ldc) {
  if (lda <= 0) lda = K;
  if (ldc <= 0) ldc = N;
  for (int32_t m = 0; m < M; ++m)
    for (int32_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int32_t k = 0; k < K; ++k)
        acc += load_act(A, a_dt, (int64_t)m * lda + k) * (float)B[(int64_t)k * N + n];
      store_out(C, c_dt, (int64_t)m * ldc + n, acc * scales[n]);
    }
}

// ---------------------------------------------------------------------------
// fp16 GEMV, restating matmul_neon.h:101-105 (scalar fallback) with the NEON
// tail loop's bias (:90-94): acc = sum_k A[k]*B[k*N+n] (+ bias[n]); C = fp16(acc).
// Extension: rows m < M, activation/output dtypes as above (default fp16).
// ---------------------------------------------------------------------------
void orc_matmul_f16w(const void* A, int a_dt, const uint16_t* B, const uint16_t* bias, void* C,
                     int c_dt, int32_t M, int32_t K, int32_t N, int32_t lda, int32_t ldc) {
  if (a_dt == DT_DEFAULT) a_dt = DT_F16;
  if (lda <= 0) lda = K;
  if (ldc <= 0) ldc = N;
  for (int32_t m = 0; m < M; ++m)
    for (int32_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int32_t k = 0; k < K; ++k)
        acc += load_act(A, a_dt, (int64_t)m * lda + k) * h2f(B[(int64_t)k * N + n]);
      if (bias) acc += h2f(bias[n]);
      store_out(C, c_dt, (int64_t)m * ldc + n, acc);
    }
}

// ---------------------------------------------------------------------------
// Causal flash attention, restating compiler/kernels/cpu/flash_attention.h.
// One query (flash_attn_head, :49-90): running max m = -inf, normaliser l = 0,
// out = 0; for keys j (stop at j > query_pos when causal):
//   s = (sum_d q[d]*k[j,d]) * scale
//   m' = max(m, s); e = expf(s - m'); c = expf(m - m'); l = l*c + e
//   out[d] = out[d]*c + e*v[j,d]; m = m'
// then out *= 1/l if l > 0.
// Driver (flash_attention_fp16, :95-144): scale = p.scale > 0 ? p.scale :
// 1/sqrtf(D) (:101); kv_group = H / max(1, Hkv) (:102); kv_head = h / kv_group
// (:113); layout [B, heads, S, D] (:116,124,137).
// Extension for decode: queries and keys may differ in length (Sq <= Skv);
// query i sits at position q_pos0 + i.  Sq == Skv with q_pos0 == 0 is the
// reference's self-attention call exactly.  I/O dtype io_dt: f32, f16 or bf16
// (the reference's fp16 I/O is io_dt = f16; flash_attn_head itself is fp32).
// ---------------------------------------------------------------------------
static void attn_head_f32(const float* q, const float* k, const float* v, float* out,
                          int32_t S, int32_t D, float scale, bool causal, int32_t query_pos) {
  float m = -std::numeric_limits<float>::infinity();
  float l = 0.0f;
  std::fill(out, out + D, 0.0f);
  for (int32_t j = 0; j < S; ++j) {
    if (causal && j > query_pos) break;
    float s = 0.0f;
    for (int32_t d = 0; d < D; ++d) s += q[d] * k[(int64_t)j * D + d];
    s *= scale;
    const float m_new = std::max(m, s);
    const float exp_s = expf(s - m_new);
    const float scale_old = expf(m - m_new);
    l = l * scale_old + exp_s;
    for (int32_t d = 0; d < D; ++d) out[d] = out[d] * scale_old + exp_s * v[(int64_t)j * D + d];
    m = m_new;
  }
  if (l > 0) {
    const float inv_l = 1.0f / l;
    for (int32_t d = 0; d < D; ++d) out[d] *= inv_l;
  }
}

static inline float load_io(const void* p, int dt, int64_t i) {
  if (dt == DT_F32) return ((const float*)p)[i];
  if (dt == DT_BF16) return bf2f(((const uint16_t*)p)[i]);
  return h2f(((const uint16_t*)p)[i]);
}

void orc_flash_attention(const void* Q, const void* K, const void* V, void* O, int io_dt,
                         int32_t B, int32_t H, int32_t Hkv, int32_t Sq, int32_t Skv, int32_t D,
                         float scale_in, int32_t causal, int32_t q_pos0) {
  const float scale = (scale_in > 0) ? scale_in : 1.0f / sqrtf((float)D);
  const int32_t kv_group = H / std::max(1, Hkv);
  std::vector<float> q(D), kf((size_t)Skv * D), vf((size_t)Skv * D), out(D);
  for (int32_t b = 0; b < B; ++b)
    for (int32_t h = 0; h < H; ++h) {
      const int32_t kvh = h / kv_group;
      const int64_t kvbase = ((int64_t)b * Hkv + kvh) * Skv * D;
      for (int64_t j = 0; j < (int64_t)Skv * D; ++j) {
        kf[j] = load_io(K, io_dt, kvbase + j);
        vf[j] = load_io(V, io_dt, kvbase + j);
      }
      const int64_t qbase = ((int64_t)b * H + h) * Sq * D;
      for (int32_t s = 0; s < Sq; ++s) {
        for (int32_t d = 0; d < D; ++d) q[d] = load_io(Q, io_dt, qbase + (int64_t)s * D + d);
        attn_head_f32(q.data(), kf.data(), vf.data(), out.data(), Skv, D, scale, causal != 0,
                      q_pos0 + s);
        for (int32_t d = 0; d < D; ++d) {
          const int64_t i = qbase + (int64_t)s * D + d;
          if (io_dt == DT_F32) ((float*)O)[i] = out[d];
          else if (io_dt == DT_BF16) ((uint16_t*)O)[i] = f2bf(out[d]);
          else ((uint16_t*)O)[i] = f2h(out[d]);
        }
      }
    }
}

// ---------------------------------------------------------------------------
// Block elementwise ops (fp16 I/O), restating the scalar branches of
// compiler/kernels/cpu/matmul_neon.h.
// ---------------------------------------------------------------------------
// :185-188  ss = sum x^2 ; r = 1/sqrtf(ss/n + eps) ; y = fp16(x * r * w)
void orc_rmsnorm_f16(const uint16_t* x, const uint16_t* w, uint16_t* y, int32_t n, float eps) {
  float ss = 0;
  for (int32_t i = 0; i < n; ++i) ss += h2f(x[i]) * h2f(x[i]);
  const float rms_inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (int32_t i = 0; i < n; ++i) y[i] = f2h(h2f(x[i]) * rms_inv * h2f(w[i]));
}

// :220-223  y = fp16(x / (1 + expf(-x)))
void orc_silu_f16(const uint16_t* x, uint16_t* y, int32_t n) {
  for (int32_t i = 0; i < n; ++i) {
    const float xi = h2f(x[i]);
    y[i] = f2h(xi / (1.0f + expf(-xi)));
  }
}

// :230-255  max; y = fp16(expf(x - max)); sum += float(y); y = fp16(y * (1/sum))
void orc_softmax_f16(const uint16_t* x, uint16_t* y, int32_t n) {
  float xmax = h2f(x[0]);
  for (int32_t i = 1; i < n; ++i)
    if (h2f(x[i]) > xmax) xmax = h2f(x[i]);
  float sum = 0.0f;
  for (int32_t i = 0; i < n; ++i) {
    y[i] = f2h(expf(h2f(x[i]) - xmax));
    sum += h2f(y[i]);
  }
  const float inv_sum = 1.0f / sum;
  for (int32_t i = 0; i < n; ++i) y[i] = f2h(h2f(y[i]) * inv_sum);
}

// :262-274  rotate-half pairs (i, i + D/2): theta = pos / powf(base, 2i/D)
void orc_rope_f16(uint16_t* x, int32_t head_dim, int32_t position, float base) {
  for (int32_t i = 0; i < head_dim / 2; ++i) {
    const float theta = (float)position / powf(base, 2.0f * i / (float)head_dim);
    const float cos_t = cosf(theta);
    const float sin_t = sinf(theta);
    const float x0 = h2f(x[i]);
    const float x1 = h2f(x[i + head_dim / 2]);
    x[i] = f2h(x0 * cos_t - x1 * sin_t);
    x[i + head_dim / 2] = f2h(x0 * sin_t + x1 * cos_t);
  }
}

// fp32 forms of the same three block ops (fp32 I/O, same operation order),
// used by the decoder composition oracle.
void orc_rmsnorm_f32(const float* x, const float* w, float* y, int32_t n, float eps) {
  float ss = 0;
  for (int32_t i = 0; i < n; ++i) ss += x[i] * x[i];
  const float rms_inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (int32_t i = 0; i < n; ++i) y[i] = x[i] * rms_inv * w[i];
}
void orc_silu_f32(const float* x, float* y, int32_t n) {
  for (int32_t i = 0; i < n; ++i) y[i] = x[i] / (1.0f + expf(-x[i]));
}
void orc_rope_f32(float* x, int32_t head_dim, int32_t position, float base) {
  for (int32_t i = 0; i < head_dim / 2; ++i) {
    const float theta = (float)position / powf(base, 2.0f * i / (float)head_dim);
    const float cos_t = cosf(theta);
    const float sin_t = sinf(theta);
    const float x0 = x[i];
    const float x1 = x[i + head_dim / 2];
    x[i] = x0 * cos_t - x1 * sin_t;
    x[i + head_dim / 2] = x0 * sin_t + x1 * cos_t;
  }
}

}  // extern "C"
