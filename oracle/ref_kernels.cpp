// Test infrastructure only: C-ABI wrappers around the reference's own CPU
// kernels, compiled unmodified from their headers where they lie in the
// reference checkout (compiler/kernels/cpu/matmul_neon.h,
// compiler/kernels/cpu/flash_attention.h).  Nothing here is product code;
// only tests, the golden-vector generator and bench.py's CPU baseline load
// the resulting library (oracle/_ref/libsg_ref.so).
//
// The recipe (oracle/Makefile) compiles this file twice:
//   * REF_NEON=1: with -D__ARM_NEON and oracle/neon_shim on the include path,
//     so the NEON branches run -- this is the only way to execute the real
//     INT4 loop (matmul_neon.h:114-142) off-ARM.  Symbols: sgref_neon_*.
//   * REF_NEON=0: plain x86, the headers' scalar `#else` branches.
//     Symbols: sgref_scalar_*.
// Both builds pass -D__fp16=_Float16 (the headers use the ARM-only __fp16
// type, flash_attention.h:96) and -include vector (flash_attention.h:105
// uses std::vector without including it).
#include <cstdint>
#include <vector>

// Keep the two builds' copies of the header functions apart: the headers
// define non-inline functions in namespace armcc::kernels::cpu.
#if REF_NEON
#define armcc armcc_ref_neon
#define SGREF(name) sgref_neon_##name
#else
#define armcc armcc_ref_scalar
#define SGREF(name) sgref_scalar_##name
#endif

#include "matmul_neon.h"
#include "flash_attention.h"

using namespace armcc::kernels::cpu;

extern "C" {

// matmul_neon.h:113 matmul_int4_grouped_neon -- A int8 [K], B u8 [K/2, N],
// scales fp16 [ceil(K/gs), N], zeros int8 [ceil(K/gs), N] or NULL, C fp16 [N].
void SGREF(matmul_int4_grouped)(const int8_t* A, const uint8_t* B, const uint16_t* scales,
                                const int8_t* zeros, uint16_t* C, int32_t K, int32_t N,
                                int32_t group_size) {
  MatMulParams p{};
  p.A = A;
  p.B = B;
  p.bias = nullptr;
  p.C = C;
  p.M = 1;
  p.K = K;
  p.N = N;
  p.lda = K;
  p.ldb = N;
  p.ldc = N;
  p.scale_A = 1.0f;
  p.scales_B = reinterpret_cast<const float*>(scales);  // read as fp16 by the kernel
  p.zeros_B = zeros;
  p.group_size = group_size;
  matmul_int4_grouped_neon(p);
}

// matmul_neon.h:48 matmul_fp16_neon_m1 -- A fp16 [K], B fp16 [K, N], bias fp16 [N] or NULL.
void SGREF(matmul_fp16_m1)(const uint16_t* A, const uint16_t* B, const uint16_t* bias,
                           uint16_t* C, int32_t K, int32_t N) {
  MatMulParams p{};
  p.A = A;
  p.B = B;
  p.bias = bias;
  p.C = C;
  p.M = 1;
  p.K = K;
  p.N = N;
  p.lda = K;
  p.ldb = N;
  p.ldc = N;
  p.scale_A = 1.0f;
  matmul_fp16_neon_m1(p);
}

void SGREF(rmsnorm)(const uint16_t* x, const uint16_t* w, uint16_t* y, int32_t n, float eps) {
  rmsnorm_fp16_neon(reinterpret_cast<const __fp16*>(x), reinterpret_cast<const __fp16*>(w),
                    reinterpret_cast<__fp16*>(y), n, eps);
}

void SGREF(silu)(const uint16_t* x, uint16_t* y, int32_t n) {
  silu_fp16_neon(reinterpret_cast<const __fp16*>(x), reinterpret_cast<__fp16*>(y), n);
}

void SGREF(softmax)(const uint16_t* x, uint16_t* y, int32_t n) {
  softmax_fp16_neon(reinterpret_cast<const __fp16*>(x), reinterpret_cast<__fp16*>(y), n);
}

void SGREF(rope)(uint16_t* x, int32_t head_dim, int32_t position, float base) {
  rope_apply_neon(reinterpret_cast<__fp16*>(x), head_dim, position, base);
}

// flash_attention.h:49 flash_attn_head -- one fp32 query against fp32 K/V rows.
void SGREF(flash_attn_head)(const float* q, const float* k, const float* v, float* out,
                            int32_t S, int32_t head_dim, float scale, int causal,
                            int32_t query_pos) {
  std::vector<float> scores(S > 0 ? S : 1);
  flash_attn_head(q, k, v, out, scores.data(), S, head_dim, scale, causal != 0, query_pos);
}

// flash_attention.h:95 flash_attention_fp16 -- fp16 Q/K/V/O, [B, H, S, D] layout.
void SGREF(flash_attention_fp16)(const uint16_t* Q, const uint16_t* K, const uint16_t* V,
                                 uint16_t* O, int32_t B, int32_t S, int32_t H, int32_t Hkv,
                                 int32_t D, float scale, int causal) {
  FlashAttentionParams p{};
  p.Q = Q;
  p.K = K;
  p.V = V;
  p.O = O;
  p.mask = nullptr;
  p.B = B;
  p.S = S;
  p.num_heads = H;
  p.num_kv_heads = Hkv;
  p.head_dim = D;
  p.scale = scale;
  p.causal = causal != 0;
  p.streaming = false;
  p.chunk_size = 0;
  flash_attention_fp16(p);
}

}  // extern "C"
