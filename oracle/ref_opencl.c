/* Test infrastructure only: runs the reference's OpenCL-C INT8 per-channel
 * kernel gemm_int8_m1 (compiler/kernels/gpu/opencl_kernels.h:36-52, held there
 * as the string literal k_gemm_int8_opencl) as plain host C, so that the INT8
 * row is pinned by the reference's own arithmetic without an OpenCL runtime.
 *
 * The recipe (oracle/Makefile, target `ref`) cuts the kernel's source out of
 * that string into oracle/_ref/gemm_int8_m1.cl and compiles this file with it.
 * OpenCL-C's address-space and kernel qualifiers become nothing, `char` is the
 * 8-bit signed type it is in OpenCL (-fsigned-char), and get_global_id(0) is
 * the work-item index that the loop below walks, one call per output column,
 * as the OpenCL runtime would launch one work-item per n.
 *
 * Only tests, the golden-vector generator and bench.py's CPU legs load the
 * resulting library (oracle/_ref/libsg_ref.so). */
#include <stdint.h>

static int sgref_work_item;

#define __kernel static
#define __global
#define get_global_id(dim) (sgref_work_item)

#include "gemm_int8_m1.cl"

/* A int8 [K]; B int8 [K, N] row-major; scales_B f32 [N]; C f32 [N]. */
void sgref_cl_gemm_int8_m1(const int8_t* A, const int8_t* B, const float* scales_B, float* C,
                           int32_t K, int32_t N, float scale_A) {
  for (sgref_work_item = 0; sgref_work_item < N; ++sgref_work_item)
    gemm_int8_m1((const char*)A, (const char*)B, scales_B, C, K, N, scale_A);
}
