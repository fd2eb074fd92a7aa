// One decode token of a Llama-style INT4 decoder (one sequence, one GPU) as a
// single persistent kernel (decode_step.cu).  Internal to the library: the
// SDK session (sdk_runtime.cpp) builds a DecodeStep for a model that
// qualifies and runs it in place of the per-op decode step.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "sg_kernels.h"

namespace sg {

struct DsLinear {
  const uint8_t* qw = nullptr;    // [ceil(K / 2)][N] packed INT4, the reference layout (matmul_neon.h:113-143)
  const void* scales = nullptr;   // [K / gs][N] fp16
  const int8_t* zeros = nullptr;  // [K / gs][N] int8, or null (symmetric)
  int K = 0, N = 0;
};

struct DsModel {
  int layers = 0, hidden = 0, heads = 0, kv_heads = 0, head_dim = 0, ffn = 0, vocab = 0, group_size = 0;
  float rope_theta = 10000.f, rms_eps = 1e-5f;
  const void* embed = nullptr;  // [vocab_rows][hidden] fp16
  int vocab_rows = 0;
  const void* final_norm = nullptr;  // fp16 [hidden]
  std::vector<const void*> in_norm, post_norm;
  std::vector<DsLinear> qkv, o, gu, down;  // per layer: q|k|v, o, gate|up, down
  DsLinear lm;
  // KV cache per layer: flat [kv_head][max_context][head_dim] fp16 (kv_head_stride
  // elements between heads), or page pools described by `pages` (one per layer)
  std::vector<void*> k_cache, v_cache;
  int64_t kv_head_stride = 0;
  std::vector<SgKvPages> pages;
  int max_context = 0;
};

struct DecodeStep;

// Why this model cannot run as the persistent kernel on `dev`, or nullptr.
const char* decode_step_unsupported(const DsModel& m, int dev);
SgStatus decode_step_create(const DsModel& m, int dev, DecodeStep** out);
// One token: the token id at next[0], its position at pos[0] (device words);
// writes logits [vocab] (fp32), next[0] (the greedy token) and logprob[0], and
// appends the token's K and V rows to the cache.
SgStatus decode_step_run(DecodeStep* ds, const int32_t* pos, int32_t* next, float* logprob, float* logits,
                         cudaStream_t st);
void decode_step_destroy(DecodeStep* ds);
// Device bytes the step holds besides the model (scratch and tensor maps).
size_t decode_step_device_bytes(const DecodeStep* ds);
// Phase timeline (diagnostics): on = record from the next step on (off frees
// the buffer); host (may be null) receives up to cap stamps, [cta][512]: the
// start, then per grid barrier its arrival and release (ns, global timer).
SgStatus decode_step_trace(DecodeStep* ds, bool on, uint64_t* host, size_t cap, size_t* n, int* ctas);

}  // namespace sg
