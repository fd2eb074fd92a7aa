/*
 * Extensions of the armcc SDK session API (armcc_sdk.h) provided by
 * libsg_b200.so.  No reference counterpart.
 */
#ifndef SG_SDK_EXT_H_
#define SG_SDK_EXT_H_

#include <stdint.h>

#include "armcc_sdk.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Copies the fp32 logits of the last processed token (after
 * armsess_prefill, or after a armsess_decode that ran a step) into host
 * memory: min(n, vocab) values, or for a batched session min(n, batch *
 * vocab) values, sequence by sequence.  Returns ARMCC_OK, or an error
 * status with armpack_last_error() set. */
ArmStatus sg_session_last_logits(ArmSession* sess, float* host_out, uint32_t n);

/* Number of tokens in the session's KV cache. */
uint32_t sg_session_position(const ArmSession* sess);

/* ---- memory-aware graph selection -----------------------------------------
 * armpack_select_graph scores the package's runnable "cuda" graphs as the
 * reference's GraphSelector::score does (compiler/lib/generator/
 * graph_selector.cpp:34-94) and refuses before allocating: a graph whose
 * session would need more than 95 % of the device memory available (free
 * memory of the session's device now, capped by ArmDeviceState.ram_mb when
 * that is non-zero) is rejected (:45-51); NULL when none fits, with the
 * reason in armpack_last_error().  The call below does the same against a
 * stated number of available bytes (no device query: a caller that manages
 * its own device budget, or a test). */
ArmGraph* sg_select_graph_within(ArmPackage* pkg, const ArmDeviceState* state, uint64_t device_bytes_available);

/* Device bytes a session of `batch` sequences on `graph` allocates (its one
 * slab: weights, KV cache for the graph's context, activations, scratch); 0
 * for a graph this library cannot run. */
uint64_t sg_graph_session_bytes(const ArmGraph* graph, uint32_t batch);

/* ---- tensor parallelism --------------------------------------------------
 * One session spread over `world` processes, one GPU each, in the Megatron
 * layout: the q|k|v and gate|up projections are split by output columns
 * (query heads with their kv heads, FFN columns), the output and down
 * projections by input rows, the LM head by vocabulary columns; embedding
 * and norms are replicated.  After each row-split projection the partial
 * hidden states are summed with an NCCL all-reduce; the greedy token is
 * picked from the ranks' (max, log-sum-exp, index) triples after an NCCL
 * all-gather, so every rank emits the same token. */
typedef struct SgTpModel {
  int32_t hidden, heads, kv_heads, head_dim, ffn, vocab, group_size;
} SgTpModel;

typedef struct SgTpShard {
  int32_t q_head0, q_head1;   /* query heads [q_head0, q_head1)                       */
  int32_t kv_head0, kv_head1; /* kv heads [kv_head0, kv_head1); with more ranks than
                                 kv heads each rank holds one kv head, replicated    */
  int32_t ffn0, ffn1;         /* gate / up columns and down rows [ffn0, ffn1)        */
  int32_t vocab0, vocab1;     /* LM head columns [vocab0, vocab1)                    */
} SgTpShard;

/* The shard of `rank` in a group of `world` (host only, no device needed).
 * ARMCC_ERR_UNSUPPORTED when the shapes do not split: heads must divide
 * among the ranks through their kv heads, FFN and vocabulary splits fall on
 * group (resp. 16-column) boundaries, and every o / down row split on a
 * quantisation group boundary. */
ArmStatus sg_tp_shard(const SgTpModel* model, int32_t rank, int32_t world, SgTpShard* out);

/* A fresh 128-byte NCCL unique id: create it on one rank and give the same
 * bytes to every rank's sg_session_create_tp. */
ArmStatus sg_tp_unique_id(uint8_t id_out[128]);

/* This rank's session of a tensor-parallel group.  Collective: every rank
 * of the group calls it with the same id and world, each on its own GPU
 * (SG_DEVICE, else the current device).  NCCL is loaded at run time
 * (libnccl.so.2, or the path in SG_NCCL_LIBRARY). */
ArmSession* sg_session_create_tp(ArmGraph* graph, const ArmSessionOptions* opts, int32_t rank, int32_t world,
                                 const uint8_t id[128]);

/* The vocabulary range [lo, hi) whose logits sg_session_last_logits returns
 * (the whole vocabulary unless the session is tensor-parallel). */
void sg_session_vocab_range(const ArmSession* sess, uint32_t* lo, uint32_t* hi);

/* ---- batched greedy decoding ----------------------------------------------
 * A session of `batch` sequences decoded in lockstep (one position for all):
 * every linear runs on batch rows, attention on batch sequences of the
 * session's KV cache [sequence][layer][K|V][kv_head][seq][dim].  rank /
 * world / id as for sg_session_create_tp (world 1: no NCCL, id unused).
 * armsess_prefill / armsess_decode serve batch-1 sessions; batched ones use
 * the two calls below. */
ArmSession* sg_session_create_ex(ArmGraph* graph, const ArmSessionOptions* opts, uint32_t batch, int32_t rank,
                                 int32_t world, const uint8_t id[128]);

/* ---- failure handling ------------------------------------------------------
 * A tensor-parallel session never blocks forever on its group: the host
 * polls each step, and an asynchronous NCCL error, or a step that has not
 * completed after SG_TP_TIMEOUT_MS milliseconds (default 60000: a rank that
 * stopped answering), aborts the group (ncclCommAbort) and the call returns
 * ARMCC_ERR_RUNTIME with the reason; the peer all-reduce's own waits are
 * bounded (sg_tp_allreduce_f16).  A caller that learns on the host that a
 * rank has left (a store, a heartbeat) calls sg_session_abort before the next
 * step, so nothing is launched towards the departed rank.  An aborted
 * session refuses every later prefill / decode with ARMCC_ERR_RUNTIME and
 * the reason, and can still be destroyed; after a failure in flight the
 * destructor waits at most 10 s for the session's stream and otherwise
 * leaves its device memory allocated (end the process).  This mirrors the reference
 * runtime's refusal with a reason (compiler/lib/runtime/
 * resource_controller.cpp:195-247); the reference itself has no multi-device
 * group. */
ArmStatus sg_session_abort(ArmSession* sess, const char* reason);

/* ---- paged KV cache ---------------------------------------------------------
 * Sessions lay out their KV cache as the reference's planner recommends
 * (compiler/lib/memory/kv_cache_layout.cpp:107-130): flat up to a 4096-token
 * context, paged above it -- a pool of pages [page][K|V][kv_head][16][dim]
 * and a page table [logical page][layer][sequence] (:65-102).  Pages are
 * taken from the pool as the positions advance and returned by
 * armsess_reset.  SG_KV_LAYOUT=flat or =paged in the environment overrides
 * the rule.  This call always pages, with a pool of kv_pool_tokens tokens
 * over all sequences (0: every sequence's full context), so a session
 * reserves only the KV memory its prompts and generations will use; a
 * prefill or decode that needs more pages than are left fails with
 * ARMCC_ERR_OOM before launching anything.  rank / world / id as for
 * sg_session_create_ex. */
ArmSession* sg_session_create_paged(ArmGraph* graph, const ArmSessionOptions* opts, uint32_t batch,
                                    uint64_t kv_pool_tokens, int32_t rank, int32_t world, const uint8_t id[128]);

/* 1 when the session's KV cache is paged (then *pool_pages and
 * *pages_in_use are set), else 0 (both set to 0). */
int32_t sg_session_kv_pages(const ArmSession* sess, uint32_t* pool_pages, uint32_t* pages_in_use);

/* 1 when the session's one-token decode steps run as the persistent
 * decode-step kernel (one sequence on one GPU, built on the first decode
 * step while tuning key "sdk.decode_step_kernel" is 1), else 0 with the
 * reason in *why (static or session-owned text; may be NULL). */
int32_t sg_session_step_kernel(const ArmSession* sess, const char** why);

/* Diagnostics of the decode-step kernel: on != 0 makes the following steps
 * record a timeline (on == 0 stops and frees it); host (may be NULL) receives
 * up to cap global-timer stamps in ns, [cta][512]: the step's start, then per
 * grid barrier its arrival and its release, then the end of the LM head.
 * Returns the stamps copied (and the CTA count in *ctas), or -1. */
int32_t sg_session_step_trace(ArmSession* sess, int32_t on, uint64_t* host, uint32_t cap, int32_t* ctas);

/* Device time of decode steps: on != 0 starts timing the following steps
 * (CUDA events on the session's stream around each step) and returns 0;
 * on == 0 stops and returns the mean device milliseconds per timed step (0
 * when none ran).  -1 on error.  The host-side time per step is
 * ArmInferenceResult.tpot_ms. */
double sg_session_step_gpu_ms(ArmSession* sess, int32_t on);

/* Kernel launches in one captured decode step (the kernel nodes of the
 * session's decode graph whose kernels are this library's: NCCL's excluded), or -1 before the
 * graph exists (the second decode step captures it) or when steps run eagerly. */
int32_t sg_session_graph_kernels(const ArmSession* sess);

/* Prefills every sequence with n_tokens tokens (tokens[b * n_tokens + i] is
 * token i of sequence b). */
ArmStatus sg_batch_prefill(ArmSession* sess, const int32_t* tokens, uint32_t n_tokens);

/* Greedy tokens of all sequences into next_tokens[batch]: the first call
 * after a prefill returns the tokens the prompts predict, later calls run
 * one decode step each. */
ArmStatus sg_batch_decode(ArmSession* sess, int32_t* next_tokens);

/* Sequences of the session. */
uint32_t sg_session_batch(const ArmSession* sess);

#ifdef __cplusplus
}
#endif
#endif /* SG_SDK_EXT_H_ */
