/*
 * armcc SDK C API, implemented by libsg_b200.so for packages whose graph entry
 * has execution_backend "cuda".
 *
 * Same names, argument meanings, status codes and struct layouts as the
 * reference's declaration (compiler/include/armcc_sdk.h:36-214), so a runtime
 * written against it links here unchanged.  The reference ships no
 * implementation of these functions; the behaviour below is this library's:
 *   - constructors return NULL on failure; armpack_last_error() gives the
 *     message (thread-local);
 *   - the package owns its graphs; sessions are destroyed by the caller and
 *     must not outlive their package; one session per host thread at a time;
 *   - a session holds one device allocation (weights, KV cache, activation
 *     arena, kernel scratch), sized when it is created;
 *   - armpack_select_graph picks the "cuda" graph with the largest context
 *     length >= state->context_length (else the largest) when a CUDA device
 *     is present; graphs for other backends are listed but their sessions
 *     report ARMCC_ERR_UNSUPPORTED;
 *   - the tokenizer entry points return NULL (token ids in, token ids out).
 * Added here (README.md:72 of the reference names it): armgraph_run.
 */
#ifndef ARMCC_SDK_H_
#define ARMCC_SDK_H_

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ARMCC_SDK_VERSION_MAJOR 0
#define ARMCC_SDK_VERSION_MINOR 1
#define ARMCC_SDK_VERSION_PATCH 0

typedef enum {
  ARMCC_SOC_UNKNOWN = 0,
  ARMCC_SOC_SNAPDRAGON_8_GEN1 = 1,
  ARMCC_SOC_SNAPDRAGON_8_GEN2 = 2,
  ARMCC_SOC_SNAPDRAGON_8_GEN3 = 3,
  ARMCC_SOC_SNAPDRAGON_8_ELITE = 4,
  ARMCC_SOC_SNAPDRAGON_7_GEN3 = 5,
  ARMCC_SOC_DIMENSITY_9300 = 10,
  ARMCC_SOC_DIMENSITY_9200 = 11,
  ARMCC_SOC_DIMENSITY_8300 = 12,
  ARMCC_SOC_EXYNOS_2400 = 20,
  ARMCC_SOC_EXYNOS_2200 = 21,
  ARMCC_SOC_APPLE_A17 = 30,
  ARMCC_SOC_APPLE_A18 = 31,
  ARMCC_SOC_APPLE_M3 = 32,
  ARMCC_SOC_APPLE_M4 = 33,
  ARMCC_SOC_BCM2712 = 40,
  ARMCC_SOC_JETSON_ORIN_NX = 50,
  ARMCC_SOC_GENERIC_ARM64 = 0xFF,
} ArmSoCID;

typedef enum {
  ARMCC_THERMAL_NOMINAL = 0,
  ARMCC_THERMAL_WARM = 1,
  ARMCC_THERMAL_HOT = 2,
  ARMCC_THERMAL_CRITICAL = 3,
} ArmThermalState;

typedef enum {
  ARMCC_LATENCY_INTERACTIVE = 0,
  ARMCC_LATENCY_BATCH = 1,
  ARMCC_LATENCY_BACKGROUND = 2,
} ArmLatencyMode;

typedef enum {
  ARMCC_OK = 0,
  ARMCC_ERR_NOT_FOUND = -1,
  ARMCC_ERR_INVALID_PACKAGE = -2,
  ARMCC_ERR_OOM = -3,
  ARMCC_ERR_UNSUPPORTED = -4,
  ARMCC_ERR_RUNTIME = -5,
} ArmStatus;

typedef struct ArmPackage_ ArmPackage;
typedef struct ArmGraph_ ArmGraph;
typedef struct ArmSession_ ArmSession;

typedef struct {
  ArmSoCID soc_id;
  uint32_t ram_mb;
  int32_t battery_pct;
  ArmThermalState thermal_state;
  ArmLatencyMode latency_mode;
  uint32_t context_length;
  bool gpu_available;
  bool npu_available;
} ArmDeviceState;

typedef struct {
  int32_t num_threads;
  bool use_gpu;
  bool use_npu;
  uint32_t seed;
  bool verbose;
} ArmSessionOptions;

typedef struct {
  int32_t next_token_id;
  float logprob;
  float ttft_ms;
  float tpot_ms;
  uint32_t tokens_generated;
  ArmStatus status;
} ArmInferenceResult;

/* ---------------------------------------------------------------- package */
ArmPackage* armpack_load(const char* path);
void armpack_destroy(ArmPackage* pkg);
const char* armpack_last_error(void);
ArmGraph* armpack_select_graph(ArmPackage* pkg, const ArmDeviceState* state);
uint32_t armpack_num_graphs(const ArmPackage* pkg);
ArmGraph* armpack_get_graph(ArmPackage* pkg, uint32_t index);
const char* armgraph_description(const ArmGraph* graph);
float armgraph_estimated_tpot_ms(const ArmGraph* graph);
uint64_t armgraph_peak_memory_bytes(const ArmGraph* graph);

/* ---------------------------------------------------------------- session */
ArmSession* armgraph_create_session(ArmGraph* graph, const ArmSessionOptions* opts);
void armsess_destroy(ArmSession* sess);
void armsess_reset(ArmSession* sess);
ArmStatus armsess_prefill(ArmSession* sess, const int32_t* tokens, uint32_t n_tokens);
ArmInferenceResult armsess_decode(ArmSession* sess);
ArmStatus armsess_generate(ArmSession* sess, const int32_t* prompt_tokens, uint32_t prompt_len,
                           uint32_t max_new_tokens, void (*output_cb)(int32_t token_id, void* ctx), void* ctx);

/* Convenience: a session on `graph`, prefill `tokens`, one greedy token. */
ArmInferenceResult armgraph_run(ArmGraph* graph, const int32_t* tokens, uint32_t n_tokens);

/* ---------------------------------------------------------------- inspection */
typedef struct {
  char model_id[256];
  char model_family[64];
  char compiler_version[32];
  uint32_t num_graphs;
  uint32_t num_kernels;
  uint32_t num_weight_files;
  uint32_t num_layers;
  uint32_t hidden_size;
  uint32_t vocab_size;
} ArmPackageInfo;

ArmStatus armpack_get_info(const ArmPackage* pkg, ArmPackageInfo* info);
void armpack_print_summary(const ArmPackage* pkg);

/* ---------------------------------------------------------------- tokenizer */
typedef struct ArmTokenizer_ ArmTokenizer;
ArmTokenizer* armpack_get_tokenizer(ArmPackage* pkg);
int32_t* armtok_encode(ArmTokenizer* tok, const char* text, uint32_t* out_len);
char* armtok_decode(ArmTokenizer* tok, const int32_t* tokens, uint32_t n_tokens);
void armtok_free_text(char* text);
void armtok_free_tokens(int32_t* tokens);

#ifdef __cplusplus
}
#endif
#endif /* ARMCC_SDK_H_ */
