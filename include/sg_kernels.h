/*
 * SiliconGraph-B200 kernel C ABI.
 *
 * The reference dispatches its CPU kernels "via function pointer through the
 * runtime's kernel table" (compiler/kernels/cpu/matmul_neon.h:9) with the
 * signature `void k(const MatMulParams&)` (matmul_neon.h:32-43) and
 * `void flash_attention_fp16(const FlashAttentionParams&)`
 * (flash_attention.h:25-42, :95).  This header is the table a CUDA graph
 * profile binds instead: the parameter structs keep the reference's field
 * names and meanings, with device pointers, an explicit CUDA stream and a
 * status return added.
 *
 * Conventions
 *  - Every pointer in a params struct is a DEVICE pointer (cudaMalloc'd or
 *    otherwise device-accessible), caller-owned.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *    Calls are asynchronous on that stream and never abort the process.
 *  - Return value: SG_OK (0) or a negative code whose values equal the
 *    reference SDK's ArmStatus (compiler/include/armcc_sdk.h:80-87).  On error
 *    sg_last_error() returns a thread-local message.
 *  - Zero-initialised extension fields select the reference's behaviour.
 *  - There is no CPU fallback: without a usable CUDA device every compute
 *    entry point returns SG_ERR_RUNTIME.
 */
#ifndef SG_KERNELS_H_
#define SG_KERNELS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t SgStatus;
#define SG_OK 0
#define SG_ERR_NOT_FOUND (-1)   /* ARMCC_ERR_NOT_FOUND */
#define SG_ERR_INVALID (-2)     /* ARMCC_ERR_INVALID_PACKAGE: bad argument / layout */
#define SG_ERR_OOM (-3)         /* ARMCC_ERR_OOM */
#define SG_ERR_UNSUPPORTED (-4) /* ARMCC_ERR_UNSUPPORTED */
#define SG_ERR_RUNTIME (-5)     /* ARMCC_ERR_RUNTIME: CUDA error */

/* Element types.  SG_DT_DEFAULT means "the reference kernel's own type". */
typedef enum {
  SG_DT_DEFAULT = 0,
  SG_DT_F32 = 1,
  SG_DT_F16 = 2,
  SG_DT_BF16 = 3,
  SG_DT_I8 = 4
} SgDType;

/* SgMatMulParams.flags */
#define SG_MM_STATIC_WEIGHTS 1u /* B, scales_B and zeros_B are not written by the
                                   kernel launched just before this call on the
                                   stream: the GEMV may start streaming them before
                                   it waits for that kernel (programmatic dependent
                                   launch); A is always read after the wait */
#define SG_MM_A_SWIGLU 2u       /* A holds rows of [gate | up] (2K values each, row
                                   stride lda >= 2K, fp16 or bf16): the GEMM consumes
                                   silu(gate) * up rounded to A's type exactly as
                                   sg_swiglu_rows writes it (the SwiGLU of
                                   ops_swiglu, fused into the down projection).
                                   INT4 only, on the one-row and 2..16-row
                                   kernels; other shapes return SG_ERR_UNSUPPORTED */
#define SG_MM_A_RMSNORM 4u      /* A is one row of the decoder's residual stream
                                   (fp16 or bf16, K values, K % 8 == 0, K <= 8192):
                                   the GEMV consumes the RMSNorm of it with weight
                                   norm_weight and eps norm_eps, rounded to A's
                                   type exactly as sg_rmsnorm writes it (the norm
                                   fused into the next projection).  INT4, one
                                   row, groups of 32k; else SG_ERR_UNSUPPORTED */
#define SG_MM_C_ACCUMULATE 8u   /* C (fp16 or bf16) holds the residual stream:
                                   C = round(C + round(result)), the residual add
                                   of sg_rmsnorm with a residual, fused into the
                                   producing projection.  Same restrictions as
                                   SG_MM_A_RMSNORM */

/*
 * Mirrors armcc::kernels::cpu::MatMulParams (matmul_neon.h:32-43).
 * Fields up to group_size keep the reference's names and meanings; the
 * reference declares scales_B as `const float*` but its INT4 kernel reads it
 * as fp16 (matmul_neon.h:40,118,132) -- here it is `const void*` and its
 * element type is fixed per entry point (documented on each).
 */
typedef struct SgMatMulParams {
  const void* A;          /* [M, K] activations (row m at m*lda)               */
  const void* B;          /* weights; layout per entry point                   */
  const void* bias;       /* [N] fp16, or NULL                                 */
  void* C;                /* [M, N] output (row m at m*ldc)                    */
  int32_t M, K, N;
  int32_t lda, ldb, ldc;  /* leading dims in elements; <= 0 means dense       */
  float scale_A;          /* int8 activation dequant scale                     */
  const void* scales_B;   /* per-group (INT4) or per-channel (INT8) scales     */
  const int8_t* zeros_B;  /* per-group INT4 zero points in [-8, 7], or NULL    */
  int32_t group_size;     /* INT4 group along K; <= 0 means 128 (:120)         */
  /* ---- extensions (zero = reference behaviour) ---- */
  int32_t a_dtype;        /* SgDType of A                                      */
  int32_t c_dtype;        /* SgDType of C                                      */
  void* workspace;        /* optional caller scratch, see *_workspace_size()   */
  size_t workspace_bytes;
  uint32_t flags;         /* SG_MM_* bits; 0 = no assumptions                  */
  const void* norm_weight;/* SG_MM_A_RMSNORM: [K] weight, A's type             */
  float norm_eps;         /* SG_MM_A_RMSNORM: eps (rmsnorm_fp16_neon's)        */
} SgMatMulParams;

/*
 * Mirrors armcc::kernels::cpu::FlashAttentionParams (flash_attention.h:25-42),
 * layouts [B, heads, S, head_dim] (flash_attention.h:116,124,137).
 */
/* Paged KV cache (the reference's planPagedLayout,
 * compiler/lib/memory/kv_cache_layout.cpp:65-102): a pool of pages
 * [page][K|V][kv_head][page_size][head_dim] and a table of int32 physical
 * page ids.  The token at position j of sequence b lives in page
 * table[b * table_batch_stride + (j / page_size) * table_page_stride], row
 * j % page_size.  With paging, the K and V pointers of the calls below are
 * the K and V halves of physical page 0 (V = K + kv_heads * page_size *
 * head_dim elements in the reference layout), and head h of page p starts
 * page_stride * p + h * page_size * head_dim elements after them.  A table
 * entry outside [0, num_pages) is never dereferenced: reads take page 0,
 * writes are dropped, and bit 4 of the device error word is set
 * (sg_device_error_check).  No reference counterpart as a C struct (the
 * reference plans the layout but has no kernel that reads it). */
typedef struct SgKvPages {
  const int32_t* table;       /* device int32 page ids                             */
  int32_t page_size;          /* tokens per page: 16 (the reference's page size)   */
  int32_t num_pages;          /* pages in the pool                                 */
  int64_t page_stride;        /* elements between consecutive physical pages       */
  int64_t table_batch_stride; /* table entries between sequences                   */
  int64_t table_page_stride;  /* table entries between logical pages               */
} SgKvPages;

typedef struct SgFlashAttentionParams {
  const void* Q;          /* [B, num_heads,    S_q,  head_dim]                 */
  const void* K;          /* [B, num_kv_heads, S_kv, head_dim]                 */
  const void* V;          /* [B, num_kv_heads, S_kv, head_dim]                 */
  void* O;                /* [B, num_heads,    S_q,  head_dim]                 */
  const void* mask;       /* must be NULL (the reference never reads it)       */
  int32_t B;
  int32_t S;              /* query length (== key length unless S_kv > 0)      */
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  float scale;            /* <= 0 means 1/sqrt(head_dim) (flash_attention.h:101) */
  int32_t causal;         /* bool in the reference                             */
  int32_t streaming;      /* accepted and ignored, as in the reference         */
  int32_t chunk_size;     /* accepted and ignored, as in the reference         */
  /* ---- extensions (zero = reference behaviour) ---- */
  int32_t io_dtype;       /* SgDType of Q/K/V/O; DEFAULT = fp16 (:96-99)       */
  int32_t S_kv;           /* key/value length; <= 0 means S                    */
  int32_t q_pos0;         /* position of query 0 for the causal test; < 0 means S_kv - S */
  int64_t kv_batch_stride;/* elements between batches of K/V; <= 0 = dense     */
  int64_t kv_head_stride; /* elements between kv heads of K/V; <= 0 = dense    */
  void* workspace;        /* optional caller scratch (decode split-K)          */
  size_t workspace_bytes;
  /* Optional device int32: the position of query 0, read by the kernel at run
   * time (queries then sit at the end: keys = *q_pos_device + S).  S_kv is the
   * capacity the launch is sized for.  Lets one captured CUDA graph of a decode
   * step serve every position.  Decode (sg_flash_decode) form only. */
  const int32_t* q_pos_device;
  /* Optional paged KV cache (NULL: K / V are flat [B, num_kv_heads, S_kv,
   * head_dim] with the strides above, which are then ignored otherwise). */
  const SgKvPages* kv_pages;
} SgFlashAttentionParams;

/* ---------------------------------------------------------------- status */
const char* sg_last_error(void);
int32_t sg_version(void);       /* (major << 16) | (minor << 8) | patch */
/* Number of CUDA devices usable by the library (0 when none). */
int32_t sg_device_count(void);
/* Read and clear the device-side error words of the current device (waits on
 * `stream`): the library's own and the one sg_matmul_int4_grouped_noalloc
 * gives its kernels.  Kernels whose internal waits are bounded record a timeout
 * there instead of hanging; returns SG_ERR_RUNTIME with a message if one was
 * set.  Allocates no device memory. */
int32_t sg_device_error_check(void* stream);
/* Override a launch heuristic (benchmark sweeps).  Keys:
 *   "w4_gemv.groups_per_warp"  INT4 GEMV (CUDA-core path) split-K granularity (0 = heuristic)
 *   "w4_gemv.path"             INT4 GEMV path: 0 auto, 1 CUDA-core, 2 generic
 *   "w4_gemv_mma.variant"      tensor-core GEMV launch shape (0 default .. 3)
 *   "w4_gemv_mma.sleep"        tensor-core GEMV: sleep between stage polls (0/1)
 *   "w4_gemv_mma.cluster"      tensor-core GEMV: allow the cluster-reduced split (1, default) or not (0)
 *   "attn_tc.pair"             tensor-core flash attention: two 128-query tiles per CTA (1, default)
 *                              or one (0); the same bits either way
 *   "w8_gemv_mma.enable"       INT8 per-channel GEMV, one float activation row: the int8 tensor-core
 *                              kernel (1, default) or the dp4a kernel (0)
 *   "gemm_tc.bt"               prefill GEMM token tile: 128, 192 or 256 (0 = heuristic)
 *   "gemm_tc.par"              prefill GEMM dequant warp groups on alternate k steps (1 or 2, default)
 *   "gemm_tc.split"            prefill GEMM: a last round of tiles that fills at most half the SMs runs
 *                              as two k halves per tile on two SMs (1, default; needs the scratch
 *                              the workspace query reports) or whole (0)
 *   "gemm_tc.pair"             prefill GEMM on clusters of two CTAs sharing each MMA (tcgen05
 *                              cta_group::2, 256-column tiles): 0 never (default), 1 when the tiles
 *                              fill the pairs, 2 whenever the token tile is 256
 *   "gemm_tc.tma_store"        prefill GEMM 16-bit C through TMA stores (1, default) or direct stores (0)
 *   "gemm_tc.min_rows"         fewest activation rows sent to the prefill GEMM (default 5)
 *   "gemm_tc.spin"             prefill GEMM single-thread waits spin on test_wait (0 default)
 *   "tp_allreduce.wait_ms"     peer all-reduce: how long a rank waits for the others' flags
 *                              before it gives up and reports (1 .. 2000 ms; <= 0 restores 2000)
 *   "sdk.fuse_norm", "sdk.fuse_rope", "sdk.fuse_swiglu"
 *                              SDK one-row steps: fuse the norms / rope + KV append / SwiGLU
 *                              into the projections (1, default) or run separate kernels (0)
 *   "sdk.decode_step_kernel"   SDK one-sequence decode steps as one persistent kernel (1, when
 *                              the model qualifies) or one kernel per op (0, default)
 * Returns SG_ERR_NOT_FOUND for an unknown key.  No reference counterpart. */
int32_t sg_set_tuning(const char* key, int32_t value);

/* ---------------------------------------------------------- linear layers */

/*
 * INT4 grouped dequant GEMV/GEMM.  Replaces matmul_int4_grouped_neon
 * (compiler/kernels/cpu/matmul_neon.h:113-148).
 *   B        u8  [ceil(K/2), N]: byte (k/2)*N + n, low nibble = even k   (:127)
 *   scales_B f16 [ceil(K/gs), N]                                           (:132)
 *   zeros_B  i8  [ceil(K/gs), N] in [-8, 7], or NULL                       (:133)
 *   C[m, n] = sum_k A[m, k] * scale * ((nibble - 8) - zero)
 * a_dtype: DEFAULT/I8 (reference), F32, F16, BF16.  c_dtype: DEFAULT/F16
 * (reference), F32, BF16.  For int8 A the sum is multiplied by scale_A
 * (the reference ignores scale_A; pass 1.0 for its exact behaviour).  bias,
 * when non-NULL, is added before the output rounding (the reference ignores
 * bias).  ldb must be <= 0 or N.  group_size must be even or K <= group_size.
 */
SgStatus sg_matmul_int4_grouped(const SgMatMulParams* p, void* stream);
/* Scratch bytes the call needs.  When p->workspace is NULL the library
 * supplies it from a per-(device, stream) cache.  A caller-supplied workspace
 * must be at least this large and zero-filled before its first use; calls of
 * the same entry point leave its counters at zero, but a workspace shared with
 * a different entry point must be zero-filled again before reuse.  Returns 0
 * when no scratch is needed. */
size_t sg_matmul_int4_grouped_workspace_size(const SgMatMulParams* p);
/*
 * Same computation and results as sg_matmul_int4_grouped, for callers that are
 * not allowed to allocate device memory after start-up: runtimes that fix
 * their memory budget when a session is admitted and refuse work rather than
 * allocate later, or host frameworks whose memory pool owns the device and
 * forbids direct cudaMalloc.  This entry point has no counterpart in the
 * reference.  It never allocates: its scratch is a fixed 2 MiB array inside
 * the library, held by every GPU that loads the library until the process
 * exits.  The first call on a device looks up that array's device address
 * (make it before any stream capture on that device).  Problems needing more
 * than 2 MiB of scratch are rejected with SG_ERR_INVALID.  p->workspace is
 * ignored.  Calls share the array: calls that overlap on the GPU race, so
 * order them on one stream.  A bounded wait that runs out inside it is
 * reported by sg_device_error_check, like any other kernel's.
 */
SgStatus sg_matmul_int4_grouped_noalloc(const SgMatMulParams* p, void* stream);

/*
 * INT8 per-channel GEMV/GEMM.  Replaces the GLSL gemm_int8 shader
 * (compiler/kernels/gpu/vulkan_shaders.h:53-82) and OpenCL gemm_int8_m1
 * (compiler/kernels/gpu/opencl_kernels.h:36-52).
 *   B        i8  [K, N] row-major (B[k*N + n])
 *   scales_B f32 [N]
 * a_dtype DEFAULT/I8: C[m,n] = float(sum_k A*B as int32) * scale_A * scales_B[n]
 *                     (the shader's exact arithmetic; c_dtype DEFAULT = F32)
 * a_dtype F32/F16/BF16: weight-only variant C[m,n] = scales_B[n] * sum_k A*B
 *                     in fp32 (scale_A unused).  Few rows (decode): each row's
 *                     activations are taken as 24-bit fixed point with one
 *                     power-of-two scale per 8 consecutive k (error at most
 *                     2^-22 of the largest |A| among them, or 2^-122 absolute
 *                     where that is below 2^-100) and reduced exactly in
 *                     int32; many rows: the tcgen05 GEMM in fp32 accumulation.
 */
SgStatus sg_matmul_int8_channel(const SgMatMulParams* p, void* stream);
size_t sg_matmul_int8_channel_workspace_size(const SgMatMulParams* p);

/*
 * fp16-weight GEMV/GEMM.  Replaces matmul_fp16_neon_m1 (matmul_neon.h:48-107).
 *   B f16 [K, N] row-major; bias f16 [N] or NULL, added in fp32 before the
 *   output rounding (as the reference's NEON tail loop, :90-94).
 * a_dtype DEFAULT = F16; c_dtype DEFAULT = F16.
 */
SgStatus sg_matmul_fp16(const SgMatMulParams* p, void* stream);
size_t sg_matmul_fp16_workspace_size(const SgMatMulParams* p);

/*
 * Device-side INT4 packer: quantises W f32 [K, N] (row-major, W[k*N+n]) per
 * (group of group_size along K, column) into the layout above.
 * symmetric == 0: scale = (max-min)/15, zp = clamp(round(-8 - min/scale), -8, 7)
 *   (python/armcc/calibration.py:37-50, per group and column); zeros required.
 * symmetric != 0: scale = absmax/7, zeros may be NULL (nothing written).
 * Bit-identical to the CPU packer of the same convention.
 */
SgStatus sg_quantize_int4_grouped(const float* W, int32_t K, int32_t N, int32_t group_size,
                                  int32_t symmetric, uint8_t* B, uint16_t* scales,
                                  int8_t* zeros, void* stream);
/* Unpack to f32 W[k*N+n] = float(scale) * ((nibble - 8) - zero), the
 * reference's w0f/w1f (matmul_neon.h:127-136), bit for bit. */
SgStatus sg_dequantize_int4_grouped(const uint8_t* B, const uint16_t* scales,
                                    const int8_t* zeros, int32_t K, int32_t N,
                                    int32_t group_size, float* W, void* stream);

/* ---------------------------------------------------------------- attention */

/*
 * Causal (or full) attention.  Replaces flash_attention_fp16 and its per-query
 * kernel flash_attn_head (compiler/kernels/cpu/flash_attention.h:49-144):
 *   O[b,h,i] = softmax_j(scale * Q[b,h,i] . K[b,kvh,j]) V[b,kvh,j]
 *   kvh = h / (num_heads / num_kv_heads)                       (:102,113)
 *   causal: key j is visible to query i iff j <= q_pos0 + i    (:60)
 *   scale <= 0 means 1/sqrt(head_dim)                          (:101)
 * io_dtype: DEFAULT/F16 (reference), F32, BF16; accumulation in fp32.
 * num_heads must be a multiple of num_kv_heads; head_dim in [1, 256].
 * K/V may be strided (kv_batch_stride, kv_head_stride; rows of head_dim
 * elements are contiguous), so a KV cache with more rows than S_kv works.
 */
SgStatus sg_flash_attention(const SgFlashAttentionParams* p, void* stream);
size_t sg_flash_attention_workspace_size(const SgFlashAttentionParams* p);

/*
 * Decode form (few queries against a long KV cache): the keys are split over
 * many blocks (flash-decoding) and the partial softmax states are merged in a
 * fixed order.  Same contract as sg_flash_attention; set S (queries), S_kv
 * and q_pos0 (position of query 0; < 0 means S_kv - S).  Scratch as for the
 * linear kernels (library cache, or caller workspace of
 * sg_flash_decode_workspace_size bytes).
 */
SgStatus sg_flash_decode(const SgFlashAttentionParams* p, void* stream);
size_t sg_flash_decode_workspace_size(const SgFlashAttentionParams* p);

/* ------------------------------------------------------------------ block ops
 * Element-wise transformer-block ops (compiler/kernels/cpu/matmul_neon.h):
 * fp32 arithmetic, one rounding to io_dtype (DEFAULT/F16, BF16, F32) at the
 * end, asynchronous on the stream.
 */

/* y = x * (1 / sqrt(mean(x^2) + eps)) * w per row of n (rmsnorm_fp16_neon,
 * :154-190); x, y [rows, n], w [n].  With residual != NULL the row is first
 * h = round(x + residual), written back to residual (the decoder's residual
 * stream), and h is normalised. */
SgStatus sg_rmsnorm(const void* x, void* residual, const void* w, void* y, int32_t rows, int32_t n, float eps,
                    int32_t io_dtype, void* stream);

/* y = x / (1 + exp(-x)) (silu_fp16_neon, :196-225). */
SgStatus sg_silu(const void* x, void* y, int64_t n, int32_t io_dtype, void* stream);

/* SwiGLU: y = round(silu(gate)) * up. */
SgStatus sg_silu_mul(const void* gate, const void* up, void* y, int64_t n, int32_t io_dtype, void* stream);

/* Row softmax in the reference order (softmax_fp16_neon, :230-256): max;
 * e = round(exp(x - max)); sum of the rounded e; y = round(e * (1 / sum)). */
SgStatus sg_softmax(const void* x, void* y, int32_t rows, int32_t n, int32_t io_dtype, void* stream);

/* Rotary embedding in place on x [tokens, heads, head_dim] (rope_apply_neon,
 * :262-275): pairs (i, i + head_dim/2) rotate by theta = pos / base^(2i/head_dim);
 * pos = positions[t] (device array) or pos0 + t when positions is NULL. */
SgStatus sg_rope(void* x, int32_t tokens, int32_t heads, int32_t head_dim, const int32_t* positions, int32_t pos0,
                 float base, int32_t io_dtype, void* stream);

/* out[t, :] = table[ids[t], :] (table [vocab, hidden]); an id outside
 * [0, vocab) writes zeros and sets the device error word. */
SgStatus sg_embedding(const void* table, const int32_t* ids, void* out, int32_t tokens, int32_t hidden, int32_t vocab,
                      int32_t io_dtype, void* stream);

/* out[r] = index of the largest of logits[r, 0 .. n) (first among equals). */
SgStatus sg_argmax(const float* logits, int32_t rows, int32_t n, int32_t* out, void* stream);

/* ------------------------------------------------------------------ decoder glue
 * qkv [tokens, (heads + 2 kv_heads) * head_dim] (q heads, then k, then v) ->
 * q_out [heads, tokens, head_dim] rotated; k rotated and v appended to the
 * layer's cache rows k_cache / v_cache [kv_heads][.. position ..][head_dim]
 * (kv_head_stride elements between heads) at position positions[t] (device)
 * or pos0 + t.  io_dtype F16 or BF16. */
SgStatus sg_qkv_rope_append(const void* qkv, int32_t tokens, int32_t heads, int32_t kv_heads, int32_t head_dim,
                            const int32_t* positions, int32_t pos0, float base, void* q_out, void* k_cache,
                            void* v_cache, int64_t kv_head_stride, int32_t io_dtype, void* stream);

/* The same with the k / v rows written into a paged KV cache: k_pages / v_pages
 * are the K and V halves of physical page 0 of the layer's pool and `pages`
 * says where each position lives (SgKvPages); batch sequences of seq_tokens
 * tokens each as in sg_qkv_rope_append_batched.  No reference counterpart
 * (the reference's paged layout has no writer). */
SgStatus sg_qkv_rope_append_paged(const void* qkv, int32_t batch, int32_t seq_tokens, int32_t heads,
                                  int32_t kv_heads, int32_t head_dim, const int32_t* positions, int32_t pos0,
                                  float base, void* q_out, void* k_pages, void* v_pages, const SgKvPages* pages,
                                  int32_t io_dtype, void* stream);

/* The q|k|v projection of one decode row fused with the rotary embedding and
 * the KV append: C = the INT4 GEMV of p (M = 1, N = (heads + 2 kv_heads) *
 * head_dim, fp16 or bf16 output; p->C is not written), then exactly what
 * sg_qkv_rope_append does with that output, done in the GEMV's epilogue.  Any
 * p->flags apply (e.g. SG_MM_A_RMSNORM).  head_dim 64 or 128; shapes the
 * one-row tensor-core kernel does not take with a cluster split return
 * SG_ERR_UNSUPPORTED (use the two calls).  No reference counterpart as one
 * call (matmul_int4_grouped_neon then rope_apply_neon). */
typedef struct SgRopeAppend {
  int32_t heads, kv_heads, head_dim;
  const int32_t* positions;   /* device position of the row, or NULL for pos0     */
  int32_t pos0;
  float base;                 /* RoPE theta base                                  */
  void* q_out;                /* [heads, head_dim]                                */
  void* k_cache;              /* flat: [kv_heads] rows at kv_head_stride; paged:   */
  void* v_cache;              /*   the K / V halves of page 0 (SgKvPages)          */
  int64_t kv_head_stride;     /* flat: elements between kv heads                   */
  const SgKvPages* kv_pages;  /* NULL: flat                                        */
} SgRopeAppend;
SgStatus sg_qkv_gemv_rope_append(const SgMatMulParams* p, const SgRopeAppend* rope, void* stream);

/* The same for `batch` sequences of seq_tokens tokens each (token t of the
 * input is token t % seq_tokens of sequence t / seq_tokens): q goes to
 * q_out [batch, heads, seq_tokens, head_dim], k / v of sequence b to the
 * caches at b * kv_batch_stride (elements). */
SgStatus sg_qkv_rope_append_batched(const void* qkv, int32_t batch, int32_t seq_tokens, int32_t heads,
                                    int32_t kv_heads, int32_t head_dim, const int32_t* positions, int32_t pos0,
                                    float base, void* q_out, void* k_cache, void* v_cache, int64_t kv_head_stride,
                                    int64_t kv_batch_stride, int32_t io_dtype, void* stream);

/* SwiGLU over the fused projection gate_up [rows, 2 * ffn] (gate columns, then
 * up columns): y[t, j] = round(silu(gate)) * up. */
SgStatus sg_swiglu_rows(const void* gate_up, void* y, int32_t rows, int32_t ffn, int32_t io_dtype, void* stream);

/* out[r] = argmax of logits[r, 0 .. n) (first among equals) and, when
 * logprob != NULL, logprob[r] = its log-softmax value. */
SgStatus sg_argmax_logprob(const float* logits, int32_t rows, int32_t n, int32_t* out, float* logprob, void* stream);

/* Greedy token across a vocabulary split over ranks (tensor parallelism),
 * one row per sequence.  pack: from this rank's logits shard [rows,
 * vocab_local], its local argmax idx[rows] and local log-probs, writes
 * out3[rows][3] = {max logit, local log-sum-exp, vocab0 + idx}.  pick: from
 * the ranks' triples in rank order ([world][rows][3]), writes each row's
 * global greedy token (first rank among equal maxima, i.e. the lowest
 * vocabulary index) and its log-prob over the whole vocabulary. */
SgStatus sg_tp_argmax_pack(const float* logits, int32_t rows, int32_t vocab_local, const int32_t* idx,
                           const float* logprob, int32_t vocab0, float* out3, void* stream);
SgStatus sg_tp_argmax_pick(const float* all3, int32_t world, int32_t rows, int32_t* next, float* logprob,
                           void* stream);

/* One-shot all-reduce (sum) of n fp16 values over the `world` ranks of a
 * tensor-parallel group through NVLink peer memory, for decode-sized vectors.
 * regions[q] is rank q's region of sg_tp_allreduce_region_bytes(world, max_n)
 * bytes (zero-filled once, mapped into this process, e.g. through CUDA IPC);
 * regions[rank] is this rank's own.  Every rank calls it with the same n, in
 * the same order; n and max_n are multiples of 8, n <= max_n, world <= 8.
 * The result (summed in rank order in fp32, rounded once) replaces data on
 * every rank.  A peer that does not arrive within 2 s leaves data unreduced
 * and sets the device error word (sg_device_error_check). */
size_t sg_tp_allreduce_region_bytes(int32_t world, int32_t max_n);
SgStatus sg_tp_allreduce_f16(void* data, int32_t n, int32_t rank, int32_t world, void* const* regions, int32_t max_n,
                             void* stream);
/* The same sum, not written back to data: residual (fp16 [n]) becomes
 * round(residual + round(sum)) -- the decoder's residual add after a
 * row-parallel projection, fused (what sg_rmsnorm with a residual does to its
 * residual).  No reference counterpart. */
SgStatus sg_tp_allreduce_f16_residual(void* data, int32_t n, int32_t rank, int32_t world, void* const* regions,
                                      int32_t max_n, void* residual, void* stream);

/* in [heads, tokens, head_dim] -> out [tokens, heads, head_dim]. */
SgStatus sg_head_transpose(const void* in, void* out, int32_t heads, int32_t tokens, int32_t head_dim,
                           int32_t io_dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SG_KERNELS_H_ */
