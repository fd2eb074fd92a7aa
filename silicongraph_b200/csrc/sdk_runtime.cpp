// The armcc SDK (armcc_sdk.h) over the B200 kernels: package loading, graph
// selection and decoder sessions for graph entries with execution_backend
// "cuda".  The reference declares this API (compiler/include/armcc_sdk.h:
// 128-214) without implementing it; the runtime flow follows its documented
// intent (docs/package_format.md:164-174): load -> select -> session ->
// prefill / decode.
//
// A "cuda" graph entry points at a graph file (format "sg-cuda-decoder")
// holding the decoder's hyperparameters and a tensor index into one weight
// file of 4096-aligned tensors: fp16 embeddings and norms, and every linear
// in the reference's INT4 layout (matmul_neon.h:113-147: u8 [K/2, N], fp16
// scales and int8 zeros [K/gs, N]), with q/k/v and gate/up fused along N.
//
// A session makes one device allocation (the memory planner's arena idea,
// memory_planner.cpp:172-234, on a single cudaMalloc):
//   [weights | KV cache [layer][K|V][kv_head][seq][dim] (kv_cache_layout.cpp:
//    16-53) | activations at planner offsets | linear-kernel scratch |
//    attention scratch]
// and runs Llama-style blocks: rmsnorm -> QKV -> rope + KV append -> causal
// attention -> O -> residual rmsnorm -> gate|up -> SwiGLU -> down, then the
// final norm, the LM head (fp32 logits) and a greedy argmax.
//
// A tensor-parallel session (sg_session_create_tp) holds one rank's shard of
// every linear, cut out of the full weight image on the device with strided
// copies: q|k|v and gate|up by output columns, o and down by input rows on
// quantisation-group boundaries, the LM head by vocabulary columns.  NCCL
// (loaded with dlopen, so the library never pins an NCCL version of its own)
// sums the row-split outputs and gathers the ranks' greedy candidates.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <string_view>
#include <thread>
#include <vector>

#include "armcc_sdk.h"
#include "sdk_io.h"
#include "sg_sdk_ext.h"
#include "sg_kernels.h"
#include "decode_step.h"

namespace sg {  // libsg_b200 internals (w4_gemv_mma.cu, sg_runtime.cu)
size_t w4_gemv_mma_scratch_bytes(const SgMatMulParams* p, int sms, bool* applicable);
int sm_count(int dev);
int* existing_device_error_word(int dev);
}  // namespace sg

using sgsdk::Json;

namespace {

thread_local std::string g_err;

void set_err(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
}

uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

struct TensorRef {
  uint64_t offset = 0, bytes = 0;
  std::string dtype;
  std::vector<int64_t> shape;
};

struct ModelCfg {
  int layers = 0, hidden = 0, heads = 0, kv_heads = 0, head_dim = 0, ffn = 0, vocab = 0;
  float rope_theta = 10000.f, rms_eps = 1e-5f;
  int group_size = 128;
  bool zeros = true;
  bool lm_int4 = true;
  int max_context = 4096, max_chunk = 512;
  int vocab_global = 0;  // rows of the embedding table (vocab is the LM head's columns here)
  int nqkv() const { return (heads + 2 * kv_heads) * head_dim; }
};

// ------------------------------------------------------------------ NCCL at run time
struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  // failure handling (NULL when the loaded NCCL lacks them)
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
};

// The NCCL the host process already loaded (e.g. PyTorch's), else SG_NCCL_LIBRARY, else libnccl.so.2.
const NcclApi& nccl_api() {
  static const NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) {
      const char* path = getenv("SG_NCCL_LIBRARY");
      h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    }
    if (!h) {
      const char* e = dlerror();
      a.why = std::string("cannot load NCCL: ") + (e ? e : "unknown error");
      return a;
    }
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.comm_abort = reinterpret_cast<decltype(a.comm_abort)>(dlsym(h, "ncclCommAbort"));
    a.comm_get_async_error = reinterpret_cast<decltype(a.comm_get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    a.ok = a.get_unique_id && a.comm_init_rank && a.all_reduce && a.all_gather && a.comm_destroy && a.error_string;
    if (!a.ok) a.why = "the loaded NCCL library lacks a required symbol";
    return a;
  }();
  return api;
}

// ------------------------------------------------------------------ tensor-parallel shard
bool tp_plan(const SgTpModel& m, int rank, int world, SgTpShard* s, std::string* why) {
  auto fail = [&](const std::string& w) {
    *why = w;
    return false;
  };
  if (world < 1 || rank < 0 || rank >= world) return fail("rank outside [0, world)");
  if (m.heads <= 0 || m.kv_heads <= 0 || m.heads % m.kv_heads != 0 || m.head_dim <= 0 || m.ffn <= 0 ||
      m.vocab <= 0 || m.group_size <= 0 || m.hidden <= 0)
    return fail("bad model dimensions");
  const int G = m.heads / m.kv_heads, D = m.head_dim, gs = m.group_size;
  if (world <= m.kv_heads) {
    if (m.kv_heads % world != 0) return fail("kv heads do not divide among the ranks");
    s->kv_head0 = (int)((int64_t)rank * m.kv_heads / world);
    s->kv_head1 = (int)((int64_t)(rank + 1) * m.kv_heads / world);
    s->q_head0 = s->kv_head0 * G;
    s->q_head1 = s->kv_head1 * G;
  } else {
    if (world % m.kv_heads != 0) return fail("ranks do not divide among the kv heads");
    const int R = world / m.kv_heads, kv = rank / R, sub = rank % R;
    if (G < R) return fail("fewer query heads per kv head than ranks sharing it");
    s->kv_head0 = kv;
    s->kv_head1 = kv + 1;
    s->q_head0 = kv * G + sub * G / R;
    s->q_head1 = kv * G + (sub + 1) * G / R;
  }
  if ((s->q_head0 * D) % gs != 0 || (s->q_head1 * D) % gs != 0)
    return fail("the output projection's row split falls inside a quantisation group");
  if (((s->q_head1 - s->q_head0 + 2 * (s->kv_head1 - s->kv_head0)) * D) % 16 != 0)
    return fail("the q|k|v shard is not a multiple of 16 columns");
  if (m.ffn % gs != 0 || m.ffn / gs < world) return fail("the FFN does not split on quantisation groups");
  const int64_t gf = m.ffn / gs;
  s->ffn0 = (int)(rank * gf / world * gs);
  s->ffn1 = (int)((rank + 1) * gf / world * gs);
  if (m.vocab % 16 != 0 || m.vocab / 16 < world) return fail("the vocabulary does not split on 16 columns");
  const int64_t vb = m.vocab / 16;
  s->vocab0 = (int)(rank * vb / world * 16);
  s->vocab1 = (int)((rank + 1) * vb / world * 16);
  return true;
}

// ------------------------------------------------------------------ activation plan
// Greedy best-fit interval colouring (memory_planner.cpp:172-234): buffers in
// order of first use take the smallest free slot released before their first
// use, else a new slot at the arena top.
struct Buf {
  const char* name;
  uint64_t bytes;
  int first, last;
  uint64_t offset = 0;
};

uint64_t plan_offsets(std::vector<Buf>& bufs, uint64_t align) {
  std::vector<Buf*> order;
  for (auto& b : bufs) order.push_back(&b);
  std::stable_sort(order.begin(), order.end(), [](const Buf* a, const Buf* b) { return a->first < b->first; });
  struct Slot {
    uint64_t offset, size;
    int freed_at;
  };
  std::vector<Slot> slots;
  uint64_t top = 0;
  for (Buf* b : order) {
    const uint64_t need = align_up(std::max<uint64_t>(b->bytes, 1), align);
    Slot* best = nullptr;
    for (auto& s : slots)
      if (s.freed_at <= b->first && s.size >= need && (!best || s.size < best->size)) best = &s;
    if (best) {
      b->offset = best->offset;
      best->freed_at = b->last + 1;
    } else {
      top = align_up(top, align);
      b->offset = top;
      slots.push_back({top, need, b->last + 1});
      top += need;
    }
  }
  return top;
}

// Ops of one decoder step, numbered for the lifetimes below.
enum : int { kOpEmbed = 0, kOpNorm1 = 1, kOpQkv, kOpRope, kOpAttn, kOpTrans, kOpO, kOpNorm2, kOpGu, kOpSwiglu,
             kOpDown, kOpNextLayer, kOpFinalNorm, kOpLm, kOpArgmax };

struct Plan {
  std::vector<Buf> bufs;
  uint64_t bytes = 0;
  uint64_t off(const char* n) const {
    for (auto& b : bufs)
      if (!strcmp(b.name, n)) return b.offset;
    return 0;
  }
};

// T = rows of one forward pass (sequences x tokens per sequence), B = sequences.
Plan make_plan(const ModelCfg& c, int T, int B, int world) {
  const uint64_t H = c.hidden, e = 2;
  Plan p;
  p.bufs = {
      {"ids", (uint64_t)T * 4, kOpEmbed, kOpArgmax},
      {"next", (uint64_t)B * 4, kOpEmbed, kOpArgmax},
      {"logprob", (uint64_t)B * 4, kOpEmbed, kOpArgmax},
      {"pos", 4, kOpEmbed, kOpArgmax},
      {"resid", T * H * e, kOpEmbed, kOpFinalNorm},
      {"x_emb", T * H * e, kOpEmbed, kOpNorm1},
      {"xnorm", T * H * e, kOpNorm1, kOpLm},
      {"qkv", (uint64_t)T * c.nqkv() * e, kOpQkv, kOpRope},
      {"qh", (uint64_t)c.heads * T * c.head_dim * e, kOpRope, kOpAttn},
      {"attn", (uint64_t)c.heads * T * c.head_dim * e, kOpAttn, kOpO},
      {"attn_t", (uint64_t)T * c.heads * c.head_dim * e, kOpTrans, kOpO},
      {"o", T * H * e, kOpO, kOpNorm2},
      {"gu", (uint64_t)T * 2 * c.ffn * e, kOpGu, kOpSwiglu},
      {"act", (uint64_t)T * c.ffn * e, kOpSwiglu, kOpDown},
      {"down", T * H * e, kOpDown, kOpFinalNorm},
      {"last_x", (uint64_t)B * H * e, kOpFinalNorm, kOpLm},  // each sequence's last row
      {"last_r", (uint64_t)B * H * e, kOpFinalNorm, kOpLm},
      {"last_n", (uint64_t)B * H * e, kOpFinalNorm, kOpLm},
      {"logits", (uint64_t)B * c.vocab * 4, kOpLm, kOpArgmax},
      {"tp_mine", (uint64_t)B * 12, kOpArgmax, kOpArgmax},
      {"tp_all", (uint64_t)world * B * 12, kOpArgmax, kOpArgmax},
  };
  p.bytes = plan_offsets(p.bufs, 256);
  return p;
}

}  // namespace

// ================================================================== handles
struct ArmPackage_;

struct ArmGraph_ {
  ArmPackage_* pkg = nullptr;
  uint32_t index = 0;
  std::string id, path, backend, description;
  float ttft_ms = 0, tpot_ms = 0;
  uint64_t peak_bytes = 0;
  uint32_t context_length = 0;
  int thermal = 0;             // manifest thermal_state: 0 nominal, 1 warm, 2 hot, 3 critical
  int latency = 0;             // manifest latency_mode: 0 interactive, 1 batch, 2 background
  bool runnable = false;       // a "cuda" graph whose graph file parsed
  std::string why_not;         // reason when not runnable
  ModelCfg cfg;
  std::string weight_path;     // entry of the weight file inside the package
  std::map<std::string, TensorRef> tensors;
};

struct ArmPackage_ {
  sgsdk::Container box;
  Json manifest;
  std::string model_id, family, compiler_version;
  uint32_t num_layers = 0, hidden = 0, vocab = 0;
  uint32_t num_kernels = 0, num_weight_files = 0;
  std::vector<std::unique_ptr<ArmGraph_>> graphs;
};

namespace {

bool parse_cuda_graph(ArmPackage_* pkg, ArmGraph_* g, std::string* why) {
  std::string text, err;
  if (!pkg->box.read_text(g->path, &text, &err)) {
    *why = "graph file: " + err;
    return false;
  }
  Json j;
  if (!sgsdk::json_parse(text, &j, &err)) {
    *why = "graph file " + g->path + ": " + err;
    return false;
  }
  if (j["format"].text() != "sg-cuda-decoder") {
    *why = "graph file " + g->path + " is not an sg-cuda-decoder description";
    return false;
  }
  const Json& m = j["model"];
  ModelCfg& c = g->cfg;
  c.layers = (int)m["num_layers"].integer();
  c.hidden = (int)m["hidden_size"].integer();
  c.heads = (int)m["num_heads"].integer();
  c.kv_heads = (int)m["num_kv_heads"].integer(c.heads);
  c.head_dim = (int)m["head_dim"].integer(c.heads ? c.hidden / c.heads : 0);
  c.ffn = (int)m["intermediate_size"].integer();
  c.vocab = (int)m["vocab_size"].integer();
  c.vocab_global = c.vocab;
  c.rope_theta = (float)m["rope_theta"].number(10000.0);
  c.rms_eps = (float)m["rms_norm_eps"].number(1e-5);
  const Json& qz = j["quant"];
  c.group_size = (int)qz["group_size"].integer(128);
  c.zeros = qz["zero_point"].boolean(true);
  c.lm_int4 = qz["lm_head"].text("int4") == "int4";
  c.max_context = (int)j["max_context"].integer(4096);
  c.max_chunk = (int)j["max_prefill_chunk"].integer(512);
  if (c.layers <= 0 || c.hidden <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.head_dim <= 0 || c.ffn <= 0 ||
      c.vocab <= 0 || c.heads % c.kv_heads != 0 || c.head_dim % 2 != 0 || c.max_context <= 0 || c.max_chunk <= 0) {
    *why = "graph file " + g->path + ": inconsistent model description";
    return false;
  }
  // weight file and its tensor index
  const std::string wid = j["weights"].text();
  const Json& ws = pkg->manifest["weights"];
  for (size_t i = 0; i < ws.size(); ++i)
    if (ws[i]["id"].text() == wid) g->weight_path = ws[i]["path"].text();
  if (g->weight_path.empty()) {
    *why = "weight file '" + wid + "' is not listed in the manifest";
    return false;
  }
  std::string itext;
  if (!pkg->box.read_text(j["tensor_index"].text(), &itext, &err)) {
    *why = "tensor index: " + err;
    return false;
  }
  Json idx;
  if (!sgsdk::json_parse(itext, &idx, &err)) {
    *why = "tensor index: " + err;
    return false;
  }
  for (auto& kv : idx["tensors"].obj) {
    TensorRef t;
    t.offset = (uint64_t)kv.second["offset"].integer();
    t.bytes = (uint64_t)kv.second["bytes"].integer();
    t.dtype = kv.second["dtype"].text();
    for (size_t i = 0; i < kv.second["shape"].size(); ++i) t.shape.push_back(kv.second["shape"][i].integer());
    g->tensors[kv.first] = t;
  }
  return true;
}

}  // namespace

// ================================================================== session
struct Linear {
  const uint8_t* qw = nullptr;
  const void* scales = nullptr;
  const int8_t* zeros = nullptr;
  int K = 0, N = 0;
};

struct ArmSession_ {
  ArmGraph_* g = nullptr;
  ModelCfg c;
  int dev = 0;
  cudaStream_t st = nullptr;
  char* slab = nullptr;
  uint64_t slab_bytes = 0;
  // weights
  const void* embed = nullptr;
  const void* final_norm = nullptr;
  std::vector<const void*> in_norm, post_norm;
  std::vector<Linear> qkv, o, gu, down;
  Linear lm;
  const void* lm_f16 = nullptr;
  // KV cache
  char* kv = nullptr;
  int64_t kv_head_stride = 0;  // elements
  int64_t kv_block = 0;        // elements of one [kv_head][seq][dim] block (K or V of one layer)
  // Paged KV cache (kv_cache_layout.cpp:65-102): `kv` is then a pool of
  // pages [page][K|V][kv_head][16][dim] and d_table [logical page][layer]
  // [sequence] maps every 16 positions of a sequence in a layer to a page.
  // Pages are taken from the pool as positions advance (all sequences in
  // lockstep) and returned on reset.
  bool paged = false;
  int pool_pages = 0, max_lpages = 0, lpages = 0;
  int32_t* d_table = nullptr;     // in the slab
  std::vector<int32_t> h_table;   // host copy
  std::vector<int32_t> free_pages;
  std::vector<SgKvPages> kvp;     // per layer
  // activations
  Plan plan;
  char* act = nullptr;
  char* lin_ws = nullptr;
  uint64_t lin_ws_bytes = 0;
  char* attn_ws = nullptr;
  uint64_t attn_ws_bytes = 0;
  // state
  int pos = 0;
  bool emitted = true;
  int32_t next_host = -1;
  float logprob_host = 0;
  uint32_t generated = 0;
  float ttft_ms = 0, tpot_ms = 0;
  std::chrono::steady_clock::time_point t_prefill_start;
  bool ttft_pending = false;
  // decode step as a CUDA graph: positions come from the device ("pos")
  bool use_graph = true;
  bool graph_failed = false;
  int eager_steps = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t graph_exec = nullptr;
  int32_t* h_pos = nullptr;  // pinned
  // pinned landing block of a step's results: [batch] greedy tokens, the
  // log-probability, the library's device error word
  int32_t* h_res = nullptr;
  int* graph_err_word = nullptr;  // the device error word the decode graph copies (null: none existed)
  // sequences decoded together (sg_session_create_ex), in lockstep at one position
  int batch = 1;
  std::vector<int32_t> next_all;  // host copy of every sequence's greedy token
  // tensor parallelism (tp_world == 1: a whole-model session)
  int tp_rank = 0, tp_world = 1;
  SgTpShard shard{};
  ncclComm_t comm = nullptr;
  int* tp_flag = nullptr;  // device word for the ranks' agreement on setup
  // peer-memory all-reduce of decode-sized sums (sg_tp_allreduce_f16); NCCL otherwise
  void* ar_region = nullptr;
  int ar_max = 0;
  std::vector<void*> ar_regions;  // every rank's region as mapped here (own one at tp_rank)
  // failure handling: a session whose group failed (or was aborted) refuses
  // every later call with the reason; tp_timeout_ms bounds a host wait for a
  // step whose collectives do not complete (SG_TP_TIMEOUT_MS, default 60 s)
  bool aborted = false;
  std::string abort_why;
  // every projection's one-row shape runs on the kernel that fuses the norms (SG_MM_A_RMSNORM / C_ACCUMULATE)
  bool norm_fusable = false;
  bool rope_fusable = false;  // ... and the q|k|v one is a cluster split with head_dim 64 / 128
  // one-sequence decode steps as one persistent kernel (decode_step.cu), built
  // on the first such step; ds_why says why not when it could not be
  sg::DecodeStep* ds = nullptr;
  bool ds_tried = false;
  std::string ds_why;
  // optional device time of the decode steps (sg_session_step_gpu_ms): events
  // recorded on the stream around each step
  cudaEvent_t ev_step[2] = {nullptr, nullptr};
  bool ev_pending = false;
  double step_gpu_ms = 0;
  uint64_t step_gpu_n = 0;
  int tp_timeout_ms = 60000;

  ~ArmSession_() {
    if (aborted && st) {
      // a group that failed in flight: wait a bounded time for the stream; if
      // it does not drain, leak the session's device memory rather than block
      // or free memory a kernel may still use (the process should end)
      const auto t0 = std::chrono::steady_clock::now();
      while (cudaStreamQuery(st) == cudaErrorNotReady) {
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) return;
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
      }
      cudaGetLastError();
    }
    if (st) cudaStreamSynchronize(st);
    if (graph_exec) cudaGraphExecDestroy(graph_exec);
    sg::decode_step_destroy(ds);
    for (cudaEvent_t e : ev_step)
      if (e) cudaEventDestroy(e);
    if (graph) cudaGraphDestroy(graph);
    for (size_t q = 0; q < ar_regions.size(); ++q)
      if ((int)q != tp_rank && ar_regions[q]) cudaIpcCloseMemHandle(ar_regions[q]);
    if (ar_region) cudaFree(ar_region);
    if (comm) nccl_api().comm_destroy(comm);  // after the graphs that hold its calls
    if (tp_flag) cudaFree(tp_flag);
    if (slab) cudaFree(slab);
    if (h_pos) cudaFreeHost(h_pos);
    if (h_res) cudaFreeHost(h_res);
    if (st) cudaStreamDestroy(st);
  }

  template <typename T>
  T* buf(const char* n) { return reinterpret_cast<T*>(act + plan.off(n)); }
  // KV cache [sequence][layer][K|V][kv_head][seq][dim]
  int64_t kv_bstride() const { return (int64_t)c.layers * 2 * kv_block; }  // elements per sequence
  // flat: the layer's K / V blocks; paged: the K / V halves of page 0 of the pool
  void* kcache(int l) { return paged ? kv : kv + (size_t)(2 * l) * kv_block * 2; }
  void* vcache(int l) {
    return paged ? kv + (size_t)c.kv_heads * 16 * c.head_dim * 2 : kv + (size_t)(2 * l + 1) * kv_block * 2;
  }
};

namespace {

ArmStatus fail_sg(SgStatus s, const char* what) {
  set_err("%s failed: %s", what, sg_last_error());
  return s == SG_ERR_OOM ? ARMCC_ERR_OOM : ARMCC_ERR_RUNTIME;
}

#define SG_TRY(call, what)                    \
  do {                                        \
    const SgStatus s_ = (call);               \
    if (s_ != SG_OK) return fail_sg(s_, what); \
  } while (0)

// Sums a row-split projection's fp16 output over the ranks (in place).
ArmStatus tp_sum(ArmSession_* S, void* buf, size_t count) {
  if (S->tp_world == 1) return ARMCC_OK;
  if (S->ar_region && count <= (size_t)S->ar_max && count % 8 == 0) {
    SG_TRY(sg_tp_allreduce_f16(buf, (int32_t)count, S->tp_rank, S->tp_world, S->ar_regions.data(), S->ar_max, S->st),
           "peer all-reduce");
    return ARMCC_OK;
  }
  const ncclResult_t e = nccl_api().all_reduce(buf, buf, count, ncclHalf, ncclSum, S->comm, S->st);
  if (e != ncclSuccess) {
    set_err("ncclAllReduce failed: %s", nccl_api().error_string(e));
    return ARMCC_ERR_RUNTIME;
  }
  return ARMCC_OK;
}

// Single-row decode steps fuse the SwiGLU into the down projection's
// activation staging (SG_MM_A_SWIGLU) instead of launching it separately.
// (Measured on B200, Llama-1B shape: 1 row 665 vs 687 us per step; at 16 rows
// every 128-column tile recomputing silu for its K range cost more than the
// separate kernel, 1108 vs 1084 us, so batched steps keep the two kernels.)
std::atomic<int> g_fuse_swiglu{1};

// Single-row steps on one GPU fuse the decoder's RMSNorms and residual adds
// into the projections (SG_MM_A_RMSNORM on q|k|v, gate|up and the LM head,
// SG_MM_C_ACCUMULATE on o and down): the residual stream lives in "resid", the
// embedding writes it directly, and no separate norm kernel runs.
std::atomic<int> g_fuse_norm{1};
// ... and the rope + KV append into the q|k|v projection's epilogue
// (sg_qkv_gemv_rope_append), when its plan is a cluster split.
std::atomic<int> g_fuse_rope{1};
// ... and, for one sequence, the whole step runs as one persistent kernel
// (decode_step.cu) when the model qualifies and the switch is on.
std::atomic<int> g_step_kernel{0};

ArmStatus linear(ArmSession_* S, const Linear& L, const void* A, void* C, int M, int c_dt, uint32_t flags = 0,
                 const void* norm_w = nullptr) {
  SgMatMulParams p{};
  p.norm_weight = norm_w;
  p.norm_eps = S->c.rms_eps;
  p.A = A;
  p.B = L.qw;
  p.C = C;
  p.M = M;
  p.K = L.K;
  p.N = L.N;
  p.scales_B = L.scales;
  p.zeros_B = L.zeros;
  p.group_size = S->c.group_size;
  p.a_dtype = SG_DT_F16;
  p.c_dtype = c_dt;
  p.scale_A = 1.0f;
  p.workspace = S->lin_ws;
  p.workspace_bytes = S->lin_ws_bytes;
  p.flags = SG_MM_STATIC_WEIGHTS | flags;  // weights are uploaded once, when the session is created
  SG_TRY(sg_matmul_int4_grouped(&p, S->st), "linear layer");
  return ARMCC_OK;
}

// down(SwiGLU(gate | up)) over M rows: one fused GEMM where the kernels take
// it (few rows), else the SwiGLU kernel and the plain GEMM.
ArmStatus swiglu_down(ArmSession_* S, const Linear& down, void* gu, void* act, void* out, int M, int ffn,
                      uint32_t extra_flags = 0) {
  if (g_fuse_swiglu.load() && M == 1) {
    SgMatMulParams p{};
    p.A = gu;
    p.B = down.qw;
    p.C = out;
    p.M = M;
    p.K = down.K;
    p.N = down.N;
    p.lda = 2 * down.K;
    p.scales_B = down.scales;
    p.zeros_B = down.zeros;
    p.group_size = S->c.group_size;
    p.a_dtype = SG_DT_F16;
    p.c_dtype = SG_DT_F16;
    p.scale_A = 1.0f;
    p.workspace = S->lin_ws;
    p.workspace_bytes = S->lin_ws_bytes;
    p.flags = SG_MM_STATIC_WEIGHTS | SG_MM_A_SWIGLU | extra_flags;
    const SgStatus st = sg_matmul_int4_grouped(&p, S->st);
    if (st == SG_OK) return ARMCC_OK;
    if (st != SG_ERR_UNSUPPORTED) {
      set_err("down projection (SwiGLU fused) failed: %s", sg_last_error());
      return (ArmStatus)st;
    }
  }
  SG_TRY(sg_swiglu_rows(gu, act, M, ffn, SG_DT_F16, S->st), "SwiGLU");
  return linear(S, down, act, out, M, SG_DT_F16);
}

// One forward pass over Ts tokens of each of the session's B sequences, at
// positions pos .. pos+Ts-1 (ids already in the "ids" buffer, sequence-major,
// or the device-resident next tokens when from_next).  With dev_pos (one
// decode token per sequence) the kernels read the position from the "pos"
// buffer instead of launch arguments, so the launches can be captured once.
ArmStatus forward(ArmSession_* S, int Ts, bool from_next, bool dev_pos = false) {
  const ModelCfg& c = S->c;
  cudaStream_t st = S->st;
  const int B = S->batch, T = B * Ts;
  const int H = c.hidden, D = c.head_dim;
  const int32_t* ids = from_next ? S->buf<int32_t>("next") : S->buf<int32_t>("ids");
  // one row on one GPU: norms and residual adds fused into the projections
  // (tensor-parallel: the peer all-reduce adds the row-parallel sums into the residual stream)
  const bool tp_peer = S->tp_world > 1 && S->ar_region && H % 8 == 0 && H <= S->ar_max;
  const bool fuse = T == 1 && (S->tp_world == 1 || tp_peer) && S->norm_fusable && g_fuse_norm.load() != 0;
  void* resid = S->buf<void>("resid");
  if (fuse) {
    // the residual stream starts as the embedding (round(x + 0) = x)
    SG_TRY(sg_embedding(S->embed, ids, resid, T, H, c.vocab_global, SG_DT_F16, st), "embedding");
  } else {
    SG_TRY(sg_embedding(S->embed, ids, S->buf<void>("x_emb"), T, H, c.vocab_global, SG_DT_F16, st), "embedding");
    if (cudaMemsetAsync(resid, 0, (size_t)T * H * 2, st) != cudaSuccess) {
      set_err("cudaMemsetAsync failed");
      return ARMCC_ERR_RUNTIME;
    }
  }
  ArmStatus r;
  for (int l = 0; l < c.layers; ++l) {
    bool appended = false;  // the q|k|v GEMV's epilogue did the rope and the KV append
    if (fuse) {
      if (S->rope_fusable && g_fuse_rope.load()) {
        SgMatMulParams p{};
        p.A = resid;
        p.B = S->qkv[l].qw;
        p.C = S->buf<void>("qkv");
        p.M = 1;
        p.K = S->qkv[l].K;
        p.N = S->qkv[l].N;
        p.scales_B = S->qkv[l].scales;
        p.zeros_B = S->qkv[l].zeros;
        p.group_size = c.group_size;
        p.a_dtype = SG_DT_F16;
        p.c_dtype = SG_DT_F16;
        p.scale_A = 1.0f;
        p.flags = SG_MM_STATIC_WEIGHTS | SG_MM_A_RMSNORM;
        p.norm_weight = S->in_norm[l];
        p.norm_eps = c.rms_eps;
        SgRopeAppend ra{};
        ra.heads = c.heads;
        ra.kv_heads = c.kv_heads;
        ra.head_dim = D;
        ra.positions = dev_pos ? S->buf<int32_t>("pos") : nullptr;
        ra.pos0 = S->pos;
        ra.base = c.rope_theta;
        ra.q_out = S->buf<void>("qh");
        ra.k_cache = S->kcache(l);
        ra.v_cache = S->vcache(l);
        ra.kv_head_stride = S->kv_head_stride;
        ra.kv_pages = S->paged ? &S->kvp[l] : nullptr;
        SG_TRY(sg_qkv_gemv_rope_append(&p, &ra, st), "q|k|v projection with rope and KV append");
        appended = true;
      } else if ((r = linear(S, S->qkv[l], resid, S->buf<void>("qkv"), T, SG_DT_F16, SG_MM_A_RMSNORM,
                             S->in_norm[l])) != ARMCC_OK) {
        return r;
      }
    } else {
      const void* x_in = l == 0 ? S->buf<void>("x_emb") : S->buf<void>("down");
      SG_TRY(sg_rmsnorm(x_in, resid, S->in_norm[l], S->buf<void>("xnorm"), T, H, c.rms_eps, SG_DT_F16, st),
             "input rmsnorm");
      if ((r = linear(S, S->qkv[l], S->buf<void>("xnorm"), S->buf<void>("qkv"), T, SG_DT_F16)) != ARMCC_OK) return r;
    }
    if (appended) {
      // done in the q|k|v projection
    } else if (S->paged) {
      SG_TRY(sg_qkv_rope_append_paged(S->buf<void>("qkv"), B, Ts, c.heads, c.kv_heads, D,
                                      dev_pos ? S->buf<int32_t>("pos") : nullptr, S->pos, c.rope_theta,
                                      S->buf<void>("qh"), S->kcache(l), S->vcache(l), &S->kvp[l], SG_DT_F16, st),
             "rope / KV append");
    } else {
      SG_TRY(sg_qkv_rope_append_batched(S->buf<void>("qkv"), B, Ts, c.heads, c.kv_heads, D,
                                        dev_pos ? S->buf<int32_t>("pos") : nullptr, S->pos, c.rope_theta,
                                        S->buf<void>("qh"), S->kcache(l), S->vcache(l), S->kv_head_stride,
                                        S->kv_bstride(), SG_DT_F16, st),
             "rope / KV append");
    }
    SgFlashAttentionParams a{};
    a.Q = S->buf<void>("qh");
    a.K = S->kcache(l);
    a.V = S->vcache(l);
    a.O = S->buf<void>("attn");
    a.B = B;
    a.S = Ts;
    a.num_heads = c.heads;
    a.num_kv_heads = c.kv_heads;
    a.head_dim = D;
    a.scale = 0.f;
    a.causal = 1;
    a.io_dtype = SG_DT_F16;
    a.S_kv = dev_pos ? c.max_context : S->pos + Ts;
    a.q_pos0 = dev_pos ? 0 : S->pos;
    a.q_pos_device = dev_pos ? S->buf<int32_t>("pos") : nullptr;
    a.kv_head_stride = S->kv_head_stride;
    a.kv_batch_stride = S->kv_bstride();
    a.kv_pages = S->paged ? &S->kvp[l] : nullptr;
    a.workspace = S->attn_ws;
    a.workspace_bytes = S->attn_ws_bytes;
    const void* attn_rows = S->buf<void>("attn");
    if (Ts == 1) {
      SG_TRY(sg_flash_decode(&a, st), "decode attention");  // [B, H, 1, D] = B rows of H * D
    } else {
      SG_TRY(sg_flash_attention(&a, st), "prefill attention");
      const size_t seq = (size_t)c.heads * Ts * D * 2;  // bytes of one sequence's [H, Ts, D]
      for (int b = 0; b < B; ++b)
        SG_TRY(sg_head_transpose(S->buf<char>("attn") + b * seq, S->buf<char>("attn_t") + b * seq, c.heads, Ts, D,
                                 SG_DT_F16, st),
               "head transpose");
      attn_rows = S->buf<void>("attn_t");
    }
    if (fuse) {
      // resid += o; gate|up of the post-attention norm; resid += down(SwiGLU).  Tensor-parallel:
      // the partial sums go through the peer all-reduce, which adds them into resid.
      if (S->tp_world == 1) {
        if ((r = linear(S, S->o[l], attn_rows, resid, T, SG_DT_F16, SG_MM_C_ACCUMULATE)) != ARMCC_OK) return r;
      } else {
        if ((r = linear(S, S->o[l], attn_rows, S->buf<void>("o"), T, SG_DT_F16)) != ARMCC_OK) return r;
        SG_TRY(sg_tp_allreduce_f16_residual(S->buf<void>("o"), H, S->tp_rank, S->tp_world, S->ar_regions.data(),
                                            S->ar_max, resid, st),
               "peer all-reduce into the residual");
      }
      if ((r = linear(S, S->gu[l], resid, S->buf<void>("gu"), T, SG_DT_F16, SG_MM_A_RMSNORM, S->post_norm[l])) !=
          ARMCC_OK)
        return r;
      if (S->tp_world == 1) {
        if ((r = swiglu_down(S, S->down[l], S->buf<void>("gu"), S->buf<void>("act"), resid, T, S->down[l].K,
                             SG_MM_C_ACCUMULATE)) != ARMCC_OK)
          return r;
      } else {
        if ((r = swiglu_down(S, S->down[l], S->buf<void>("gu"), S->buf<void>("act"), S->buf<void>("down"), T,
                             S->down[l].K)) != ARMCC_OK)
          return r;
        SG_TRY(sg_tp_allreduce_f16_residual(S->buf<void>("down"), H, S->tp_rank, S->tp_world, S->ar_regions.data(),
                                            S->ar_max, resid, st),
               "peer all-reduce into the residual");
      }
      continue;
    }
    if ((r = linear(S, S->o[l], attn_rows, S->buf<void>("o"), T, SG_DT_F16)) != ARMCC_OK) return r;
    if ((r = tp_sum(S, S->buf<void>("o"), (size_t)T * H)) != ARMCC_OK) return r;
    SG_TRY(sg_rmsnorm(S->buf<void>("o"), resid, S->post_norm[l], S->buf<void>("xnorm"), T, H, c.rms_eps, SG_DT_F16,
                      st),
           "post-attention rmsnorm");
    if ((r = linear(S, S->gu[l], S->buf<void>("xnorm"), S->buf<void>("gu"), T, SG_DT_F16)) != ARMCC_OK) return r;
    if ((r = swiglu_down(S, S->down[l], S->buf<void>("gu"), S->buf<void>("act"), S->buf<void>("down"), T,
                         S->down[l].K)) != ARMCC_OK)
      return r;
    if ((r = tp_sum(S, S->buf<void>("down"), (size_t)T * H)) != ARMCC_OK) return r;
  }
  // each sequence's last token: final norm, LM head, greedy token
  const void *x_last = S->buf<void>("down"), *r_last = S->buf<void>("resid");
  if (Ts > 1) {
    const size_t row = (size_t)H * 2, pitch = (size_t)Ts * row, off = (size_t)(Ts - 1) * row;
    if (cudaMemcpy2DAsync(S->buf<void>("last_x"), row, S->buf<char>("down") + off, pitch, row, B,
                          cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        cudaMemcpy2DAsync(S->buf<void>("last_r"), row, S->buf<char>("resid") + off, pitch, row, B,
                          cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
      set_err("gathering the last rows failed");
      return ARMCC_ERR_RUNTIME;
    }
    x_last = S->buf<void>("last_x");
    r_last = S->buf<void>("last_r");
  }
  if (fuse && c.lm_int4) {
    // the residual stream already holds h: the final norm is the LM head's activation staging
    if ((r = linear(S, S->lm, resid, S->buf<void>("logits"), B, SG_DT_F32, SG_MM_A_RMSNORM, S->final_norm)) !=
        ARMCC_OK)
      return r;
  } else if (fuse) {
    SG_TRY(sg_rmsnorm(resid, nullptr, S->final_norm, S->buf<void>("last_n"), B, H, c.rms_eps, SG_DT_F16, st),
           "final rmsnorm");
  } else {
    SG_TRY(sg_rmsnorm(x_last, const_cast<void*>(r_last), S->final_norm, S->buf<void>("last_n"), B, H, c.rms_eps,
                      SG_DT_F16, st),
           "final rmsnorm");
  }
  if (fuse && c.lm_int4) {
    // done above
  } else if (c.lm_int4) {
    if ((r = linear(S, S->lm, S->buf<void>("last_n"), S->buf<void>("logits"), B, SG_DT_F32)) != ARMCC_OK) return r;
  } else {
    SgMatMulParams p{};
    p.A = S->buf<void>("last_n");
    p.B = S->lm_f16;
    p.C = S->buf<void>("logits");
    p.M = B;
    p.K = H;
    p.N = c.vocab;
    p.a_dtype = SG_DT_F16;
    p.c_dtype = SG_DT_F32;
    SG_TRY(sg_matmul_fp16(&p, st), "LM head");
  }
  SG_TRY(sg_argmax_logprob(S->buf<float>("logits"), B, c.vocab, S->buf<int32_t>("next"), S->buf<float>("logprob"),
                           st),
         "argmax");
  if (S->tp_world > 1) {
    // every rank's (max, log-sum-exp, index) per sequence, gathered in rank order, then the global pick
    SG_TRY(sg_tp_argmax_pack(S->buf<float>("logits"), B, c.vocab, S->buf<int32_t>("next"), S->buf<float>("logprob"),
                             S->shard.vocab0, S->buf<float>("tp_mine"), st),
           "tensor-parallel argmax");
    const ncclResult_t e = nccl_api().all_gather(S->buf<float>("tp_mine"), S->buf<float>("tp_all"), (size_t)3 * B,
                                                 ncclFloat, S->comm, st);
    if (e != ncclSuccess) {
      set_err("ncclAllGather failed: %s", nccl_api().error_string(e));
      return ARMCC_ERR_RUNTIME;
    }
    SG_TRY(sg_tp_argmax_pick(S->buf<float>("tp_all"), S->tp_world, B, S->buf<int32_t>("next"),
                             S->buf<float>("logprob"), st),
           "tensor-parallel argmax");
  }
  S->pos += Ts;
  return ARMCC_OK;
}

ArmStatus enqueue_results(ArmSession_* S);

// Whether this session's one-token steps run as the persistent decode-step
// kernel: one sequence on one GPU with the norms fused, and a model the kernel
// takes (built here on the first such step, outside any capture).
bool use_step_kernel(ArmSession_* S) {
  if (S->batch != 1 || S->tp_world != 1 || !S->norm_fusable || g_fuse_norm.load() == 0 ||
      g_step_kernel.load() == 0 || !S->c.lm_int4)
    return false;
  if (S->ds || S->ds_tried) return S->ds != nullptr;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(S->st, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return false;  // built on an eager step only (it allocates)
  }
  S->ds_tried = true;
  const ModelCfg& c = S->c;
  sg::DsModel m;
  m.layers = c.layers;
  m.hidden = c.hidden;
  m.heads = c.heads;
  m.kv_heads = c.kv_heads;
  m.head_dim = c.head_dim;
  m.ffn = c.ffn;
  m.vocab = c.vocab;
  m.group_size = c.group_size;
  m.rope_theta = c.rope_theta;
  m.rms_eps = c.rms_eps;
  m.embed = S->embed;
  m.vocab_rows = c.vocab_global;
  m.final_norm = S->final_norm;
  m.in_norm = S->in_norm;
  m.post_norm = S->post_norm;
  auto lin = [](const Linear& L) {
    sg::DsLinear d;
    d.qw = L.qw;
    d.scales = L.scales;
    d.zeros = L.zeros;
    d.K = L.K;
    d.N = L.N;
    return d;
  };
  for (int l = 0; l < c.layers; ++l) {
    m.qkv.push_back(lin(S->qkv[l]));
    m.o.push_back(lin(S->o[l]));
    m.gu.push_back(lin(S->gu[l]));
    m.down.push_back(lin(S->down[l]));
    m.k_cache.push_back(S->kcache(l));
    m.v_cache.push_back(S->vcache(l));
    if (S->paged) m.pages.push_back(S->kvp[l]);
  }
  m.lm = lin(S->lm);
  m.kv_head_stride = S->kv_head_stride;
  m.max_context = c.max_context;
  if (const char* why = sg::decode_step_unsupported(m, S->dev)) {
    S->ds_why = why;
    return false;
  }
  if (sg::decode_step_create(m, S->dev, &S->ds) != SG_OK) {
    S->ds_why = sg_last_error();
    S->ds = nullptr;
    return false;
  }
  return true;
}

// One decode token through the captured graph (captured on the second step,
// after an eager step has done every first-use allocation and attribute call).
// The graph holds the whole step: the position from the pinned host word, the
// forward pass and the copies of the results into the pinned result block.
ArmStatus decode_step_inner(ArmSession_* S);

// A decode step, bracketed by the timing events when they are on.
ArmStatus decode_step(ArmSession_* S) {
  const bool timed = S->ev_step[0] != nullptr;
  if (timed) cudaEventRecord(S->ev_step[0], S->st);
  const ArmStatus r = decode_step_inner(S);
  if (timed && r == ARMCC_OK) {
    cudaEventRecord(S->ev_step[1], S->st);
    S->ev_pending = true;
  }
  return r;
}

ArmStatus decode_step_inner(ArmSession_* S) {
  *S->h_pos = S->pos;
  if (S->use_graph && S->graph_exec) {
    if (cudaGraphLaunch(S->graph_exec, S->st) != cudaSuccess) {
      set_err("cudaGraphLaunch failed: %s", cudaGetErrorString(cudaGetLastError()));
      return ARMCC_ERR_RUNTIME;
    }
    S->pos += 1;
    return ARMCC_OK;
  }
  auto whole_step = [&]() -> ArmStatus {
    if (cudaMemcpyAsync(S->buf<int32_t>("pos"), S->h_pos, 4, cudaMemcpyHostToDevice, S->st) != cudaSuccess) {
      set_err("copying the position failed");
      return ARMCC_ERR_RUNTIME;
    }
    if (use_step_kernel(S)) {
      SG_TRY(sg::decode_step_run(S->ds, S->buf<int32_t>("pos"), S->buf<int32_t>("next"), S->buf<float>("logprob"),
                                 S->buf<float>("logits"), S->st),
             "decode step kernel");
      S->pos += 1;
      return enqueue_results(S);
    }
    const ArmStatus r = forward(S, 1, true, true);
    return r == ARMCC_OK ? enqueue_results(S) : r;
  };
  if (S->use_graph && !S->graph_failed && S->eager_steps > 0) {
    const int pos_before = S->pos;
    if (cudaStreamBeginCapture(S->st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
      const ArmStatus r = whole_step();
      cudaGraph_t g = nullptr;
      const cudaError_t e = cudaStreamEndCapture(S->st, &g);
      cudaGraphExec_t x = nullptr;
      if (r == ARMCC_OK && e == cudaSuccess && g && cudaGraphInstantiate(&x, g, 0) == cudaSuccess) {
        S->graph = g;
        S->graph_exec = x;
        S->graph_err_word = sg::existing_device_error_word(S->dev);
        if (cudaGraphLaunch(x, S->st) != cudaSuccess) {
          set_err("cudaGraphLaunch failed: %s", cudaGetErrorString(cudaGetLastError()));
          return ARMCC_ERR_RUNTIME;
        }
        return ARMCC_OK;  // forward() advanced pos
      }
      if (g) cudaGraphDestroy(g);
    }
    cudaGetLastError();
    S->graph_failed = true;  // run eagerly from now on
    S->pos = pos_before;
  }
  const ArmStatus r = whole_step();
  if (r == ARMCC_OK) S->eager_steps += 1;
  return r;
}

// Paged cache: makes sure every sequence has pages for positions < upto in
// every layer, taking them from the pool; the new table rows go to the
// device in stream order (one contiguous copy: the table is [logical page]
// [layer][sequence]).  ARMCC_ERR_OOM when the pool is exhausted.
ArmStatus ensure_pages(ArmSession_* S, int upto, const char* fn) {
  if (!S->paged) return ARMCC_OK;
  const int need = (upto + 15) / 16;
  if (need <= S->lpages) return ARMCC_OK;
  const int L = S->c.layers, B = S->batch;
  if (need > S->max_lpages) {
    set_err("%s: position %d is past the page table (%d pages of 16 tokens)", fn, upto, S->max_lpages);
    return ARMCC_ERR_OOM;
  }
  const size_t count = (size_t)(need - S->lpages) * L * B;
  if (S->free_pages.size() < count) {
    set_err("%s: the KV page pool (%d pages of 16 tokens) cannot hold position %d of %d sequences", fn,
            S->pool_pages, upto, B);
    return ARMCC_ERR_OOM;
  }
  const size_t first = (size_t)S->lpages * L * B;
  for (size_t i = first; i < first + count; ++i) {
    S->h_table[i] = S->free_pages.back();
    S->free_pages.pop_back();
  }
  // from pageable memory: staged before the call returns, so the host copy may change afterwards
  if (cudaMemcpyAsync(S->d_table + first, S->h_table.data() + first, count * 4, cudaMemcpyHostToDevice, S->st) !=
      cudaSuccess) {
    set_err("%s: updating the KV page table failed", fn);
    return ARMCC_ERR_RUNTIME;
  }
  S->lpages = need;
  return ARMCC_OK;
}

// Returns every page to the pool (reset): the next positions start from page 0 again.
void release_pages(ArmSession_* S) {
  if (!S->paged) return;
  S->free_pages.clear();
  for (int pg = S->pool_pages - 1; pg >= 0; --pg) S->free_pages.push_back(pg);
  S->lpages = 0;
}

// Ends a tensor-parallel session's group after a failure: the NCCL
// communicator is aborted (which makes its kernels in flight return), the
// session's own kernels finish (their waits are bounded), and the peers'
// mapped regions are closed.  Every later call is refused with `why`; this
// mirrors the reference runtime's clean refusal with a reason
// (compiler/lib/runtime/resource_controller.cpp:195-247).
// in_flight: a step may still be running on the stream (a collective that did
// not complete); then nothing here waits for it and the peers' mappings stay
// open until the stream drains (the destructor's bounded wait).
void abort_session(ArmSession_* S, const std::string& why, bool in_flight) {
  if (S->aborted) return;
  S->aborted = true;
  S->abort_why = why;
  if (S->comm) {
    if (nccl_api().comm_abort) nccl_api().comm_abort(S->comm);
    S->comm = nullptr;  // aborted: not destroyed again
  }
  if (in_flight) return;
  cudaStreamSynchronize(S->st);
  cudaGetLastError();
  for (size_t q = 0; q < S->ar_regions.size(); ++q)
    if ((int)q != S->tp_rank && S->ar_regions[q]) cudaIpcCloseMemHandle(S->ar_regions[q]);
  S->ar_regions.clear();
}

// Waits for the session's stream.  A tensor-parallel session polls instead of
// blocking: an asynchronous NCCL error, or no completion within
// tp_timeout_ms (a peer that stopped answering), aborts the group and returns
// ARMCC_ERR_RUNTIME instead of hanging the caller.
ArmStatus wait_stream(ArmSession_* S, const char* fn) {
  if (S->tp_world == 1 || !S->comm) {
    if (cudaStreamSynchronize(S->st) != cudaSuccess) {
      set_err("%s: device error: %s", fn, cudaGetErrorString(cudaGetLastError()));
      return ARMCC_ERR_RUNTIME;
    }
    return ARMCC_OK;
  }
  const auto t0 = std::chrono::steady_clock::now();
  for (int spin = 0;; ++spin) {
    const cudaError_t q = cudaStreamQuery(S->st);
    if (q == cudaSuccess) return ARMCC_OK;
    if (q != cudaErrorNotReady) {
      cudaGetLastError();
      set_err("%s: device error: %s", fn, cudaGetErrorString(q));
      return ARMCC_ERR_RUNTIME;
    }
    ncclResult_t ae = ncclSuccess;
    if (nccl_api().comm_get_async_error && nccl_api().comm_get_async_error(S->comm, &ae) == ncclSuccess &&
        ae != ncclSuccess && ae != ncclInProgress) {
      const std::string why = std::string("NCCL reported an asynchronous error: ") + nccl_api().error_string(ae);
      abort_session(S, why, true);
      set_err("%s: %s; the tensor-parallel group was aborted", fn, why.c_str());
      return ARMCC_ERR_RUNTIME;
    }
    const auto ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (ms > S->tp_timeout_ms) {
      char buf[160];
      snprintf(buf, sizeof buf, "a step did not complete within %d ms (a rank stopped answering)",
               S->tp_timeout_ms);
      abort_session(S, buf, true);
      set_err("%s: %s; the tensor-parallel group was aborted", fn, buf);
      return ARMCC_ERR_RUNTIME;
    }
    if (spin > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// Refuses a call on a session whose group failed.
bool session_usable(ArmSession_* S, const char* fn) {
  if (!S->aborted) return true;
  set_err("%s: the session was aborted: %s", fn, S->abort_why.c_str());
  return false;
}

// Queues the copies of every sequence's greedy token, the log-probability and
// the library's device error word into the pinned result block (inside the
// decode graph for a captured step, so a step costs one launch and one wait).
ArmStatus enqueue_results(ArmSession_* S) {
  const int B = S->batch;
  int* derr = sg::existing_device_error_word(S->dev);
  if (cudaMemcpyAsync(S->h_res, S->buf<int32_t>("next"), (size_t)B * 4, cudaMemcpyDeviceToHost, S->st) !=
          cudaSuccess ||
      cudaMemcpyAsync(S->h_res + B, S->buf<float>("logprob"), 4, cudaMemcpyDeviceToHost, S->st) != cudaSuccess ||
      (derr && cudaMemcpyAsync(S->h_res + B + 1, derr, 4, cudaMemcpyDeviceToHost, S->st) != cudaSuccess)) {
    set_err("device error: %s", cudaGetErrorString(cudaGetLastError()));
    return ARMCC_ERR_RUNTIME;
  }
  if (!derr) S->h_res[B + 1] = 0;
  return ARMCC_OK;
}

// Waits for the step and takes every sequence's greedy token from the pinned
// result block; enqueued: the step already queued the copies (enqueue_results).
// A nonzero device error word is read and cleared through sg_device_error_check.
ArmStatus fetch_next(ArmSession_* S, bool enqueued = false) {
  const int B = S->batch;
  if (!enqueued) {
    const ArmStatus e = enqueue_results(S);
    if (e != ARMCC_OK) return e;
  }
  const ArmStatus ws = wait_stream(S, "decode");
  if (ws != ARMCC_OK) return ws;
  // a graph captured before the error word existed does not copy it: read it directly
  const bool direct = S->graph_exec && !S->graph_err_word && sg::existing_device_error_word(S->dev);
  if (direct && sg_device_error_check(S->st) != 0) {
    set_err("a kernel reported a device error (%s)", sg_last_error());
    return ARMCC_ERR_RUNTIME;
  }
  if (S->h_res[B + 1] != 0) {
    const int32_t derr = sg_device_error_check(S->st);
    set_err("a kernel reported device error %d (%s)", S->h_res[B + 1], derr != 0 ? sg_last_error() : "");
    return ARMCC_ERR_RUNTIME;
  }
  if (S->ev_pending) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, S->ev_step[0], S->ev_step[1]) == cudaSuccess) {
      S->step_gpu_ms += ms;
      S->step_gpu_n += 1;
    }
    cudaGetLastError();
    S->ev_pending = false;
  }
  S->next_all.assign(S->h_res, S->h_res + B);
  float lp = 0;
  memcpy(&lp, S->h_res + B, 4);
  S->next_host = S->next_all[0];
  S->logprob_host = lp;
  return ARMCC_OK;
}

// Prefill of n tokens per sequence (tokens sequence-major: sequence b's
// token i at tokens[b * n + i]), in chunks of at most max_chunk per sequence.
ArmStatus prefill_tokens(ArmSession_* S, const int32_t* tokens, uint32_t n, const char* fn) {
  const ModelCfg& c = S->c;
  if (!session_usable(S, fn)) return ARMCC_ERR_RUNTIME;
  if ((uint64_t)S->pos + n > (uint64_t)c.max_context) {
    set_err("%s: %u tokens after %d exceed the context of %d", fn, n, S->pos, c.max_context);
    return ARMCC_ERR_OOM;
  }
  for (uint64_t i = 0; i < (uint64_t)n * S->batch; ++i)
    if (tokens[i] < 0 || tokens[i] >= c.vocab_global) {
      set_err("%s: token %d at %llu is outside the vocabulary", fn, tokens[i], (unsigned long long)i);
      return ARMCC_ERR_RUNTIME;
    }
  if (cudaSetDevice(S->dev) != cudaSuccess) {
    set_err("%s: cannot use device %d", fn, S->dev);
    return ARMCC_ERR_RUNTIME;
  }
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<int32_t> chunk;
  for (uint32_t done = 0; done < n;) {
    const int T = (int)std::min<uint32_t>(n - done, (uint32_t)c.max_chunk);
    const int32_t* src = tokens + done;
    if (S->batch > 1) {  // gather this chunk of every sequence
      chunk.resize((size_t)S->batch * T);
      for (int b = 0; b < S->batch; ++b)
        memcpy(chunk.data() + (size_t)b * T, tokens + (size_t)b * n + done, (size_t)T * 4);
      src = chunk.data();
    }
    if (cudaMemcpyAsync(S->buf<int32_t>("ids"), src, (size_t)S->batch * T * 4, cudaMemcpyHostToDevice, S->st) !=
            cudaSuccess ||
        (S->batch > 1 && cudaStreamSynchronize(S->st) != cudaSuccess)) {  // the gather buffer is reused
      set_err("%s: copying token ids failed", fn);
      return ARMCC_ERR_RUNTIME;
    }
    ArmStatus r = ensure_pages(S, S->pos + T, fn);
    if (r == ARMCC_OK) r = forward(S, T, false);
    if (r != ARMCC_OK) return r;
    done += T;
  }
  const ArmStatus r = fetch_next(S);
  if (r != ARMCC_OK) return r;
  S->emitted = false;
  S->t_prefill_start = t0;
  S->ttft_pending = true;
  return ARMCC_OK;
}

// Emits the pending greedy tokens, running one decode step first when the
// previous ones were already emitted.
ArmStatus step_tokens(ArmSession_* S, const char* fn, float* step_ms) {
  if (!session_usable(S, fn)) return ARMCC_ERR_RUNTIME;
  if (S->pos == 0) {
    set_err("%s: prefill a prompt first", fn);
    return ARMCC_ERR_RUNTIME;
  }
  cudaSetDevice(S->dev);
  const auto t0 = std::chrono::steady_clock::now();
  if (S->emitted) {
    // feed the last emitted tokens (still on the device) and predict the next ones
    if (S->pos + 1 > S->c.max_context) {
      set_err("%s: the context of %d tokens is full", fn, S->c.max_context);
      return ARMCC_ERR_OOM;
    }
    ArmStatus r = ensure_pages(S, S->pos + 1, fn);
    if (r == ARMCC_OK) r = decode_step(S);
    if (r == ARMCC_OK) r = fetch_next(S, true);
    if (r != ARMCC_OK) return r;
  }
  const auto t1 = std::chrono::steady_clock::now();
  S->emitted = true;
  S->generated += 1;
  *step_ms = std::chrono::duration<float, std::milli>(t1 - t0).count();
  if (S->ttft_pending) {
    S->ttft_ms = std::chrono::duration<float, std::milli>(t1 - S->t_prefill_start).count();
    S->ttft_pending = false;
  } else {
    S->tpot_ms = S->generated > 1 ? (S->tpot_ms * (S->generated - 2) + *step_ms) / (S->generated - 1) : *step_ms;
  }
  return ARMCC_OK;
}

bool bind_linear(ArmGraph_* g, const std::string& name, char* wbase, int K, int N, Linear* out, std::string* why) {
  auto find = [&](const std::string& n) -> const TensorRef* {
    auto it = g->tensors.find(n);
    return it == g->tensors.end() ? nullptr : &it->second;
  };
  const TensorRef* q = find(name + ".qweight");
  const TensorRef* s = find(name + ".scales");
  const TensorRef* z = find(name + ".zeros");
  const int gs = g->cfg.group_size;
  const uint64_t G = (uint64_t)(K + gs - 1) / gs;
  if (!q || !s || q->bytes != (uint64_t)((K + 1) / 2) * N || s->bytes != G * N * 2) {
    *why = "tensor " + name + " missing or of the wrong size";
    return false;
  }
  if (g->cfg.zeros && (!z || z->bytes != G * N)) {
    *why = "tensor " + name + ".zeros missing or of the wrong size";
    return false;
  }
  out->qw = reinterpret_cast<const uint8_t*>(wbase + q->offset);
  out->scales = wbase + s->offset;
  out->zeros = g->cfg.zeros ? reinterpret_cast<const int8_t*>(wbase + z->offset) : nullptr;
  out->K = K;
  out->N = N;
  return true;
}

// One rank's cut of a linear in the reference INT4 layout: input rows
// [r0, r1) (on quantisation-group boundaries) and the listed output column
// ranges, packed side by side.  With dry only the space is reserved.
struct ColRange {
  int c0, c1;
};

bool shard_linear(ArmGraph_* g, const std::string& name, int K, int N, int r0, int r1,
                  std::initializer_list<ColRange> cols, const char* full, char* wbase, uint64_t* cursor, bool dry,
                  cudaStream_t st, Linear* out, std::string* why) {
  Linear whole;
  if (!bind_linear(g, name, const_cast<char*>(full), K, N, &whole, why)) return false;
  const int gs = g->cfg.group_size;
  const int Kl = r1 - r0;
  int Nl = 0;
  for (const ColRange& c : cols) Nl += c.c1 - c.c0;
  const uint64_t KPl = (uint64_t)(Kl + 1) / 2, Gl = (uint64_t)(Kl + gs - 1) / gs;
  const uint64_t p0 = (uint64_t)r0 / 2, g0 = (uint64_t)r0 / gs;
  const uint64_t offB = *cursor;
  *cursor = align_up(*cursor + KPl * Nl, 256);
  const uint64_t offS = *cursor;
  *cursor = align_up(*cursor + Gl * Nl * 2, 256);
  uint64_t offZ = 0;
  if (whole.zeros) {
    offZ = *cursor;
    *cursor = align_up(*cursor + Gl * Nl, 256);
  }
  out->qw = reinterpret_cast<const uint8_t*>(wbase + offB);
  out->scales = wbase + offS;
  out->zeros = whole.zeros ? reinterpret_cast<const int8_t*>(wbase + offZ) : nullptr;
  out->K = Kl;
  out->N = Nl;
  if (dry) return true;
  const char* qsrc = reinterpret_cast<const char*>(whole.qw);
  const char* ssrc = static_cast<const char*>(whole.scales);
  const char* zsrc = reinterpret_cast<const char*>(whole.zeros);
  uint64_t dc = 0;
  for (const ColRange& c : cols) {
    const size_t w = (size_t)(c.c1 - c.c0);
    if (cudaMemcpy2DAsync(wbase + offB + dc, Nl, qsrc + p0 * N + c.c0, N, w, KPl, cudaMemcpyDeviceToDevice, st) !=
            cudaSuccess ||
        cudaMemcpy2DAsync(wbase + offS + dc * 2, (size_t)Nl * 2, ssrc + (g0 * N + c.c0) * 2, (size_t)N * 2, w * 2, Gl,
                          cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        (zsrc && cudaMemcpy2DAsync(wbase + offZ + dc, Nl, zsrc + g0 * N + c.c0, N, w, Gl, cudaMemcpyDeviceToDevice,
                                   st) != cudaSuccess)) {
      cudaGetLastError();
      *why = "copying the shard of " + name + " failed";
      return false;
    }
    dc += w;
  }
  return true;
}

// Maps every rank's peer all-reduce region into this process (CUDA IPC
// handles exchanged with one NCCL all-gather).  Collective and symmetric: if
// any rank cannot set it up (or SG_TP_P2P=0 on any rank), every rank keeps
// NCCL for all sums.  Returns false only when a collective itself failed.
bool setup_peer_allreduce(ArmSession_* S, int max_n) {
  const int world = S->tp_world, rank = S->tp_rank;
  const char* env = getenv("SG_TP_P2P");
  bool ok = world <= 8 && !(env && atoi(env) == 0);
  const size_t bytes = sg_tp_allreduce_region_bytes(world, max_n);
  cudaIpcMemHandle_t mine{};
  if (ok) ok = bytes > 0 && cudaMalloc(&S->ar_region, bytes) == cudaSuccess;
  if (ok) ok = cudaMemset(S->ar_region, 0, bytes) == cudaSuccess && cudaIpcGetMemHandle(&mine, S->ar_region) == cudaSuccess;
  if (!ok) cudaGetLastError();
  // [world][handle | status] on the device, gathered in place
  struct Slot {
    cudaIpcMemHandle_t h;
    int32_t ok;
    int32_t pad[3];
  };
  Slot* dslots = nullptr;
  std::vector<Slot> slots(world);
  slots[rank].h = mine;
  slots[rank].ok = ok ? 1 : 0;
  if (cudaMalloc(&dslots, sizeof(Slot) * world) != cudaSuccess ||
      cudaMemcpy(dslots + rank, &slots[rank], sizeof(Slot), cudaMemcpyHostToDevice) != cudaSuccess ||
      nccl_api().all_gather(dslots + rank, dslots, sizeof(Slot), ncclChar, S->comm, S->st) != ncclSuccess ||
      cudaMemcpyAsync(slots.data(), dslots, sizeof(Slot) * world, cudaMemcpyDeviceToHost, S->st) != cudaSuccess ||
      cudaStreamSynchronize(S->st) != cudaSuccess) {
    cudaGetLastError();
    if (dslots) cudaFree(dslots);
    return false;
  }
  cudaFree(dslots);
  bool all = true;
  for (const Slot& x : slots) all = all && x.ok;
  S->ar_regions.assign(world, nullptr);
  int opened = 1;
  if (all) {
    S->ar_regions[rank] = S->ar_region;
    for (int q = 0; q < world && opened; ++q) {
      if (q == rank) continue;
      if (cudaIpcOpenMemHandle(&S->ar_regions[q], slots[q].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        S->ar_regions[q] = nullptr;
        opened = 0;
      }
    }
  }
  // every rank learns whether every rank mapped every peer
  int bad = (all && opened) ? 0 : 1;
  if (cudaMemcpyAsync(S->tp_flag, &bad, 4, cudaMemcpyHostToDevice, S->st) != cudaSuccess ||
      nccl_api().all_reduce(S->tp_flag, S->tp_flag, 1, ncclInt32, ncclMax, S->comm, S->st) != ncclSuccess ||
      cudaMemcpyAsync(&bad, S->tp_flag, 4, cudaMemcpyDeviceToHost, S->st) != cudaSuccess ||
      cudaStreamSynchronize(S->st) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (bad) {  // NCCL for every sum on every rank
    for (int q = 0; q < world; ++q)
      if (q != rank && S->ar_regions[q]) cudaIpcCloseMemHandle(S->ar_regions[q]);
    S->ar_regions.clear();
    if (S->ar_region) cudaFree(S->ar_region);
    S->ar_region = nullptr;
    return true;
  }
  S->ar_max = max_n;
  return true;
}

// Session of rank `rank` in a group of `world` (world 1: the whole model, no NCCL).
// KV cache layout of a session: flat [sequence][layer][K|V][kv_head][seq][dim]
// (kv_cache_layout.cpp:16-53), or paged (:65-102) -- the reference's rule
// (recommendKVCacheLayout, :107-130) pages contexts above 4096 tokens, in
// pages of 16 tokens.  kv_mode: 0 that rule, 1 flat, 2 paged; SG_KV_LAYOUT=
// flat|paged overrides the rule.  pool_tokens: tokens the paged pool holds
// over all sequences (0 = every sequence's full context).
struct KvLayout {
  bool paged = false;
  int max_lpages = 0, pool_pages = 0;
  uint64_t pool_bytes = 0, table_bytes = 0;  // paged
  uint64_t bytes = 0;                          // the KV region of the slab (pool + table, or the flat cache)
};

KvLayout kv_layout(const ModelCfg& c, int batch, int kv_mode, int64_t pool_tokens) {
  KvLayout k;
  k.paged = kv_mode == 2 || (kv_mode == 0 && c.max_context > 4096);
  if (kv_mode == 0) {
    if (const char* e = getenv("SG_KV_LAYOUT")) {
      if (!strcmp(e, "flat")) k.paged = false;
      else if (!strcmp(e, "paged")) k.paged = true;
    }
  }
  if (!k.paged) {
    k.bytes = (uint64_t)batch * c.layers * 2 * (uint64_t)c.kv_heads * c.max_context * c.head_dim * 2;
    return k;
  }
  k.max_lpages = (c.max_context + 15) / 16;
  const int64_t lp_pool = pool_tokens > 0 ? (pool_tokens + 15) / 16 : (int64_t)batch * k.max_lpages;
  k.pool_pages = (int)std::min<int64_t>(lp_pool * c.layers, INT32_MAX);
  k.pool_bytes = (uint64_t)k.pool_pages * 2 * c.kv_heads * 16 * c.head_dim * 2;
  k.table_bytes = align_up((uint64_t)k.max_lpages * c.layers * batch * 4, 256);
  k.bytes = align_up(k.pool_bytes, 4096) + k.table_bytes;
  return k;
}

// Scratch of the linear kernels (largest over the shapes and token counts a
// session of `batch` sequences uses) and of the attention kernels.
void session_scratch(const ModelCfg& c, int batch, size_t* lws_out, size_t* aws_out) {
  const int T = c.max_chunk;
  SgMatMulParams mp{};
  auto lin_ws = [&](int M, int K, int N, int cdt) {
    mp = SgMatMulParams{};
    mp.A = mp.B = mp.scales_B = reinterpret_cast<void*>(256);
    mp.C = reinterpret_cast<void*>(256);
    mp.M = M;
    mp.K = K;
    mp.N = N;
    mp.group_size = c.group_size;
    mp.a_dtype = SG_DT_F16;
    mp.c_dtype = cdt;
    return sg_matmul_int4_grouped_workspace_size(&mp);
  };
  size_t lws = 0;
  // every token count a call can see: the row kernels' scratch depends on M
  // below the tensor-core GEMM's threshold
  const int TB = T * batch;  // rows of the largest forward pass
  for (int M = 1; M <= TB; M = (M < 64 ? M + 1 : (M == TB ? TB + 1 : std::min(2 * M, TB)))) {
    lws = std::max({lws, lin_ws(M, c.hidden, c.nqkv(), SG_DT_F16), lin_ws(M, c.heads * c.head_dim, c.hidden, SG_DT_F16),
                    lin_ws(M, c.hidden, 2 * c.ffn, SG_DT_F16), lin_ws(M, c.ffn, c.hidden, SG_DT_F16)});
  }
  lws = std::max(lws, lin_ws(batch, c.hidden, c.vocab, SG_DT_F32));
  SgFlashAttentionParams ap{};
  ap.Q = ap.K = ap.V = ap.O = reinterpret_cast<void*>(256);
  ap.B = batch;
  ap.num_heads = c.heads;
  ap.num_kv_heads = c.kv_heads;
  ap.head_dim = c.head_dim;
  ap.causal = 1;
  ap.io_dtype = SG_DT_F16;
  ap.S = 1;
  ap.S_kv = c.max_context;
  ap.q_pos0 = c.max_context - 1;
  size_t aws = sg_flash_decode_workspace_size(&ap);
  ap.S = T;
  ap.q_pos0 = c.max_context - T;
  aws = std::max(aws, sg_flash_attention_workspace_size(&ap));

  *lws_out = lws;
  *aws_out = aws;
}

// The norms (and the rope + KV append) fuse into the projections when the
// one-row kernel takes every shape of this session (its shards when
// tensor-parallel).
void decide_fusion(ArmSession_* S) {
  const ModelCfg& c = S->c;
  {
    const int sms = sg::sm_count(S->dev);
    bool ok = c.hidden % 8 == 0 && c.hidden <= 8192;
    auto takes = [&](const Linear& L, int cdt) {
      SgMatMulParams p{};
      p.A = p.C = S->act;
      p.B = L.qw;
      p.scales_B = L.scales;
      p.zeros_B = L.zeros;
      p.M = 1;
      p.K = L.K;
      p.N = L.N;
      p.group_size = c.group_size;
      p.a_dtype = SG_DT_F16;
      p.c_dtype = cdt;
      bool applicable = false;
      const size_t ws = sg::w4_gemv_mma_scratch_bytes(&p, sms, &applicable);
      return applicable ? (ws == 0 ? 2 : 1) : 0;  // 2: a cluster split (no scratch)
    };
    bool cluster_qkv = c.head_dim == 64 || c.head_dim == 128;
    for (int l = 0; ok && l < c.layers; ++l) {
      const int q = takes(S->qkv[l], SG_DT_F16);
      cluster_qkv = cluster_qkv && q == 2;
      ok = q && takes(S->o[l], SG_DT_F16) && takes(S->gu[l], SG_DT_F16) && takes(S->down[l], SG_DT_F16);
    }
    if (ok && c.lm_int4) ok = takes(S->lm, SG_DT_F32) != 0;
    S->norm_fusable = ok;
    S->rope_fusable = ok && cluster_qkv;
  }
}

ArmSession* create_session(ArmGraph* graph, const ArmSessionOptions* opts, int rank, int world, const uint8_t* id,
                           int batch, int kv_mode = 0, int64_t pool_tokens = 0) {
  const char* fn = world > 1 ? "sg_session_create_tp" : "armgraph_create_session";
  if (!graph) {
    set_err("%s: graph is NULL", fn);
    return nullptr;
  }
  if (!graph->runnable) {
    set_err("%s: %s", fn, graph->why_not.c_str());
    return nullptr;
  }
  if (opts && !opts->use_gpu) {
    set_err("%s: use_gpu is false, but this library only runs on the GPU", fn);
    return nullptr;
  }
  if (batch < 1 || batch > 1024) {
    set_err("%s: batch %d outside [1, 1024]", fn, batch);
    return nullptr;
  }
  auto S = std::make_unique<ArmSession_>();
  S->g = graph;
  S->c = graph->cfg;
  S->tp_rank = rank;
  S->tp_world = world;
  S->batch = batch;
  const ModelCfg& gc = graph->cfg;
  std::string why;
  if (world > 1) {
    if (!gc.lm_int4) {
      set_err("%s: tensor parallelism needs an INT4 LM head", fn);
      return nullptr;
    }
    if (world > 64) {
      set_err("%s: at most 64 ranks", fn);
      return nullptr;
    }
    const SgTpModel m{gc.hidden, gc.heads, gc.kv_heads, gc.head_dim, gc.ffn, gc.vocab, gc.group_size};
    if (!tp_plan(m, rank, world, &S->shard, &why)) {
      set_err("%s: %s", fn, why.c_str());
      return nullptr;
    }
    if (!nccl_api().ok) {
      set_err("%s: %s", fn, nccl_api().why.c_str());
      return nullptr;
    }
    S->c.heads = S->shard.q_head1 - S->shard.q_head0;
    S->c.kv_heads = S->shard.kv_head1 - S->shard.kv_head0;
    S->c.ffn = S->shard.ffn1 - S->shard.ffn0;
    S->c.vocab = S->shard.vocab1 - S->shard.vocab0;
  } else {
    S->shard = SgTpShard{0, gc.heads, 0, gc.kv_heads, 0, gc.ffn, 0, gc.vocab};
  }
  const ModelCfg& c = S->c;
  if (const char* d = getenv("SG_DEVICE")) S->dev = atoi(d);
  else if (cudaGetDevice(&S->dev) != cudaSuccess) S->dev = 0;
  if (cudaSetDevice(S->dev) != cudaSuccess) {
    cudaGetLastError();
    set_err("%s: cannot use CUDA device %d", fn, S->dev);
    return nullptr;
  }
  if (cudaStreamCreateWithFlags(&S->st, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMallocHost(&S->h_pos, sizeof(int32_t)) != cudaSuccess ||
      cudaMallocHost(&S->h_res, sizeof(int32_t) * ((size_t)S->batch + 2)) != cudaSuccess) {
    cudaGetLastError();
    set_err("%s: cannot create the session's stream", fn);
    return nullptr;
  }
  if (const char* gflag = getenv("SG_DECODE_GRAPH")) S->use_graph = atoi(gflag) != 0;
  if (const char* t = getenv("SG_TP_TIMEOUT_MS")) S->tp_timeout_ms = std::max(1, atoi(t));
  if (world > 1) {
    ncclUniqueId uid;
    memcpy(uid.internal, id, sizeof uid.internal);
    if (cudaMalloc(&S->tp_flag, 256) != cudaSuccess) {
      cudaGetLastError();
      set_err("%s: cannot allocate device memory", fn);
      return nullptr;
    }
    const ncclResult_t e = nccl_api().comm_init_rank(&S->comm, world, uid, rank);
    if (e != ncclSuccess) {
      S->comm = nullptr;
      set_err("%s: ncclCommInitRank failed: %s", fn, nccl_api().error_string(e));
      return nullptr;
    }
    if (!setup_peer_allreduce(S.get(), (int)align_up((uint64_t)batch * gc.hidden, 8))) {
      set_err("%s: a collective of the peer all-reduce setup failed", fn);
      return nullptr;
    }
  }
  // weight file
  const uint8_t* wdata = nullptr;
  uint64_t wbytes = 0;
  std::string err;
  if (!graph->pkg->box.map_entry(graph->weight_path, &wdata, &wbytes, &err)) {
    set_err("%s: %s", fn, err.c_str());
    return nullptr;
  }
  for (auto& kv : graph->tensors)
    if (kv.second.offset + kv.second.bytes > wbytes) {
      set_err("%s: tensor %s lies outside the weight file", fn, kv.first.c_str());
      return nullptr;
    }
  // scratch sizes of the linear kernels (largest over the shapes and token counts used)
  const int T = c.max_chunk;
  size_t lws = 0, aws = 0;
  session_scratch(c, batch, &lws, &aws);

  // weights: the whole file (one rank), or this rank's shards (several)
  const SgTpShard& sh = S->shard;
  const int H = gc.hidden, D = gc.head_dim, Hq = gc.heads, Hkv = gc.kv_heads, F = gc.ffn;
  const uint64_t H2 = (uint64_t)H * 2;
  auto find = [&](const std::string& n, uint64_t expect) -> const TensorRef* {
    auto it = graph->tensors.find(n);
    return (it == graph->tensors.end() || it->second.bytes != expect) ? nullptr : &it->second;
  };
  // Places (dry: sizes only) the replicated tensors and every linear shard at
  // offsets from wbase; returns the bytes used or 0 with `why` set.
  auto place = [&](const char* full, char* wbase, bool dry) -> uint64_t {
    uint64_t cur = 0;
    auto replicate = [&](const std::string& n, uint64_t bytes, const void** dst) -> bool {
      const TensorRef* r = find(n, bytes);
      if (!r) {
        why = "tensor " + n + " missing or of the wrong size";
        return false;
      }
      const uint64_t off = cur;
      cur = align_up(cur + bytes, 256);
      *dst = wbase + off;
      if (!dry && cudaMemcpyAsync(wbase + off, full + r->offset, bytes, cudaMemcpyDeviceToDevice, S->st) != cudaSuccess) {
        cudaGetLastError();
        why = "copying " + n + " failed";
        return false;
      }
      return true;
    };
    S->in_norm.assign(gc.layers, nullptr);
    S->post_norm.assign(gc.layers, nullptr);
    S->qkv.assign(gc.layers, Linear{});
    S->o.assign(gc.layers, Linear{});
    S->gu.assign(gc.layers, Linear{});
    S->down.assign(gc.layers, Linear{});
    if (!replicate("embed_tokens", (uint64_t)gc.vocab_global * H2, &S->embed) ||
        !replicate("final_norm", H2, &S->final_norm))
      return 0;
    for (int l = 0; l < gc.layers; ++l) {
      const std::string p = "layers." + std::to_string(l) + ".";
      if (!replicate(p + "input_norm", H2, &S->in_norm[l]) || !replicate(p + "post_norm", H2, &S->post_norm[l]))
        return 0;
      const int nq = gc.nqkv();
      if (!shard_linear(graph, p + "qkv", H, nq, 0, H,
                        {{sh.q_head0 * D, sh.q_head1 * D},
                         {(Hq + sh.kv_head0) * D, (Hq + sh.kv_head1) * D},
                         {(Hq + Hkv + sh.kv_head0) * D, (Hq + Hkv + sh.kv_head1) * D}},
                        full, wbase, &cur, dry, S->st, &S->qkv[l], &why) ||
          !shard_linear(graph, p + "o", Hq * D, H, sh.q_head0 * D, sh.q_head1 * D, {{0, H}}, full, wbase, &cur, dry,
                        S->st, &S->o[l], &why) ||
          !shard_linear(graph, p + "gate_up", H, 2 * F, 0, H, {{sh.ffn0, sh.ffn1}, {F + sh.ffn0, F + sh.ffn1}}, full,
                        wbase, &cur, dry, S->st, &S->gu[l], &why) ||
          !shard_linear(graph, p + "down", F, H, sh.ffn0, sh.ffn1, {{0, H}}, full, wbase, &cur, dry, S->st,
                        &S->down[l], &why))
        return 0;
    }
    if (!shard_linear(graph, "lm_head", H, gc.vocab, 0, H, {{sh.vocab0, sh.vocab1}}, full, wbase, &cur, dry, S->st,
                      &S->lm, &why))
      return 0;
    return std::max<uint64_t>(cur, 256);
  };
  uint64_t w_region = wbytes;
  if (world > 1) {
    w_region = place(nullptr, nullptr, true);
    if (w_region == 0) {
      set_err("%s: %s", fn, why.c_str());
      return nullptr;
    }
  }
  // slab layout
  S->plan = make_plan(c, T * batch, batch, world);
  S->kv_head_stride = (int64_t)c.max_context * c.head_dim;
  S->kv_block = (int64_t)c.kv_heads * S->kv_head_stride;
  const uint64_t off_w = 0;
  const uint64_t off_kv = align_up(off_w + w_region, 4096);
  const KvLayout kl = kv_layout(c, batch, kv_mode, pool_tokens);
  const uint64_t kv_bytes = kl.bytes;
  const uint64_t off_act = align_up(off_kv + kv_bytes, 4096);
  const uint64_t off_lws = align_up(off_act + S->plan.bytes, 4096);
  S->lin_ws_bytes = align_up(std::max<size_t>(lws, 4096), 256);
  const uint64_t off_aws = align_up(off_lws + S->lin_ws_bytes, 4096);
  S->attn_ws_bytes = align_up(std::max<size_t>(aws, 256), 256);
  S->slab_bytes = align_up(off_aws + S->attn_ws_bytes, 4096);
  char* full = nullptr;  // the whole weight image, while the shards are cut (several ranks)
  bool ok = cudaMalloc(&S->slab, S->slab_bytes) == cudaSuccess;
  if (ok && world > 1) ok = cudaMalloc(&full, wbytes) == cudaSuccess;
  if (!ok) cudaGetLastError();
  if (world > 1) {
    // every rank learns whether all ranks got their memory before any goes on
    int bad = ok ? 0 : 1;
    ncclResult_t e = ncclSuccess;
    if (cudaMemcpyAsync(S->tp_flag, &bad, 4, cudaMemcpyHostToDevice, S->st) != cudaSuccess ||
        (e = nccl_api().all_reduce(S->tp_flag, S->tp_flag, 1, ncclInt32, ncclMax, S->comm, S->st)) != ncclSuccess ||
        cudaMemcpyAsync(&bad, S->tp_flag, 4, cudaMemcpyDeviceToHost, S->st) != cudaSuccess ||
        cudaStreamSynchronize(S->st) != cudaSuccess)
      bad = 1;
    if (bad) ok = false;
  }
  if (!ok) {
    if (full) cudaFree(full);
    set_err("%s: cannot allocate %llu bytes on device %d (or another rank could not)", fn,
            (unsigned long long)S->slab_bytes, S->dev);
    return nullptr;
  }
  graph->peak_bytes = std::max(graph->peak_bytes, S->slab_bytes);
  char* wbase = S->slab + off_w;
  S->kv = S->slab + off_kv;
  if (kl.paged) {
    S->paged = true;
    S->pool_pages = kl.pool_pages;
    S->max_lpages = kl.max_lpages;
    S->d_table = reinterpret_cast<int32_t*>(S->kv + align_up(kl.pool_bytes, 4096));
    S->h_table.assign((size_t)kl.max_lpages * c.layers * batch, 0);
    S->kvp.resize(c.layers);
    for (int l = 0; l < c.layers; ++l) {
      SgKvPages& kp = S->kvp[l];
      kp.table = S->d_table + (size_t)l * batch;
      kp.page_size = 16;
      kp.num_pages = kl.pool_pages;
      kp.page_stride = (int64_t)2 * c.kv_heads * 16 * c.head_dim;
      kp.table_batch_stride = 1;
      kp.table_page_stride = (int64_t)c.layers * batch;
    }
    release_pages(S.get());
  }
  S->act = S->slab + off_act;
  S->lin_ws = S->slab + off_lws;
  S->attn_ws = S->slab + off_aws;
  auto cleanup_fail = [&](const char* what) -> ArmSession* {
    if (full) {
      cudaStreamSynchronize(S->st);
      cudaFree(full);
    }
    set_err("%s: %s", fn, what);
    return nullptr;
  };
  char* image = world > 1 ? full : wbase;
  if (cudaMemcpyAsync(image, wdata, wbytes, cudaMemcpyHostToDevice, S->st) != cudaSuccess ||
      cudaMemsetAsync(S->kv, 0, kv_bytes, S->st) != cudaSuccess ||
      cudaMemsetAsync(S->lin_ws, 0, S->lin_ws_bytes, S->st) != cudaSuccess ||
      cudaMemsetAsync(S->attn_ws, 0, S->attn_ws_bytes, S->st) != cudaSuccess) {
    cudaGetLastError();
    return cleanup_fail("uploading the weights failed");
  }
  if (world > 1) {
    if (place(full, wbase, false) == 0) return cleanup_fail(why.c_str());
    if (cudaStreamSynchronize(S->st) != cudaSuccess) return cleanup_fail("cutting the weight shards failed");
    cudaFree(full);
    full = nullptr;
    decide_fusion(S.get());
    return S.release();
  }
  if (cudaStreamSynchronize(S->st) != cudaSuccess) {
    cudaGetLastError();
    return cleanup_fail("uploading the weights failed");
  }
  // bind tensors of the whole image
  auto t = [&](const std::string& n, uint64_t expect) -> const void* {
    const TensorRef* r = find(n, expect);
    return r ? wbase + r->offset : nullptr;
  };
  S->embed = t("embed_tokens", (uint64_t)c.vocab * H2);
  S->final_norm = t("final_norm", H2);
  if (!S->embed || !S->final_norm) return cleanup_fail("embed_tokens / final_norm missing or of the wrong size");
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    S->in_norm.push_back(t(p + "input_norm", H2));
    S->post_norm.push_back(t(p + "post_norm", H2));
    if (!S->in_norm.back() || !S->post_norm.back()) return cleanup_fail(("norm weights of layer " + std::to_string(l) + " missing").c_str());
    Linear a, b, g3, d;
    if (!bind_linear(graph, p + "qkv", wbase, c.hidden, c.nqkv(), &a, &why) ||
        !bind_linear(graph, p + "o", wbase, c.heads * c.head_dim, c.hidden, &b, &why) ||
        !bind_linear(graph, p + "gate_up", wbase, c.hidden, 2 * c.ffn, &g3, &why) ||
        !bind_linear(graph, p + "down", wbase, c.ffn, c.hidden, &d, &why))
      return cleanup_fail(why.c_str());
    S->qkv.push_back(a);
    S->o.push_back(b);
    S->gu.push_back(g3);
    S->down.push_back(d);
  }
  if (c.lm_int4) {
    if (!bind_linear(graph, "lm_head", wbase, c.hidden, c.vocab, &S->lm, &why)) return cleanup_fail(why.c_str());
  } else {
    S->lm_f16 = t("lm_head.weight", (uint64_t)c.vocab * H2);
    if (!S->lm_f16) return cleanup_fail("lm_head.weight missing or of the wrong size");
  }
  decide_fusion(S.get());
  return S.release();
}

}  // namespace

namespace sg {

// Session-level tuning keys, reached through sg_set_tuning.
bool sdk_tuning(std::string_view key, int value) {
  if (key == "sdk.fuse_swiglu") {
    g_fuse_swiglu.store(value);
    return true;
  }
  if (key == "sdk.fuse_norm") {
    g_fuse_norm.store(value);
    return true;
  }
  if (key == "sdk.fuse_rope") {
    g_fuse_rope.store(value);
    return true;
  }
  if (key == "sdk.decode_step_kernel") {
    g_step_kernel.store(value);
    return true;
  }
  return false;
}

}  // namespace sg

// ================================================================== C API
extern "C" {

const char* armpack_last_error(void) { return g_err.c_str(); }

ArmPackage* armpack_load(const char* path) {
  if (!path) {
    set_err("armpack_load: path is NULL");
    return nullptr;
  }
  auto pkg = std::make_unique<ArmPackage_>();
  std::string err, text;
  if (!pkg->box.open(path, &err)) {
    set_err("armpack_load: %s", err.c_str());
    return nullptr;
  }
  if (!pkg->box.read_text("manifest.json", &text, &err)) {
    set_err("armpack_load: %s", err.c_str());
    return nullptr;
  }
  if (!sgsdk::json_parse(text, &pkg->manifest, &err)) {
    set_err("armpack_load: manifest.json: %s", err.c_str());
    return nullptr;
  }
  const Json& m = pkg->manifest;
  pkg->model_id = m["model_id"].text();
  pkg->family = m["model_family"].text();
  pkg->compiler_version = m["compiler_version"].text();
  const Json& arch = m["arch"];
  pkg->num_layers = (uint32_t)arch["num_layers"].integer();
  pkg->hidden = (uint32_t)arch["hidden_size"].integer();
  pkg->vocab = (uint32_t)arch["vocab_size"].integer();
  pkg->num_kernels = (uint32_t)m["kernels"].size();
  pkg->num_weight_files = (uint32_t)m["weights"].size();
  const Json& gs = m["graphs"];
  if (gs.kind != Json::Array) {
    set_err("armpack_load: manifest.json has no graphs array");
    return nullptr;
  }
  for (size_t i = 0; i < gs.size(); ++i) {
    auto g = std::make_unique<ArmGraph_>();
    const Json& e = gs[i];
    g->pkg = pkg.get();
    g->index = (uint32_t)e["index"].integer((int64_t)i);
    g->id = e["id"].text();
    g->path = e["path"].text();
    g->backend = e["execution_backend"].text("cpu");
    g->ttft_ms = (float)e["estimated_ttft_ms"].number();
    g->tpot_ms = (float)e["estimated_tpot_ms"].number();
    g->peak_bytes = (uint64_t)e["peak_memory_bytes"].integer();
    g->context_length = (uint32_t)e["context_length"].integer();
    {
      const std::string th = e["thermal_state"].text("nominal"), lm = e["latency_mode"].text("interactive");
      g->thermal = th == "warm" ? 1 : th == "hot" ? 2 : th == "critical" ? 3 : 0;
      g->latency = lm == "batch" ? 1 : lm == "background" ? 2 : 0;
    }
    g->description = g->id + " [" + g->backend + ", " + e["quant_dtype"].text("?") + ", context " +
                     std::to_string(g->context_length) + "]";
    if (g->backend == "cuda") {
      g->runnable = parse_cuda_graph(pkg.get(), g.get(), &g->why_not);
    } else {
      g->why_not = "execution backend '" + g->backend + "' is not run by this library (only 'cuda')";
    }
    pkg->graphs.push_back(std::move(g));
  }
  return pkg.release();
}

void armpack_destroy(ArmPackage* pkg) { delete pkg; }

uint32_t armpack_num_graphs(const ArmPackage* pkg) { return pkg ? (uint32_t)pkg->graphs.size() : 0; }

ArmGraph* armpack_get_graph(ArmPackage* pkg, uint32_t index) {
  if (!pkg || index >= pkg->graphs.size()) {
    set_err("armpack_get_graph: index %u out of range", index);
    return nullptr;
  }
  return pkg->graphs[index].get();
}

// Device memory a one-sequence session of `g` allocates: the weight image,
// the KV cache for the graph's full context, the planned activations and the
// kernels' scratch -- the slab armgraph_create_session asks cudaMalloc for.
static uint64_t planned_session_bytes(const ArmGraph_* g, int batch) {
  const ModelCfg& c = g->cfg;
  uint64_t w = 0;
  for (const auto& kv : g->tensors) w = std::max(w, kv.second.offset + kv.second.bytes);
  size_t lws = 0, aws = 0;
  session_scratch(c, batch, &lws, &aws);
  const Plan plan = make_plan(c, c.max_chunk * batch, batch, 1);
  const uint64_t kv_bytes = kv_layout(c, batch, 0, 0).bytes;
  uint64_t off = align_up(w, 4096);
  off = align_up(off + kv_bytes, 4096);
  off = align_up(off + plan.bytes, 4096);
  off = align_up(off + align_up(std::max<size_t>(lws, 4096), 256), 4096);
  return align_up(off + align_up(std::max<size_t>(aws, 256), 256), 4096);
}

// GraphSelector::score (compiler/lib/generator/graph_selector.cpp:34-94) for
// "cuda" graphs, lower is better: a graph whose peak memory exceeds 95 % of
// the available device memory is rejected (:45-51); latency-mode mismatch
// +20, thermal mismatch +10 per step, a context shorter than requested
// +500 + 0.1 per missing token, a longer one +0.001 per extra token, memory
// use above 85 % of the budget +50 and below 30 % +10, and half the
// estimated TPOT.  The SoC and precision rules do not apply to a CUDA graph,
// and there is no Vulkan penalty (no Vulkan candidate is run here).
static bool score_graph(const ArmGraph_* g, const ArmDeviceState* st, uint64_t avail, uint64_t need, float* out) {
  if (need > avail / 100 * 95) return false;
  float s = 0.f;
  const int lat = st ? (int)st->latency_mode : 0, th = st ? (int)st->thermal_state : 0;
  if (g->latency != lat) s += 20.f;
  if (g->thermal != th) s += 10.f * (float)std::abs(g->thermal - th);
  const uint32_t ctx = g->context_length ? g->context_length : (uint32_t)g->cfg.max_context;
  const int64_t diff = (int64_t)ctx - (int64_t)(st ? st->context_length : 0);
  s += diff < 0 ? 500.f + (float)(-diff) * 0.1f : (float)diff * 0.001f;
  const float use = avail ? (float)need / (float)avail : 1.f;
  if (use > 0.85f) s += 50.f;
  else if (use < 0.3f) s += 10.f;
  s += g->tpot_ms * 0.5f;
  *out = s;
  return true;
}

static ArmGraph* select_within(ArmPackage* pkg, const ArmDeviceState* state, uint64_t avail, const char* fn) {
  ArmGraph_* best = nullptr;
  float best_score = 0.f;
  std::string refused;
  for (auto& g : pkg->graphs) {
    if (!g->runnable) continue;
    const uint64_t need = std::max(g->peak_bytes, planned_session_bytes(g.get(), 1));
    float sc = 0.f;
    if (!score_graph(g.get(), state, avail, need, &sc)) {
      char buf[256];
      snprintf(buf, sizeof buf, "; %s needs %llu bytes, more than 95%% of the %llu available", g->id.c_str(),
               (unsigned long long)need, (unsigned long long)avail);
      refused += buf;
      continue;
    }
    if (!best || sc < best_score) {
      best = g.get();
      best_score = sc;
    }
  }
  if (!best) {
    std::string why = refused.empty() ? std::string("; no runnable 'cuda' graph in the package") : refused;
    for (auto& g : pkg->graphs)
      if (g->backend == "cuda" && !g->runnable) why += "; " + g->id + ": " + g->why_not;
    set_err("%s: no graph fits%s", fn, why.c_str());
  }
  return best;
}

ArmGraph* armpack_select_graph(ArmPackage* pkg, const ArmDeviceState* state) {
  if (!pkg) {
    set_err("armpack_select_graph: package is NULL");
    return nullptr;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    set_err("armpack_select_graph: no CUDA device (this library runs only 'cuda' graphs)");
    return nullptr;
  }
  // the device a session would run on (SG_DEVICE, else the current one) and its free memory now:
  // the selection refuses before allocating, as the reference's execution policy requires
  int prev = 0, dev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = 0;
  dev = prev;
  if (const char* d = getenv("SG_DEVICE")) dev = atoi(d);
  size_t free_b = 0, total_b = 0;
  const bool ok = cudaSetDevice(dev) == cudaSuccess && cudaMemGetInfo(&free_b, &total_b) == cudaSuccess;
  cudaSetDevice(prev);
  if (!ok) {
    cudaGetLastError();
    set_err("armpack_select_graph: cannot query the memory of CUDA device %d", dev);
    return nullptr;
  }
  uint64_t avail = free_b;
  // a caller-stated budget (ArmDeviceState.ram_mb, the reference's ram_available_mb) caps it
  if (state && state->ram_mb > 0) avail = std::min<uint64_t>(avail, (uint64_t)state->ram_mb << 20);
  return select_within(pkg, state, avail, "armpack_select_graph");
}

ArmGraph* sg_select_graph_within(ArmPackage* pkg, const ArmDeviceState* state, uint64_t device_bytes_available) {
  if (!pkg) {
    set_err("sg_select_graph_within: package is NULL");
    return nullptr;
  }
  return select_within(pkg, state, device_bytes_available, "sg_select_graph_within");
}

uint64_t sg_graph_session_bytes(const ArmGraph* graph, uint32_t batch) {
  if (!graph || !graph->runnable || batch == 0) return 0;
  return planned_session_bytes(graph, (int)std::min<uint32_t>(batch, 1u << 20));
}

const char* armgraph_description(const ArmGraph* graph) { return graph ? graph->description.c_str() : ""; }
float armgraph_estimated_tpot_ms(const ArmGraph* graph) { return graph ? graph->tpot_ms : 0.f; }
uint64_t armgraph_peak_memory_bytes(const ArmGraph* graph) { return graph ? graph->peak_bytes : 0; }

ArmSession* armgraph_create_session(ArmGraph* graph, const ArmSessionOptions* opts) {
  return create_session(graph, opts, 0, 1, nullptr, 1);
}

void armsess_destroy(ArmSession* sess) {
  if (sess) cudaSetDevice(sess->dev);
  delete sess;  // the destructor waits for the stream and frees the slab
}

void armsess_reset(ArmSession* sess) {
  if (!sess) return;
  release_pages(sess);
  sess->pos = 0;
  sess->emitted = true;
  sess->next_host = -1;
  sess->generated = 0;
  sess->ttft_ms = sess->tpot_ms = 0;
}

ArmStatus armsess_prefill(ArmSession* sess, const int32_t* tokens, uint32_t n_tokens) {
  if (!sess || (!tokens && n_tokens)) {
    set_err("armsess_prefill: NULL argument");
    return ARMCC_ERR_RUNTIME;
  }
  if (sess->batch != 1) {
    set_err("armsess_prefill: the session decodes %d sequences; use sg_batch_prefill", sess->batch);
    return ARMCC_ERR_UNSUPPORTED;
  }
  if (n_tokens == 0) return ARMCC_OK;
  return prefill_tokens(sess, tokens, n_tokens, "armsess_prefill");
}

ArmInferenceResult armsess_decode(ArmSession* sess) {
  ArmInferenceResult res{};
  res.next_token_id = -1;
  if (!sess) {
    set_err("armsess_decode: session is NULL");
    res.status = ARMCC_ERR_RUNTIME;
    return res;
  }
  if (sess->batch != 1) {
    set_err("armsess_decode: the session decodes %d sequences; use sg_batch_decode", sess->batch);
    res.status = ARMCC_ERR_UNSUPPORTED;
    return res;
  }
  float step_ms = 0;
  const ArmStatus r = step_tokens(sess, "armsess_decode", &step_ms);
  if (r != ARMCC_OK) {
    res.status = r;
    return res;
  }
  res.next_token_id = sess->next_host;
  res.logprob = sess->logprob_host;
  res.ttft_ms = sess->ttft_ms;
  res.tpot_ms = sess->tpot_ms;
  res.tokens_generated = sess->generated;
  res.status = ARMCC_OK;
  return res;
}

ArmStatus armsess_generate(ArmSession* sess, const int32_t* prompt_tokens, uint32_t prompt_len,
                           uint32_t max_new_tokens, void (*output_cb)(int32_t token_id, void* ctx), void* ctx) {
  ArmStatus r = armsess_prefill(sess, prompt_tokens, prompt_len);
  if (r != ARMCC_OK) return r;
  for (uint32_t i = 0; i < max_new_tokens; ++i) {
    const ArmInferenceResult res = armsess_decode(sess);
    if (res.status != ARMCC_OK) return res.status;
    if (output_cb) output_cb(res.next_token_id, ctx);
  }
  return ARMCC_OK;
}

ArmInferenceResult armgraph_run(ArmGraph* graph, const int32_t* tokens, uint32_t n_tokens) {
  ArmInferenceResult res{};
  res.next_token_id = -1;
  ArmSession* s = armgraph_create_session(graph, nullptr);
  if (!s) {
    res.status = ARMCC_ERR_RUNTIME;
    return res;
  }
  const ArmStatus r = armsess_prefill(s, tokens, n_tokens);
  if (r != ARMCC_OK) {
    res.status = r;
  } else {
    res = armsess_decode(s);
  }
  armsess_destroy(s);
  return res;
}

ArmStatus armpack_get_info(const ArmPackage* pkg, ArmPackageInfo* info) {
  if (!pkg || !info) {
    set_err("armpack_get_info: NULL argument");
    return ARMCC_ERR_RUNTIME;
  }
  memset(info, 0, sizeof *info);
  snprintf(info->model_id, sizeof info->model_id, "%s", pkg->model_id.c_str());
  snprintf(info->model_family, sizeof info->model_family, "%s", pkg->family.c_str());
  snprintf(info->compiler_version, sizeof info->compiler_version, "%s", pkg->compiler_version.c_str());
  info->num_graphs = (uint32_t)pkg->graphs.size();
  info->num_kernels = pkg->num_kernels;
  info->num_weight_files = pkg->num_weight_files;
  info->num_layers = pkg->num_layers;
  info->hidden_size = pkg->hidden;
  info->vocab_size = pkg->vocab;
  return ARMCC_OK;
}

void armpack_print_summary(const ArmPackage* pkg) {
  if (!pkg) return;
  printf("armpack: %s (%s), compiler %s\n", pkg->model_id.c_str(), pkg->family.c_str(),
         pkg->compiler_version.c_str());
  printf("  layers %u, hidden %u, vocab %u, %u weight file(s), %u kernel(s)\n", pkg->num_layers, pkg->hidden,
         pkg->vocab, pkg->num_weight_files, pkg->num_kernels);
  for (auto& g : pkg->graphs)
    printf("  graph %u: %s%s%s\n", g->index, g->description.c_str(), g->runnable ? "" : "  -- not runnable: ",
           g->runnable ? "" : g->why_not.c_str());
}

ArmTokenizer* armpack_get_tokenizer(ArmPackage* pkg) {
  (void)pkg;
  set_err("armpack_get_tokenizer: not provided by this library (sessions take token ids)");
  return nullptr;
}
int32_t* armtok_encode(ArmTokenizer* tok, const char* text, uint32_t* out_len) {
  (void)tok;
  (void)text;
  if (out_len) *out_len = 0;
  set_err("armtok_encode: no tokenizer");
  return nullptr;
}
char* armtok_decode(ArmTokenizer* tok, const int32_t* tokens, uint32_t n_tokens) {
  (void)tok;
  (void)tokens;
  (void)n_tokens;
  set_err("armtok_decode: no tokenizer");
  return nullptr;
}
void armtok_free_text(char* text) { free(text); }

ArmStatus sg_session_last_logits(ArmSession* sess, float* host_out, uint32_t n) {
  if (!sess || !host_out) {
    set_err("sg_session_last_logits: NULL argument");
    return ARMCC_ERR_RUNTIME;
  }
  if (sess->pos == 0) {
    set_err("sg_session_last_logits: no token processed yet");
    return ARMCC_ERR_RUNTIME;
  }
  const size_t count = std::min<size_t>(n, (size_t)sess->batch * sess->c.vocab);
  cudaSetDevice(sess->dev);
  if (cudaMemcpyAsync(host_out, sess->buf<float>("logits"), count * 4, cudaMemcpyDeviceToHost, sess->st) !=
          cudaSuccess ||
      cudaStreamSynchronize(sess->st) != cudaSuccess) {
    set_err("sg_session_last_logits: copy failed");
    return ARMCC_ERR_RUNTIME;
  }
  return ARMCC_OK;
}

uint32_t sg_session_position(const ArmSession* sess) { return sess ? (uint32_t)sess->pos : 0; }

ArmStatus sg_tp_shard(const SgTpModel* model, int32_t rank, int32_t world, SgTpShard* out) {
  if (!model || !out) {
    set_err("sg_tp_shard: NULL argument");
    return ARMCC_ERR_RUNTIME;
  }
  std::string why;
  if (!tp_plan(*model, rank, world, out, &why)) {
    set_err("sg_tp_shard: %s", why.c_str());
    return ARMCC_ERR_UNSUPPORTED;
  }
  return ARMCC_OK;
}

ArmStatus sg_tp_unique_id(uint8_t id_out[128]) {
  if (!id_out) {
    set_err("sg_tp_unique_id: NULL argument");
    return ARMCC_ERR_RUNTIME;
  }
  if (!nccl_api().ok) {
    set_err("sg_tp_unique_id: %s", nccl_api().why.c_str());
    return ARMCC_ERR_UNSUPPORTED;
  }
  ncclUniqueId uid;
  const ncclResult_t e = nccl_api().get_unique_id(&uid);
  if (e != ncclSuccess) {
    set_err("sg_tp_unique_id: ncclGetUniqueId failed: %s", nccl_api().error_string(e));
    return ARMCC_ERR_RUNTIME;
  }
  static_assert(sizeof uid.internal == 128, "NCCL unique id size");
  memcpy(id_out, uid.internal, 128);
  return ARMCC_OK;
}

ArmSession* sg_session_create_ex(ArmGraph* graph, const ArmSessionOptions* opts, uint32_t batch, int32_t rank,
                                 int32_t world, const uint8_t id[128]) {
  if (world > 1 && !id) {
    set_err("sg_session_create_ex: id is NULL");
    return nullptr;
  }
  if (world < 1 || rank < 0 || rank >= world) {
    set_err("sg_session_create_ex: rank %d outside a group of %d", rank, world);
    return nullptr;
  }
  return create_session(graph, opts, rank, world, id, (int)std::min<uint32_t>(batch, 1u << 20));
}

ArmSession* sg_session_create_paged(ArmGraph* graph, const ArmSessionOptions* opts, uint32_t batch,
                                    uint64_t kv_pool_tokens, int32_t rank, int32_t world, const uint8_t id[128]) {
  if (world > 1 && !id) {
    set_err("sg_session_create_paged: id is NULL");
    return nullptr;
  }
  if (world < 1 || rank < 0 || rank >= world || batch == 0) {
    set_err("sg_session_create_paged: rank %d outside a group of %d, or batch 0", rank, world);
    return nullptr;
  }
  return create_session(graph, opts, rank, world, id, (int)std::min<uint32_t>(batch, 1u << 20), 2,
                        (int64_t)std::min<uint64_t>(kv_pool_tokens, (uint64_t)INT64_MAX / 2));
}

ArmStatus sg_session_abort(ArmSession* sess, const char* reason) {
  if (!sess) {
    set_err("sg_session_abort: session is NULL");
    return ARMCC_ERR_RUNTIME;
  }
  cudaSetDevice(sess->dev);
  abort_session(sess, reason && *reason ? reason : "aborted by the caller", false);
  return ARMCC_OK;
}

int32_t sg_session_kv_pages(const ArmSession* sess, uint32_t* pool_pages, uint32_t* pages_in_use) {
  if (!sess || !sess->paged) {
    if (pool_pages) *pool_pages = 0;
    if (pages_in_use) *pages_in_use = 0;
    return 0;
  }
  if (pool_pages) *pool_pages = (uint32_t)sess->pool_pages;
  if (pages_in_use) *pages_in_use = (uint32_t)(sess->pool_pages - (int)sess->free_pages.size());
  return 1;
}

int32_t sg_session_step_trace(ArmSession* sess, int32_t on, uint64_t* host, uint32_t cap, int32_t* ctas) {
  if (!sess || !sess->ds) {
    set_err("sg_session_step_trace: the session has no decode-step kernel");
    return -1;
  }
  cudaSetDevice(sess->dev);
  cudaStreamSynchronize(sess->st);
  size_t n = 0;
  int nct = 0;
  if (sg::decode_step_trace(sess->ds, on != 0, host, cap, &n, &nct) != SG_OK) {
    set_err("sg_session_step_trace: %s", sg_last_error());
    return -1;
  }
  if (ctas) *ctas = nct;
  return (int32_t)n;
}

int32_t sg_session_graph_kernels(const ArmSession* sess) {
  if (!sess || !sess->graph) return -1;
  size_t n = 0;
  if (cudaGraphGetNodes(sess->graph, nullptr, &n) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  std::vector<cudaGraphNode_t> nodes(n);
  if (n && cudaGraphGetNodes(sess->graph, nodes.data(), &n) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  // only this library's kernels: a kernel node's function lies in this shared object
  Dl_info self{};
  const bool know_self = dladdr(reinterpret_cast<void*>(&sg_session_graph_kernels), &self) != 0 && self.dli_fname;
  int k = 0;
  for (size_t i = 0; i < n; ++i) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nodes[i], &t) != cudaSuccess || t != cudaGraphNodeTypeKernel) continue;
    cudaKernelNodeParams kp{};
    Dl_info where{};
    if (know_self && cudaGraphKernelNodeGetParams(nodes[i], &kp) == cudaSuccess && kp.func &&
        dladdr(kp.func, &where) != 0 && where.dli_fname && strcmp(where.dli_fname, self.dli_fname) != 0)
      continue;  // another library's kernel (NCCL's collectives)
    ++k;
  }
  cudaGetLastError();
  return k;
}

double sg_session_step_gpu_ms(ArmSession* sess, int32_t on) {
  if (!sess) return -1.0;
  cudaSetDevice(sess->dev);
  if (on && !sess->ev_step[0]) {
    if (cudaEventCreate(&sess->ev_step[0]) != cudaSuccess || cudaEventCreate(&sess->ev_step[1]) != cudaSuccess) {
      cudaGetLastError();
      return -1.0;
    }
    sess->step_gpu_ms = 0;
    sess->step_gpu_n = 0;
    return 0.0;
  }
  const double avg = sess->step_gpu_n ? sess->step_gpu_ms / (double)sess->step_gpu_n : 0.0;
  if (!on) {
    cudaStreamSynchronize(sess->st);
    for (cudaEvent_t& e : sess->ev_step)
      if (e) {
        cudaEventDestroy(e);
        e = nullptr;
      }
    sess->ev_pending = false;
  }
  return avg;
}

int32_t sg_session_step_kernel(const ArmSession* sess, const char** why) {
  const char* w = nullptr;
  if (!sess) w = "no session";
  else if (sess->ds) w = nullptr;
  else if (!sess->ds_why.empty()) w = sess->ds_why.c_str();
  else if (sess->batch != 1) w = "more than one sequence";
  else if (sess->tp_world != 1) w = "tensor-parallel";
  else if (!sess->ds_tried) w = "not built yet (the first decode step builds it)";
  else w = "not eligible (norm fusion off, an fp16 LM head, or the switch is off)";
  if (why) *why = w;
  return sess && sess->ds ? 1 : 0;
}

ArmStatus sg_batch_prefill(ArmSession* sess, const int32_t* tokens, uint32_t n_tokens) {
  if (!sess || (!tokens && n_tokens)) {
    set_err("sg_batch_prefill: NULL argument");
    return ARMCC_ERR_RUNTIME;
  }
  if (n_tokens == 0) return ARMCC_OK;
  return prefill_tokens(sess, tokens, n_tokens, "sg_batch_prefill");
}

ArmStatus sg_batch_decode(ArmSession* sess, int32_t* next_tokens) {
  if (!sess || !next_tokens) {
    set_err("sg_batch_decode: NULL argument");
    return ARMCC_ERR_RUNTIME;
  }
  float step_ms = 0;
  const ArmStatus r = step_tokens(sess, "sg_batch_decode", &step_ms);
  if (r != ARMCC_OK) return r;
  memcpy(next_tokens, sess->next_all.data(), (size_t)sess->batch * 4);
  return ARMCC_OK;
}

uint32_t sg_session_batch(const ArmSession* sess) { return sess ? (uint32_t)sess->batch : 0; }

ArmSession* sg_session_create_tp(ArmGraph* graph, const ArmSessionOptions* opts, int32_t rank, int32_t world,
                                 const uint8_t id[128]) {
  if (world > 1 && !id) {
    set_err("sg_session_create_tp: id is NULL");
    return nullptr;
  }
  if (world < 1 || rank < 0 || rank >= world) {
    set_err("sg_session_create_tp: rank %d outside a group of %d", rank, world);
    return nullptr;
  }
  return create_session(graph, opts, rank, world, id, 1);
}

void sg_session_vocab_range(const ArmSession* sess, uint32_t* lo, uint32_t* hi) {
  if (lo) *lo = sess ? (uint32_t)sess->shard.vocab0 : 0;
  if (hi) *hi = sess ? (uint32_t)sess->shard.vocab1 : 0;
}
void armtok_free_tokens(int32_t* tokens) { free(tokens); }

}  // extern "C"
