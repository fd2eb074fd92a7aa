// sg_matmul_int4_grouped_noalloc: the INT4 grouped GEMV for callers that may
// not allocate device memory once they are running.
//
// Who needs it: a runtime that fixes its whole device-memory budget when a
// session is admitted and refuses work rather than allocate later (the
// reference's execution policy decides before allocating, see
// scripts/test_armpack.py:92-96), or a host framework whose memory pool owns
// the device and forbids direct cudaMalloc/cudaFree.  sg_matmul_int4_grouped
// normally takes its split-reduction scratch from a library cache that grows
// with cudaMalloc; this entry point never does.
//
// How: the scratch lives in one file-scope __device__ array of
// kNoAllocScratchBytes (2 MiB), which every GPU that loads the library holds
// until the process exits.  Host code cannot use the array's name as a device
// address (on the host it is only a stand-in symbol), so on the first call on
// each device -- with that device current -- cudaGetSymbolAddress fetches the
// real address, which is then passed to the kernels.  Make that first call on
// a device before any stream capture on it.
//
// Contract: results are those of sg_matmul_int4_grouped; p->workspace and
// p->workspace_bytes are ignored.  A problem whose scratch exceeds 2 MiB is
// rejected with SG_ERR_INVALID and a message.  All calls share the one array
// per device and it keeps the previous call's contents: each call zeroes the
// ticket counters it relies on before its kernel runs, and calls that overlap
// on the GPU (for example on two streams at once) race on the array -- order
// them on one stream.  No cudaMalloc, cudaFree or allocating library routine
// is called.  A bounded wait that runs out in these kernels sets this file's
// own error word, which sg_device_error_check reads and clears together with
// the library's (that check allocates nothing either).
#include <mutex>

#include "sm100.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB
constexpr int kMaxDevices = 64;
constexpr int kTileCols = 512;  // column tile of both GEMV paths (ticket per tile)

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ __align__(256) int g_noalloc_err[64];  // error word for bounded waits

struct DeviceSlot {
  bool ready = false;
  void* scratch = nullptr;
  int* err = nullptr;
};
std::mutex g_mu;
DeviceSlot g_slots[kMaxDevices];

// Once per device, with that device current: the device addresses of the arrays.
SgStatus device_slot(int dev, DeviceSlot** out) {
  if (dev < 0 || dev >= kMaxDevices) {
    sg::set_error("sg_matmul_int4_grouped_noalloc: device ordinal %d out of range", dev);
    return SG_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceSlot& s = g_slots[dev];
  if (!s.ready) {
    void* scratch = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      sg::set_error("sg_matmul_int4_grouped_noalloc: cudaGetSymbolAddress(scratch) failed: %s",
                    cudaGetErrorString(e));
      return SG_ERR_RUNTIME;
    }
    void* err = nullptr;
    e = cudaGetSymbolAddress(&err, g_noalloc_err);
    if (e != cudaSuccess) {
      cudaGetLastError();
      sg::set_error("sg_matmul_int4_grouped_noalloc: cudaGetSymbolAddress(error word) failed: %s",
                    cudaGetErrorString(e));
      return SG_ERR_RUNTIME;
    }
    s.scratch = scratch;
    s.err = static_cast<int*>(err);
    s.ready = true;
  }
  *out = &s;
  return SG_OK;
}

}  // namespace

namespace sg {
int* noalloc_error_word(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  return g_slots[dev].ready ? g_slots[dev].err : nullptr;
}

SgStatus w4_gemv_run(const SgMatMulParams* p, void* stream, void* ws, size_t ws_bytes, bool ws_external,
                     int* err_word);
size_t w4_gemv_scratch_bytes(const SgMatMulParams* p, bool minimal);
}  // namespace sg

extern "C" SgStatus sg_matmul_int4_grouped_noalloc(const SgMatMulParams* p, void* stream) {
  SG_CHECK_ARG(p != nullptr, "sg_matmul_int4_grouped_noalloc: params is NULL");
  int dev = 0;
  SgStatus st = sg::current_device(&dev);
  if (st != SG_OK) return st;
  DeviceSlot* slot = nullptr;
  st = device_slot(dev, &slot);
  if (st != SG_OK) return st;

  SgMatMulParams q = *p;
  q.workspace = nullptr;
  q.workspace_bytes = 0;
  // the least scratch the call runs with: the prefill GEMM splits its last
  // round of tiles only when the fixed array has room for the partial sums
  const size_t need = sg::w4_gemv_scratch_bytes(&q, true);
  if (need > kNoAllocScratchBytes) {
    sg::set_error(
        "sg_matmul_int4_grouped_noalloc: this problem (M=%d K=%d N=%d) needs %zu bytes of scratch; the fixed "
        "maximum is %zu bytes -- use sg_matmul_int4_grouped",
        q.M, q.K, q.N, need, kNoAllocScratchBytes);
    return SG_ERR_INVALID;
  }
  if (need > 0) {
    // ticket counters (one per 512-column tile, at the start of the scratch) must start at zero
    const size_t tickets = sg::ticket_bytes((q.N + kTileCols - 1) / kTileCols);
    const cudaError_t e = cudaMemsetAsync(slot->scratch, 0, tickets < need ? tickets : need,
                                          static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
      cudaGetLastError();
      sg::set_error("sg_matmul_int4_grouped_noalloc: clearing scratch failed: %s", cudaGetErrorString(e));
      return SG_ERR_RUNTIME;
    }
  }
  return sg::w4_gemv_run(&q, stream, slot->scratch, kNoAllocScratchBytes, true, slot->err);
}
