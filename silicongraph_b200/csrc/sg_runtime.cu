// Library runtime: error reporting, device queries, library-owned scratch.
#include <mutex>
#include <unordered_map>

#include "sg_common.cuh"

namespace sg {

namespace {
thread_local char g_err[1024] = "";

struct WsKey {
  int dev;
  void* stream;
  bool operator==(const WsKey& o) const { return dev == o.dev && stream == o.stream; }
};
struct WsKeyHash {
  size_t operator()(const WsKey& k) const {
    return std::hash<void*>()(k.stream) * 31u + (size_t)k.dev;
  }
};
struct WsBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_ws_mu;
std::unordered_map<WsKey, WsBuf, WsKeyHash> g_ws;

std::mutex g_sm_mu;
std::unordered_map<int, int> g_sm;
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

const char* last_error() { return g_err; }

SgStatus check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return SG_ERR_RUNTIME;
  }
  return SG_OK;
}

SgStatus current_device(int* dev) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    set_error("no CUDA device available (%s); this library has no CPU path",
              e == cudaSuccess ? "device count 0" : cudaGetErrorString(e));
    return SG_ERR_RUNTIME;
  }
  SG_CUDA_TRY(cudaGetDevice(dev));
  return SG_OK;
}

int sm_count(int dev) {
  std::lock_guard<std::mutex> lk(g_sm_mu);
  auto it = g_sm.find(dev);
  if (it != g_sm.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    n = 148;
  }
  g_sm[dev] = n;
  return n;
}

SgStatus library_workspace(void* stream, size_t bytes, void** out) {
  int dev = 0;
  SgStatus st = current_device(&dev);
  if (st != SG_OK) return st;
  std::lock_guard<std::mutex> lk(g_ws_mu);
  WsBuf& b = g_ws[WsKey{dev, stream}];
  if (b.bytes < bytes) {
    size_t want = align_up(bytes < (1u << 20) ? (1u << 20) : bytes, 1u << 20);
    if (b.ptr) {
      // The old buffer may still be in use by queued work on this stream.
      SG_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
      SG_CUDA_TRY(cudaFree(b.ptr));
      b.ptr = nullptr;
      b.bytes = 0;
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_error("workspace cudaMalloc(%zu) failed: %s", want, cudaGetErrorString(e));
      return SG_ERR_OOM;
    }
    SG_CUDA_TRY(cudaMemset(p, 0, want));
    b.ptr = p;
    b.bytes = want;
  }
  *out = b.ptr;
  return SG_OK;
}

}  // namespace sg

extern "C" {

const char* sg_last_error(void) { return sg::last_error(); }

int32_t sg_version(void) { return (0 << 16) | (1 << 8) | 0; }

int32_t sg_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

}  // extern "C"
