// Library runtime: error reporting, device queries, library-owned scratch.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "sm100.cuh"

namespace sg {

namespace {
thread_local char g_err[1024] = "";

struct WsKey {
  int dev;
  void* stream;
  int user;
  bool operator==(const WsKey& o) const { return dev == o.dev && stream == o.stream && user == o.user; }
};
struct WsKeyHash {
  size_t operator()(const WsKey& k) const {
    return (std::hash<void*>()(k.stream) * 31u + (size_t)k.dev) * 7u + (size_t)k.user;
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

std::mutex g_err_mu;
std::unordered_map<int, int*> g_err_word;

std::mutex g_tm_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
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

SgStatus library_workspace(void* stream, size_t bytes, void** out, int user) {
  int dev = 0;
  SgStatus st = current_device(&dev);
  if (st != SG_OK) return st;
  std::lock_guard<std::mutex> lk(g_ws_mu);
  WsBuf& b = g_ws[WsKey{dev, stream, user}];
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

SgStatus device_error_word(int** out) {
  int dev = 0;
  SgStatus st = current_device(&dev);
  if (st != SG_OK) return st;
  std::lock_guard<std::mutex> lk(g_err_mu);
  auto it = g_err_word.find(dev);
  if (it != g_err_word.end()) {
    *out = it->second;
    return SG_OK;
  }
  int* p = nullptr;
  SG_CUDA_TRY(cudaMalloc(&p, 256));
  SG_CUDA_TRY(cudaMemset(p, 0, 256));
  g_err_word[dev] = p;
  *out = p;
  return SG_OK;
}

int* existing_device_error_word(int dev) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  auto it = g_err_word.find(dev);
  return it == g_err_word.end() ? nullptr : it->second;
}

SgStatus make_tensor_map(CUtensorMap* out, CUtensorMapDataType dt, int rank, void* base, const uint64_t* dims,
                         const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  {
    std::lock_guard<std::mutex> lk(g_tm_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        cudaGetLastError();
        set_error("cuTensorMapEncodeTiled unavailable");
        return SG_ERR_RUNTIME;
      }
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) gstride[i] = strides_bytes[i];
  }
  CUresult r = g_encode(out, dt, (cuuint32_t)rank, base, gdim, gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (code %d)", (int)r);
    return SG_ERR_INVALID;
  }
  return SG_OK;
}

}  // namespace sg

extern "C" {

int32_t sg_device_error_check(void* stream) {
  // Two words can hold a device-side error: the library's own (created on a
  // device's first launch that needs it) and the one the allocation-free GEMV
  // passes its kernels.  A word that does not exist yet has recorded nothing,
  // so this check allocates no device memory.
  int dev = 0;
  if (sg::current_device(&dev) != SG_OK) return SG_ERR_RUNTIME;
  int* words[2] = {sg::existing_device_error_word(dev), sg::noalloc_error_word(dev)};
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  int first = 0;
  for (int* w : words) {
    if (!w) continue;
    int v = 0;
    if (cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, cs) != cudaSuccess ||
        cudaStreamSynchronize(cs) != cudaSuccess) {
      cudaGetLastError();
      sg::set_error("sg_device_error_check: copy failed");
      return SG_ERR_RUNTIME;
    }
    if (v != 0) {
      cudaMemsetAsync(w, 0, sizeof(int), cs);
      cudaStreamSynchronize(cs);
      if (first == 0) first = v;
    }
  }
  if (first != 0) {
    sg::set_error("device-side error %d (1 = a bounded wait timed out)", first);
    return SG_ERR_RUNTIME;
  }
  return SG_OK;
}

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
