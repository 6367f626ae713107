// Library-level entry points of the C ABI and the host helpers shared by
// the kernel files (error recording, device properties, smem opt-in).
#include <mutex>
#include <string>
#include <vector>

#include "pl_common.cuh"

namespace {
thread_local std::string g_last_cuda_error;

struct SmemAttr {
  const void* kernel;
  int device;
  int bytes;
};
std::mutex g_attr_mu;
std::vector<SmemAttr> g_attrs;

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
}  // namespace

namespace pl_host {

int32_t record_cuda_error(cudaError_t err) {
  g_last_cuda_error = cudaGetErrorString(err);
  return PL_ERR_CUDA;
}

int32_t sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int32_t ensure_smem_attr(const void* kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda_error(e);
  std::lock_guard<std::mutex> lock(g_attr_mu);
  for (auto& a : g_attrs)
    if (a.kernel == kernel && a.device == dev) {
      if (a.bytes >= bytes) return PL_OK;
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      if (e != cudaSuccess) return record_cuda_error(e);
      a.bytes = bytes;
      return PL_OK;
    }
  if (bytes > 48 * 1024) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return record_cuda_error(e);
  }
  g_attrs.push_back({kernel, dev, bytes});
  return PL_OK;
}

}  // namespace pl_host

extern "C" int32_t pl_abi_version(void) { return PL_ABI_VERSION; }

extern "C" const char* pl_status_string(int32_t status) {
  switch (status) {
    case PL_OK: return "ok";
    case PL_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PL_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case PL_ERR_PAGE_OUT_OF_RANGE: return "page index out of range";
    case PL_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case PL_ERR_SPAN_START: return "page spans must start at page offset 0";
    case PL_ERR_SPAN_LENGTH: return "page span length is out of range";
    case PL_ERR_SPAN_NOT_FULL: return "non-last page spans must be full pages";
    case PL_ERR_CUDA: return "CUDA runtime error";
    case PL_ERR_TIMEOUT: return "device wait timed out";
    case PL_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

extern "C" const char* pl_last_cuda_error(void) { return g_last_cuda_error.c_str(); }

extern "C" int32_t pl_device_sm_count(void) { return pl_host::sm_count(); }

