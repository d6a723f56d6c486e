// Library-level entry points of the C ABI: version, status strings, the
// device-side error flag of bounded waits, and the cached SM count.
#include <mutex>
#include <vector>

#include "common.cuh"
#include "device_error.cuh"

namespace tileops {

int sm_count() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// One int per device in global memory: a kernel whose bounded wait gives up
// writes a non-zero code here (see device_error.cuh) and returns early.
__device__ int g_device_error = 0;

int* device_error_ptr() {
  static std::mutex mu;
  static std::vector<int*> cached;  // by device index
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cached.size() <= static_cast<size_t>(dev)) cached.resize(static_cast<size_t>(dev) + 1, nullptr);
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

}  // namespace tileops

extern "C" int tileops_abi_version(void) { return TILEOPS_ABI_VERSION; }

extern "C" const char* tileops_status_string(int status) {
  switch (status) {
    case TILEOPS_OK: return "ok";
    case TILEOPS_EBADDTYPE: return "unsupported dtype";
    case TILEOPS_EBADSHAPE: return "invalid shape or size argument";
    case TILEOPS_EALIGN: return "pointer alignment violated";
    case TILEOPS_ELAUNCH: return "CUDA launch failed";
    case TILEOPS_ETIMEOUT: return "a bounded device-side wait timed out";
    case TILEOPS_EINVAL: return "invalid argument";
    default: return "unknown status";
  }
}

extern "C" int tileops_device_error_flag(void* stream, int clear) {
  cudaStream_t s = tileops::as_stream(stream);
  int host = 0;
  if (cudaMemcpyFromSymbolAsync(&host, tileops::g_device_error, sizeof(int), 0,
                                cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return TILEOPS_ELAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return TILEOPS_ELAUNCH;
  if (clear && host != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbolAsync(tileops::g_device_error, &zero, sizeof(int), 0,
                                cudaMemcpyHostToDevice, s) != cudaSuccess)
      return TILEOPS_ELAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return TILEOPS_ELAUNCH;
  }
  return host;
}
