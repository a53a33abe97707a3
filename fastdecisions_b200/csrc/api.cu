// Library-wide entry points: version, thread-local error string, device checks.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace fdk {

static thread_local char g_last_error[512] = "no error";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FDK_ERR_LAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return FDK_OK;
}

// Per-device attributes, cached; host threads may race on the first query (each writes the same
// values, the count before the major that marks the slot filled).
static std::atomic<int> g_sm_major[64];
static std::atomic<int> g_sm_count[64];

static int query(int dev) {
  if (dev < 0 || dev >= 64) return FDK_ERR_DEVICE;
  if (g_sm_major[dev].load(std::memory_order_acquire) == 0) {
    int major = 0, count = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return FDK_ERR_DEVICE;
    }
    g_sm_count[dev].store(count, std::memory_order_relaxed);
    g_sm_major[dev].store(major, std::memory_order_release);
  }
  return FDK_OK;
}

// (kernel, device) pairs whose dynamic shared-memory limit has been raised; guarded by a mutex so
// concurrent first calls from several host threads each see the attribute set before launching.
static std::mutex g_attr_mu;
static const void* g_attr_func[256];
static int g_attr_dev[256];
static int g_attr_n = 0;

int ensure_smem_attr(const void* func, int bytes, const char* what) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return set_error(FDK_ERR_DEVICE, "%s: no current device", what);
  }
  std::lock_guard<std::mutex> lock(g_attr_mu);
  for (int i = 0; i < g_attr_n; ++i)
    if (g_attr_func[i] == func && g_attr_dev[i] == dev) return FDK_OK;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(FDK_ERR_LAUNCH, "%s: cannot set %d bytes of shared memory: %s", what, bytes, cudaGetErrorString(e));
  }
  if (g_attr_n < 256) {
    g_attr_func[g_attr_n] = func;
    g_attr_dev[g_attr_n] = dev;
    ++g_attr_n;
  }
  return FDK_OK;
}

int check_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return set_error(FDK_ERR_DEVICE, "no CUDA device available");
  }
  if (query(dev) != FDK_OK) return set_error(FDK_ERR_DEVICE, "cannot query CUDA device %d", dev);
  const int major = g_sm_major[dev].load(std::memory_order_acquire);
  if (major != 10)
    return set_error(FDK_ERR_DEVICE, "device %d is sm_%d0; this library is built for sm_100a only", dev, major);
  return FDK_OK;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (query(dev) != FDK_OK) return 148;
  return g_sm_count[dev].load(std::memory_order_relaxed);
}

}  // namespace fdk

extern "C" const char* fdk_version(void) { return "fastdecisions-b200 0.1.0 sm_100a"; }

extern "C" const char* fdk_get_last_error_string(void) { return fdk::g_last_error; }
