// Library-wide entry points: version, thread-local error string, device checks.
#include <cstdarg>
#include <cstdio>

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

static int g_sm_major[64];
static int g_sm_count[64];

static int query(int dev) {
  if (dev < 0 || dev >= 64) return FDK_ERR_DEVICE;
  if (g_sm_major[dev] == 0) {
    int major = 0, count = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return FDK_ERR_DEVICE;
    }
    g_sm_count[dev] = count;
    g_sm_major[dev] = major;
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
  if (g_sm_major[dev] != 10)
    return set_error(FDK_ERR_DEVICE, "device %d is sm_%d0; this library is built for sm_100a only", dev,
                     g_sm_major[dev]);
  return FDK_OK;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (query(dev) != FDK_OK) return 148;
  return g_sm_count[dev];
}

}  // namespace fdk

extern "C" const char* fdk_version(void) { return "fastdecisions-b200 0.1.0 sm_100a"; }

extern "C" const char* fdk_get_last_error_string(void) { return fdk::g_last_error; }
