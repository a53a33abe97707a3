// Shared helpers for the fastdecisions-b200 CUDA library (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/fdk.h"

namespace fdk {

using bf16 = __nv_bfloat16;

// Records a formatted message for fdk_get_last_error_string() and returns `code`.
int set_error(int code, const char* fmt, ...);
// Maps a pending launch error (cudaGetLastError) to FDK_ERR_LAUNCH.
int check_launch(const char* what);
// FDK_OK when the current device is an sm_100 part; FDK_ERR_DEVICE otherwise.
int check_device();
// Number of SMs of the current device (cached per device).
int sm_count();
// Raises `func`'s dynamic shared-memory limit to `bytes` on the current device, once per (kernel,
// device), safely from several host threads.  The cache assumes no cudaDeviceReset afterwards.
int ensure_smem_attr(const void* func, int bytes, const char* what);
// Reads and clears the delta-rule recurrence's device error word (set when a bounded wait ran out).
int delta_take_device_error();
// Reads and clears the GEMM kernel's device error word.
int gemm_take_device_error();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- 16-byte vectors of 8 bf16 -------------------------------------------------------------
struct alignas(16) bf16x8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// silu(x) = 0.5 x (1 + tanh(x / 2)) with the hardware tanh (tanh.approx.f32, relative error about
// 2^-11): one MUFU op instead of two, for kernels whose MUFU pipe is the limit.  Its error is well
// below the bf16 rounding of the results these kernels store.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float silu_tanh(float x) {
  const float h = 0.5f * x;
  return fmaf(h, tanh_approx(h), h);
}
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
// softplus with the identity above 20, as torch.nn.functional.softplus(beta=1, threshold=20).
__device__ __forceinline__ float softplusf_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

}  // namespace fdk
