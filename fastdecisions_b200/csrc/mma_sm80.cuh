// Warp-level bf16 tensor-core helpers (mma.sync m16n8k16 + ldmatrix) used by the delta rule's
// small 64x64 / 64x128 chunk products.  Fragment conventions (g = lane / 4, t = lane % 4):
//   A 16x16 : a0 (g, 2t..2t+1)  a1 (g+8, 2t..)  a2 (g, 2t+8..)  a3 (g+8, 2t+8..)
//   B 16x8  : b0 (k = 2t..2t+1, n = g)  b1 (k = 2t+8.., n = g)
//   C 16x8  : c0,c1 (g, 2t..2t+1)  c2,c3 (g+8, 2t..2t+1)
#pragma once
#include <stdint.h>

namespace fdk {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment of the 16x16 block at (r0, c0) of a row-major [rows][ld] bf16 smem array.
__device__ __forceinline__ void load_a(const __nv_bfloat16* base, int ld, int r0, int c0, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* p = base + (r0 + (lane & 15)) * ld + c0 + ((lane >> 4) << 3);
  ldsm_x4(smem_u32(p), a[0], a[1], a[2], a[3]);
}

// A fragment of rows m0..m0+15, cols k0..k0+15 of A, where smem holds A^T as [k][ld] (row = k).
__device__ __forceinline__ void load_a_t(const __nv_bfloat16* base, int ld, int m0, int k0, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31;
  const int m = lane >> 3;
  const __nv_bfloat16* p = base + (k0 + (lane & 7) + ((m >> 1) << 3)) * ld + m0 + ((m & 1) << 3);
  ldsm_x4_t(smem_u32(p), a[0], a[1], a[2], a[3]);
}

// B fragments of two adjacent n-tiles (n0, n0+8) for k-step k0, smem holds B^T as [n][ld].
__device__ __forceinline__ void load_b_nk(const __nv_bfloat16* base, int ld, int n0, int k0, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31;
  const int m = lane >> 3;
  const __nv_bfloat16* p = base + (n0 + (lane & 7) + ((m >> 1) << 3)) * ld + k0 + ((m & 1) << 3);
  ldsm_x4(smem_u32(p), b[0], b[1], b[2], b[3]);
}

// B fragments of two adjacent n-tiles (n0, n0+8) for k-step k0, smem holds B as [k][ld].
__device__ __forceinline__ void load_b_kn(const __nv_bfloat16* base, int ld, int n0, int k0, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31;
  const int m = lane >> 3;
  const __nv_bfloat16* p = base + (k0 + (lane & 7) + ((m & 1) << 3)) * ld + n0 + ((m >> 1) << 3);
  ldsm_x4_t(smem_u32(p), b[0], b[1], b[2], b[3]);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

}  // namespace fdk
