// Normalisation kernels of the decoder: fused residual add + RMSNorm (1 + w), the GDN gated
// RMSNorm and the attention q/k RMSNorm + partial RoPE prologue.  All HBM-bound: every input
// byte is read once with 16-byte vector loads and every output byte written once.
#include "common.cuh"

namespace fdk {

// ---------------------------------------------------------------------------------------------
// Residual add + RMSNorm: one row per 128-thread warp group; each thread keeps its NC 8-wide
// chunks of the row in registers between the sum-of-squares pass and the scaling pass.
// RES_FP32 selects the residual stream's storage: bf16 (s rounded to bf16 before the norm reads
// it, as the eager bf16 model stores it) or float32 (no rounding of the running sum).
// ---------------------------------------------------------------------------------------------
template <bool RES_FP32>
struct ResIO;
template <>
struct ResIO<false> {
  using T = bf16;
  static __device__ __forceinline__ void load(const T* p, float (&f)[8]) { unpack8(ldg_stream(p), f); }
  static __device__ __forceinline__ void store(T* p, const float (&f)[8]) { *reinterpret_cast<uint4*>(p) = pack8(f); }
  static __device__ __forceinline__ float keep(float x) { return round_bf16(x); }
};
template <>
struct ResIO<true> {
  using T = float;
  static __device__ __forceinline__ void load(const T* p, float (&f)[8]) {
    float4 a = __ldcs(reinterpret_cast<const float4*>(p)), b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  static __device__ __forceinline__ void store(T* p, const float (&f)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
  static __device__ __forceinline__ float keep(float x) { return x; }
};

template <int NC, bool HAS_RES, bool W_FP32, bool RES_FP32>
__global__ void __launch_bounds__(128) residual_rmsnorm_kernel(
    const bf16* __restrict__ x, int64_t ldx, const void* __restrict__ res_, int64_t ldr,
    const void* __restrict__ w, bf16* __restrict__ out, int64_t ldo, void* __restrict__ res_out_,
    int64_t ldro, int hidden, float eps, float woff) {
  using IO = ResIO<RES_FP32>;
  using RT = typename IO::T;
  const RT* res = static_cast<const RT*>(res_);
  RT* res_out = static_cast<RT*>(res_out_);
  const int64_t row = blockIdx.x;
  const int nvec = hidden >> 3;
  const bf16* xr = x + row * ldx;
  float v[NC][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int i = threadIdx.x + c * 128;
    if (i < nvec) {
      if (x != nullptr) {
        unpack8(ldg_stream(xr + i * 8), v[c]);
      } else {  // the norm of the residual stream alone (its producer already added into it)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[c][j] = 0.f;
      }
      if (HAS_RES) {
        float r8[8];
        IO::load(res + row * ldr + i * 8, r8);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[c][j] = IO::keep(v[c][j] + r8[j]);
      }
      if (res_out != nullptr) IO::store(res_out + row * ldro + i * 8, v[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[c][j], v[c][j], ss);
    }
  }
  __shared__ float red[4];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = (red[0] + red[1]) + (red[2] + red[3]);
  const float inv = rsqrtf(ss / (float)hidden + eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int i = threadIdx.x + c * 128;
    if (i < nvec) {
      float wv[8];
      if (W_FP32) {
        const float4* wp = reinterpret_cast<const float4*>(static_cast<const float*>(w) + i * 8);
        float4 a = __ldg(wp), b = __ldg(wp + 1);
        wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
        wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
      } else {
        uint4 uw = __ldg(reinterpret_cast<const uint4*>(static_cast<const bf16*>(w) + i * 8));
        unpack8(uw, wv);
      }
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[c][j] * inv * (woff + wv[j]);
      *reinterpret_cast<uint4*>(out + row * ldo + i * 8) = pack8(o);
    }
  }
}

template <int NC, bool RES_FP32>
static void launch_rms(bool has_res, bool w32, dim3 grid, cudaStream_t s, const bf16* x, int64_t ldx,
                       const void* r, int64_t ldr, const void* w, bf16* o, int64_t ldo, void* ro,
                       int64_t ldro, int hidden, float eps, float woff) {
  if (has_res) {
    if (w32) residual_rmsnorm_kernel<NC, true, true, RES_FP32><<<grid, 128, 0, s>>>(x, ldx, r, ldr, w, o, ldo, ro, ldro, hidden, eps, woff);
    else     residual_rmsnorm_kernel<NC, true, false, RES_FP32><<<grid, 128, 0, s>>>(x, ldx, r, ldr, w, o, ldo, ro, ldro, hidden, eps, woff);
  } else {
    if (w32) residual_rmsnorm_kernel<NC, false, true, RES_FP32><<<grid, 128, 0, s>>>(x, ldx, r, ldr, w, o, ldo, ro, ldro, hidden, eps, woff);
    else     residual_rmsnorm_kernel<NC, false, false, RES_FP32><<<grid, 128, 0, s>>>(x, ldx, r, ldr, w, o, ldo, ro, ldro, hidden, eps, woff);
  }
}

template <int NC>
static void launch_rms_any(bool res32, bool has_res, bool w32, dim3 grid, cudaStream_t s, const bf16* x, int64_t ldx,
                           const void* r, int64_t ldr, const void* w, bf16* o, int64_t ldo, void* ro,
                           int64_t ldro, int hidden, float eps, float woff) {
  if (res32) launch_rms<NC, true>(has_res, w32, grid, s, x, ldx, r, ldr, w, o, ldo, ro, ldro, hidden, eps, woff);
  else       launch_rms<NC, false>(has_res, w32, grid, s, x, ldx, r, ldr, w, o, ldo, ro, ldro, hidden, eps, woff);
}

// ---------------------------------------------------------------------------------------------
// The residual add of k-split GEMM partials, then RMSNorm: one row per 128-thread warp group,
// s = h + p_0 + ... + p_{nparts-1} in that order (float32), written back to h, and
// out = bf16(s * rsqrt(mean(s^2) + eps) * (woff + w)) unless out is null.
// ---------------------------------------------------------------------------------------------
template <int NC, bool W_FP32>
__global__ void __launch_bounds__(128) rmsnorm_add_partials_kernel(
    const float* __restrict__ parts, int nparts, int64_t plane, float* __restrict__ h, int64_t ldh,
    const void* __restrict__ w, bf16* __restrict__ out, int64_t ldo, int hidden, float eps, float woff) {
  const int64_t row = blockIdx.x;
  const int nvec = hidden >> 3;
  float v[NC][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int i = threadIdx.x + c * 128;
    if (i < nvec) {
      float* hp = h + row * ldh + i * 8;
      float4 a = *reinterpret_cast<const float4*>(hp), b = *reinterpret_cast<const float4*>(hp + 4);
      v[c][0] = a.x; v[c][1] = a.y; v[c][2] = a.z; v[c][3] = a.w;
      v[c][4] = b.x; v[c][5] = b.y; v[c][6] = b.z; v[c][7] = b.w;
      for (int sidx = 0; sidx < nparts; ++sidx) {
        const float* pp = parts + sidx * plane + row * (int64_t)hidden + i * 8;
        const float4 pa = __ldcs(reinterpret_cast<const float4*>(pp)), pb = __ldcs(reinterpret_cast<const float4*>(pp + 4));
        v[c][0] += pa.x; v[c][1] += pa.y; v[c][2] += pa.z; v[c][3] += pa.w;
        v[c][4] += pb.x; v[c][5] += pb.y; v[c][6] += pb.z; v[c][7] += pb.w;
      }
      *reinterpret_cast<float4*>(hp) = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
      *reinterpret_cast<float4*>(hp + 4) = make_float4(v[c][4], v[c][5], v[c][6], v[c][7]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[c][j], v[c][j], ss);
    }
  }
  if (out == nullptr) return;  // uniform: the add only
  __shared__ float red[4];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = (red[0] + red[1]) + (red[2] + red[3]);
  const float inv = rsqrtf(ss / (float)hidden + eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int i = threadIdx.x + c * 128;
    if (i < nvec) {
      float wv[8];
      if (W_FP32) {
        const float4* wp = reinterpret_cast<const float4*>(static_cast<const float*>(w) + i * 8);
        float4 a = __ldg(wp), b = __ldg(wp + 1);
        wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
        wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
      } else {
        unpack8(__ldg(reinterpret_cast<const uint4*>(static_cast<const bf16*>(w) + i * 8)), wv);
      }
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[c][j] * inv * (woff + wv[j]);
      *reinterpret_cast<uint4*>(out + row * ldo + i * 8) = pack8(o);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Gated RMSNorm per head row (dv = 128): 16 lanes per row, one 16-byte chunk of o and z each.
// ---------------------------------------------------------------------------------------------
template <bool W_FP32>
__global__ void __launch_bounds__(256) gated_rmsnorm_kernel(
    const bf16* __restrict__ o, const bf16* __restrict__ z, int64_t ldz, const void* __restrict__ w,
    bf16* __restrict__ out, int64_t rows, int heads, float eps) {
  const int64_t row = (int64_t)blockIdx.x * 16 + (threadIdx.x >> 4);  // row = token * heads + head
  const int lane = threadIdx.x & 15;
  if (row >= rows) return;
  const int64_t t = row / heads;
  const int h = (int)(row - t * heads);
  float ov[8], zv[8], wv[8];
  unpack8(ldg_stream(o + row * 128 + lane * 8), ov);
  unpack8(ldg_stream(z + t * ldz + (int64_t)h * 128 + lane * 8), zv);
  if (W_FP32) {
    const float* wp = static_cast<const float*>(w) + lane * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) wv[j] = __ldg(wp + j);
  } else {
    unpack8(__ldg(reinterpret_cast<const uint4*>(static_cast<const bf16*>(w) + lane * 8)), wv);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss = fmaf(ov[j], ov[j], ss);
#pragma unroll
  for (int m = 8; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  const float inv = rsqrtf(ss * (1.0f / 128.0f) + eps);
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = wv[j] * (ov[j] * inv) * silu_tanh(zv[j]);
  *reinterpret_cast<uint4*>(out + row * 128 + lane * 8) = pack8(r);
}

// ---------------------------------------------------------------------------------------------
// q/k RMSNorm (1 + w) over head_dim + partial rotary embedding.  One warp per token: it walks the
// token's hq + hkv head rows, ten at a time with all ten rows' loads issued first.  Lane l holds
// features [l*E, l*E + E) of every row (E = head_dim / 32: 4 for 128, 8 for 256), so its norm
// weights, cos / sin factors and rotate_half partner lane are loaded and computed once per token.
// rotate_half pairs feature i with i + rot/2 inside the first rot features.
// ---------------------------------------------------------------------------------------------
template <int E>
struct RowVec;
template <>
struct RowVec<4> {
  uint2 u;
  __device__ __forceinline__ void load(const bf16* p) { u = *reinterpret_cast<const uint2*>(p); }
  __device__ __forceinline__ void to_float(float (&f)[4]) const {
    float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  }
  __device__ __forceinline__ static void store(bf16* p, const float (&f)[4]) {
    uint2 o;
    o.x = pack_bf16x2(f[0], f[1]);
    o.y = pack_bf16x2(f[2], f[3]);
    *reinterpret_cast<uint2*>(p) = o;
  }
};
template <>
struct RowVec<8> {
  uint4 u;
  __device__ __forceinline__ void load(const bf16* p) { u = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void to_float(float (&f)[8]) const { unpack8(u, f); }
  __device__ __forceinline__ static void store(bf16* p, const float (&f)[8]) { *reinterpret_cast<uint4*>(p) = pack8(f); }
};

template <int E, bool W_FP32>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const bf16* __restrict__ qkv, int64_t ldq, const void* __restrict__ qw, const void* __restrict__ kw,
    const int32_t* __restrict__ pos, const float* __restrict__ rope, int max_pos, int rot, bf16* __restrict__ qo,
    bf16* __restrict__ ko, int64_t tokens, int hq, int hkv, float eps) {
  constexpr int D = E * 32;
  constexpr int G = 10;  // rows in flight per warp (hq + hkv = 20 for the decision model: two rounds)
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= tokens) return;
  // per-lane constants of this token
  float wq[E], wk[E], cf[E], sf[E];
  int partner[E];
  int p = pos[t];
  p = p < 0 ? 0 : (p >= max_pos ? max_pos - 1 : p);   // callers guarantee 0 <= pos < max_pos
  const float* cs = rope + (int64_t)p * rot;            // cos[0:half] then sin[0:half]
  const int half = rot >> 1;
  const int lane_off = half / E;                        // rot/2 is a multiple of E (rot % 8 == 0, E <= 8)
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const int f = lane * E + j;
    wq[j] = 1.0f + (W_FP32 ? __ldg(static_cast<const float*>(qw) + f) : __bfloat162float(static_cast<const bf16*>(qw)[f]));
    wk[j] = 1.0f + (W_FP32 ? __ldg(static_cast<const float*>(kw) + f) : __bfloat162float(static_cast<const bf16*>(kw)[f]));
    if (f < rot) {
      const int i = f < half ? f : f - half;
      cf[j] = __ldg(cs + i);
      sf[j] = f < half ? -__ldg(cs + half + i) : __ldg(cs + half + i);
      partner[j] = f < half ? lane + lane_off : lane - lane_off;
    } else {
      cf[j] = 1.f;
      sf[j] = 0.f;
      partner[j] = lane;
    }
  }
  const bf16* row0 = qkv + t * ldq;
  const int nrows = hq + hkv;
  for (int r0 = 0; r0 < nrows; r0 += G) {
    RowVec<E> in[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int r = r0 + g;
      if (r < nrows) in[g].load(row0 + (r < hq ? (int64_t)r * 2 * D : (int64_t)hq * 2 * D + (int64_t)(r - hq) * D) + lane * E);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int r = r0 + g;
      if (r >= nrows) break;  // warp-uniform
      float x[E];
      in[g].to_float(x);
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) ss = fmaf(x[j], x[j], ss);
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)D + eps);
      const bool is_q = r < hq;
#pragma unroll
      for (int j = 0; j < E; ++j) x[j] = x[j] * inv * (is_q ? wq[j] : wk[j]);
      float y[E];
#pragma unroll
      for (int j = 0; j < E; ++j) {
        const float other = __shfl_sync(0xffffffffu, x[j], partner[j]);
        y[j] = fmaf(x[j], cf[j], other * sf[j]);
      }
      bf16* dst = is_q ? qo + (t * hq + r) * D : ko + (t * hkv + (r - hq)) * D;
      RowVec<E>::store(dst + lane * E, y);
    }
  }
}

}  // namespace fdk

using namespace fdk;

extern "C" int fdk_residual_rmsnorm(const void* x, int64_t ld_x, const void* residual, int64_t ld_residual,
                                    int residual_is_fp32, const void* weight, int weight_is_fp32, void* out,
                                    int64_t ld_out, void* residual_out, int64_t ld_residual_out, int64_t rows,
                                    int64_t hidden, float eps, float weight_offset, void* stream) {
  if (int st = check_device()) return st;
  if ((!x && !residual) || !weight || !out) return set_error(FDK_ERR_INVALID_ARGUMENT, "residual_rmsnorm: null pointer");
  if (rows < 0 || hidden <= 0 || hidden % 8 != 0 || hidden > 8192)
    return set_error(FDK_ERR_UNSUPPORTED, "residual_rmsnorm: hidden=%lld must be a positive multiple of 8 <= 8192", (long long)hidden);
  if ((x && ld_x < hidden) || ld_out < hidden || (residual && ld_residual < hidden) || (residual_out && ld_residual_out < hidden))
    return set_error(FDK_ERR_INVALID_ARGUMENT, "residual_rmsnorm: row stride smaller than hidden");
  if ((x && !aligned16(x)) || !aligned16(out) || (residual && !aligned16(residual)) || (residual_out && !aligned16(residual_out)) ||
      !aligned16(weight) || ld_x % 8 || ld_out % 8 || (residual && ld_residual % 8) || (residual_out && ld_residual_out % 8))
    return set_error(FDK_ERR_ALIGNMENT, "residual_rmsnorm: pointers and row strides must be 16-byte aligned");
  if (rows == 0) return FDK_OK;
  if (rows > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "residual_rmsnorm: too many rows");
  dim3 grid((unsigned)rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nc = (int)((hidden / 8 + 127) / 128);
  auto xb = static_cast<const bf16*>(x);
  auto ob = static_cast<bf16*>(out);
  const bool hr = residual != nullptr, w32 = weight_is_fp32 != 0, r32 = residual_is_fp32 != 0;
  switch (nc) {
    case 1: launch_rms_any<1>(r32, hr, w32, grid, s, xb, ld_x, residual, ld_residual, weight, ob, ld_out, residual_out, ld_residual_out, (int)hidden, eps, weight_offset); break;
    case 2: launch_rms_any<2>(r32, hr, w32, grid, s, xb, ld_x, residual, ld_residual, weight, ob, ld_out, residual_out, ld_residual_out, (int)hidden, eps, weight_offset); break;
    case 3:
    case 4: launch_rms_any<4>(r32, hr, w32, grid, s, xb, ld_x, residual, ld_residual, weight, ob, ld_out, residual_out, ld_residual_out, (int)hidden, eps, weight_offset); break;
    default: launch_rms_any<8>(r32, hr, w32, grid, s, xb, ld_x, residual, ld_residual, weight, ob, ld_out, residual_out, ld_residual_out, (int)hidden, eps, weight_offset); break;
  }
  return check_launch("residual_rmsnorm");
}

extern "C" int fdk_gated_rmsnorm(const void* o, const void* z, int64_t ld_z, const void* weight, int weight_is_fp32,
                                 void* out, int64_t tokens, int64_t heads, int64_t dv, float eps, void* stream) {
  if (int st = check_device()) return st;
  if (!o || !z || !weight || !out) return set_error(FDK_ERR_INVALID_ARGUMENT, "gated_rmsnorm: null pointer");
  if (dv != 128) return set_error(FDK_ERR_UNSUPPORTED, "gated_rmsnorm: dv=%lld (only 128 supported)", (long long)dv);
  if (tokens < 0 || heads <= 0 || ld_z < heads * dv) return set_error(FDK_ERR_INVALID_ARGUMENT, "gated_rmsnorm: bad sizes");
  if (!aligned16(o) || !aligned16(z) || !aligned16(out) || ld_z % 8 || !aligned16(weight))
    return set_error(FDK_ERR_ALIGNMENT, "gated_rmsnorm: pointers and strides must be 16-byte aligned");
  const int64_t rows = tokens * heads;
  if (rows == 0) return FDK_OK;
  dim3 grid((unsigned)((rows + 15) / 16));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (weight_is_fp32)
    gated_rmsnorm_kernel<true><<<grid, 256, 0, s>>>(static_cast<const bf16*>(o), static_cast<const bf16*>(z), ld_z, weight, static_cast<bf16*>(out), rows, (int)heads, eps);
  else
    gated_rmsnorm_kernel<false><<<grid, 256, 0, s>>>(static_cast<const bf16*>(o), static_cast<const bf16*>(z), ld_z, weight, static_cast<bf16*>(out), rows, (int)heads, eps);
  return check_launch("gated_rmsnorm");
}

extern "C" int fdk_attn_qk_norm_rope(const void* qkv, int64_t ld_qkv, const void* q_norm_w, const void* k_norm_w,
                                     int weight_is_fp32, const int32_t* positions, const float* rope_table,
                                     int64_t max_pos, int rot_dim,
                                     void* q_out, void* k_out, int64_t tokens, int64_t hq, int64_t hkv, int64_t head_dim,
                                     float eps, void* stream) {
  if (int st = check_device()) return st;
  if (!qkv || !q_norm_w || !k_norm_w || !positions || !rope_table || !q_out || !k_out || max_pos < 1 || max_pos > 0x7fffffff)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "attn_qk_norm_rope: null pointer");
  if (head_dim != 128 && head_dim != 256)
    return set_error(FDK_ERR_UNSUPPORTED, "attn_qk_norm_rope: head_dim=%lld (128 or 256)", (long long)head_dim);
  if (rot_dim <= 0 || rot_dim > head_dim || rot_dim % 8 != 0 || (rot_dim / 2) % (head_dim / 32) != 0)
    return set_error(FDK_ERR_UNSUPPORTED, "attn_qk_norm_rope: rot_dim=%d unsupported", rot_dim);
  if (tokens < 0 || hq <= 0 || hkv <= 0 || ld_qkv < (2 * hq + hkv) * head_dim)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "attn_qk_norm_rope: bad sizes");
  if (!aligned16(qkv) || ld_qkv % 8 || !aligned16(q_out) || !aligned16(k_out))
    return set_error(FDK_ERR_ALIGNMENT, "attn_qk_norm_rope: pointers and strides must be 16-byte aligned");
  if (tokens == 0) return FDK_OK;
  if ((tokens + 7) / 8 > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "attn_qk_norm_rope: too many tokens");
  dim3 grid((unsigned)((tokens + 7) / 8));  // one warp per token
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto in = static_cast<const bf16*>(qkv);
  auto qo = static_cast<bf16*>(q_out);
  auto ko = static_cast<bf16*>(k_out);
  if (head_dim == 128) {
    if (weight_is_fp32) qk_norm_rope_kernel<4, true><<<grid, 256, 0, s>>>(in, ld_qkv, q_norm_w, k_norm_w, positions, rope_table, (int)max_pos, rot_dim, qo, ko, tokens, (int)hq, (int)hkv, eps);
    else qk_norm_rope_kernel<4, false><<<grid, 256, 0, s>>>(in, ld_qkv, q_norm_w, k_norm_w, positions, rope_table, (int)max_pos, rot_dim, qo, ko, tokens, (int)hq, (int)hkv, eps);
  } else {
    if (weight_is_fp32) qk_norm_rope_kernel<8, true><<<grid, 256, 0, s>>>(in, ld_qkv, q_norm_w, k_norm_w, positions, rope_table, (int)max_pos, rot_dim, qo, ko, tokens, (int)hq, (int)hkv, eps);
    else qk_norm_rope_kernel<8, false><<<grid, 256, 0, s>>>(in, ld_qkv, q_norm_w, k_norm_w, positions, rope_table, (int)max_pos, rot_dim, qo, ko, tokens, (int)hq, (int)hkv, eps);
  }
  return check_launch("attn_qk_norm_rope");
}

extern "C" int fdk_rmsnorm_add_partials(const float* partials, int nparts, float* h, int64_t ldh, const void* weight,
                                        int weight_is_fp32, void* out, int64_t ld_out, int64_t rows, int64_t hidden,
                                        float eps, float weight_offset, void* stream) {
  if (int st = check_device()) return st;
  if (!partials || !h || (out && !weight)) return set_error(FDK_ERR_INVALID_ARGUMENT, "rmsnorm_add_partials: null pointer");
  if (nparts < 1 || nparts > 16) return set_error(FDK_ERR_INVALID_ARGUMENT, "rmsnorm_add_partials: nparts in [1, 16]");
  if (rows < 0 || hidden <= 0 || hidden % 8 != 0 || hidden > 4096)
    return set_error(FDK_ERR_UNSUPPORTED, "rmsnorm_add_partials: hidden must be a positive multiple of 8 <= 4096");
  if (ldh < hidden || (out && ld_out < hidden)) return set_error(FDK_ERR_INVALID_ARGUMENT, "rmsnorm_add_partials: row stride too small");
  if (!aligned16(partials) || !aligned16(h) || ldh % 4 || (out && (!aligned16(out) || ld_out % 8 || !aligned16(weight))))
    return set_error(FDK_ERR_ALIGNMENT, "rmsnorm_add_partials: pointers and row strides must be 16-byte aligned");
  if (rows == 0) return FDK_OK;
  if (rows > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "rmsnorm_add_partials: too many rows");
  const dim3 grid((unsigned)rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t plane = rows * hidden;
  auto ob = static_cast<bf16*>(out);
  const int nc = (int)((hidden / 8 + 127) / 128);
  if (nc <= 2) {
    if (weight_is_fp32) rmsnorm_add_partials_kernel<2, true><<<grid, 128, 0, s>>>(partials, nparts, plane, h, ldh, weight, ob, ld_out, (int)hidden, eps, weight_offset);
    else rmsnorm_add_partials_kernel<2, false><<<grid, 128, 0, s>>>(partials, nparts, plane, h, ldh, weight, ob, ld_out, (int)hidden, eps, weight_offset);
  } else {
    if (weight_is_fp32) rmsnorm_add_partials_kernel<4, true><<<grid, 128, 0, s>>>(partials, nparts, plane, h, ldh, weight, ob, ld_out, (int)hidden, eps, weight_offset);
    else rmsnorm_add_partials_kernel<4, false><<<grid, 128, 0, s>>>(partials, nparts, plane, h, ldh, weight, ob, ld_out, (int)hidden, eps, weight_offset);
  }
  return check_launch("rmsnorm_add_partials");
}
