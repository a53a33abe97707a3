// Small elementwise / gather kernels around the hot path: GDN gate transform, token embedding,
// SwiGLU and the slot readout (final norm + restricted logits + masked softmax).
#include <math.h>

#include "common.cuh"

namespace fdk {

__global__ void gdn_gates_kernel(const bf16* __restrict__ a, int64_t lda, const bf16* __restrict__ b, int64_t ldb,
                                 const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                                 float* __restrict__ g, bf16* __restrict__ beta, int64_t tokens, int heads) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= tokens * heads) return;
  const int64_t t = i / heads;
  const int h = (int)(i - t * heads);
  const float av = __bfloat162float(a[t * lda + h]);
  const float bv = __bfloat162float(b[t * ldb + h]);
  g[i] = -expf(A_log[h]) * softplusf_(av + dt_bias[h]);
  beta[i] = __float2bfloat16_rn(sigmoidf_(bv));
}

__global__ void embed_kernel(const int32_t* __restrict__ ids, const bf16* __restrict__ table, int64_t vocab,
                             int hidden, bf16* __restrict__ out, int64_t tokens) {
  const int64_t t = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= tokens) return;
  int64_t id = ids[t];
  if (id < 0 || id >= vocab) id = 0;  // out-of-range ids are rejected on the host; never read out of bounds
  const uint4* src = reinterpret_cast<const uint4*>(table + id * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + t * hidden);
  for (int i = threadIdx.x & 31; i < hidden / 8; i += 32) dst[i] = __ldg(src + i);
}

// One block per token row, threads over 8-wide column groups (no index division); SiLU in the
// one-MUFU tanh form (the two-op form kept the MUFU pipe about half busy at HBM speed).
__global__ void __launch_bounds__(256) swiglu_kernel(const bf16* __restrict__ gu, int64_t ldgu, bf16* __restrict__ out,
                                                     int inter) {
  const int64_t t = blockIdx.x;
  const bf16* row = gu + t * ldgu;
  bf16* orow = out + t * (int64_t)inter;
  for (int c = threadIdx.x * 8; c < inter; c += blockDim.x * 8) {
    float gv[8], uv[8], o[8];
    unpack8(ldg_stream(row + c), gv);
    unpack8(ldg_stream(row + inter + c), uv);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = silu_tanh(gv[j]) * uv[j];
    *reinterpret_cast<uint4*>(orow + c) = pack8(o);
  }
}

// One 256-thread block per slot: RMSNorm (1 + w) of the slot row, K <= 16 restricted logits,
// masked softmax(logits / temperature).
constexpr int READOUT_MAX_H = 8192;

template <bool W_FP32, bool HID_FP32>
__global__ void __launch_bounds__(256) slot_readout_kernel(
    const void* __restrict__ hidden, const bf16* __restrict__ delta, int hsz, const int32_t* __restrict__ slots,
    const int32_t* __restrict__ nopts, const void* __restrict__ fw, const bf16* __restrict__ letters, int K,
    float eps, float temp, float* __restrict__ probs, float* __restrict__ logits, int vec) {
  const int n = blockIdx.x;
  const int64_t r = (int64_t)slots[n] * hsz;
  __shared__ float rowv[READOUT_MAX_H];   // the slot row after the final residual add (bf16 values)
  __shared__ float red[8][17];
  __shared__ float s_inv;
  float ss = 0.f;
  if (vec) {
    // 16-byte aligned rows with hsz % 8 == 0 (the decision model): 8 elements per thread and pass,
    // all of a pass's loads in flight at once (one block per slot: latency, not bandwidth)
    for (int i = threadIdx.x * 8; i < hsz; i += 256 * 8) {
      float x[8], d[8];
      if (HID_FP32) {
        const float4* hp = reinterpret_cast<const float4*>(static_cast<const float*>(hidden) + r + i);
        const float4 a = hp[0], b = hp[1];
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
      } else {
        unpack8(*reinterpret_cast<const uint4*>(static_cast<const bf16*>(hidden) + r + i), x);
      }
      if (delta) {
        unpack8(*reinterpret_cast<const uint4*>(delta + r + i), d);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          x[e] += d[e];
          if (!HID_FP32) x[e] = round_bf16(x[e]);  // the bf16 residual stream rounds the last add
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        rowv[i + e] = x[e];
        ss = fmaf(x[e], x[e], ss);
      }
    }
  } else {
    for (int i = threadIdx.x; i < hsz; i += 256) {
      float x = HID_FP32 ? static_cast<const float*>(hidden)[r + i] : __bfloat162float(static_cast<const bf16*>(hidden)[r + i]);
      if (delta) {
        x += __bfloat162float(delta[r + i]);
        if (!HID_FP32) x = round_bf16(x);
      }
      rowv[i] = x;
      ss = fmaf(x, x, ss);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][16] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w][16];
    s_inv = rsqrtf(t / (float)hsz + eps);
  }
  __syncthreads();
  const float inv = s_inv;
  float acc[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) acc[k] = 0.f;
  if (vec && !W_FP32) {  // (vec also guarantees 16-byte aligned weight and letter rows)
    for (int i = threadIdx.x * 8; i < hsz; i += 256 * 8) {
      float wf[8], hn[8];
      unpack8(*reinterpret_cast<const uint4*>(static_cast<const bf16*>(fw) + i), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) hn[e] = rowv[i + e] * inv * (1.0f + wf[e]);
      uint4 lw[16];
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (k < K) lw[k] = *reinterpret_cast<const uint4*>(letters + (int64_t)k * hsz + i);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        if (k < K) {
          float l[8];
          unpack8(lw[k], l);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[k] = fmaf(hn[e], l[e], acc[k]);
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < hsz; i += 256) {
      const float wf = W_FP32 ? static_cast<const float*>(fw)[i] : __bfloat162float(static_cast<const bf16*>(fw)[i]);
      const float hn = rowv[i] * inv * (1.0f + wf);
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (k < K) acc[k] = fmaf(hn, __bfloat162float(letters[(int64_t)k * hsz + i]), acc[k]);
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    float v = warp_sum(acc[k]);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][k] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int no = nopts[n];
    float lg[16];
    float mx = -INFINITY;
    for (int k = 0; k < K; ++k) {
      float t = 0.f;
      for (int w = 0; w < 8; ++w) t += red[w][k];
      lg[k] = t;
      if (k < no) mx = fmaxf(mx, t / temp);
    }
    float den = 0.f;
    for (int k = 0; k < K; ++k) den += (k < no) ? expf(lg[k] / temp - mx) : 0.f;
    for (int k = 0; k < K; ++k) {
      if (logits) logits[(int64_t)n * K + k] = (k < no) ? lg[k] : -INFINITY;
      probs[(int64_t)n * K + k] = (k < no) ? expf(lg[k] / temp - mx) / den : 0.f;
    }
  }
}

}  // namespace fdk

using namespace fdk;

extern "C" int fdk_gdn_gates(const void* a, int64_t ld_a, const void* b, int64_t ld_b, const float* A_log,
                             const float* dt_bias, float* g, void* beta, int64_t tokens, int64_t heads, void* stream) {
  if (int st = check_device()) return st;
  if (!a || !b || !A_log || !dt_bias || !g || !beta) return set_error(FDK_ERR_INVALID_ARGUMENT, "gdn_gates: null pointer");
  if (tokens < 0 || heads <= 0 || ld_a < heads || ld_b < heads) return set_error(FDK_ERR_INVALID_ARGUMENT, "gdn_gates: bad sizes");
  const int64_t n = tokens * heads;
  if (n == 0) return FDK_OK;
  gdn_gates_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(a), ld_a, static_cast<const bf16*>(b), ld_b, A_log, dt_bias, g, static_cast<bf16*>(beta), tokens, (int)heads);
  return check_launch("gdn_gates");
}

extern "C" int fdk_embed(const int32_t* ids, const void* table, int64_t vocab, int64_t hidden, void* out, int64_t tokens,
                         void* stream) {
  if (int st = check_device()) return st;
  if (!ids || !table || !out) return set_error(FDK_ERR_INVALID_ARGUMENT, "embed: null pointer");
  if (hidden <= 0 || hidden % 8 || vocab <= 0 || tokens < 0) return set_error(FDK_ERR_INVALID_ARGUMENT, "embed: bad sizes");
  if (!aligned16(table) || !aligned16(out)) return set_error(FDK_ERR_ALIGNMENT, "embed: pointers must be 16-byte aligned");
  if (tokens == 0) return FDK_OK;
  embed_kernel<<<(unsigned)((tokens + 3) / 4), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      ids, static_cast<const bf16*>(table), vocab, (int)hidden, static_cast<bf16*>(out), tokens);
  return check_launch("embed");
}

extern "C" int fdk_swiglu(const void* gu, int64_t ld_gu, void* out, int64_t tokens, int64_t inter, void* stream) {
  if (int st = check_device()) return st;
  if (!gu || !out) return set_error(FDK_ERR_INVALID_ARGUMENT, "swiglu: null pointer");
  if (inter <= 0 || inter % 8 || tokens < 0 || ld_gu < 2 * inter) return set_error(FDK_ERR_INVALID_ARGUMENT, "swiglu: bad sizes");
  if (!aligned16(gu) || !aligned16(out) || ld_gu % 8) return set_error(FDK_ERR_ALIGNMENT, "swiglu: 16-byte alignment");
  if (tokens == 0 || inter == 0) return FDK_OK;
  if (tokens > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "swiglu: too many tokens");
  const int threads = (int)(inter / 8 < 256 ? ((inter / 8 + 31) / 32) * 32 : 256);
  swiglu_kernel<<<(unsigned)tokens, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(gu), ld_gu, static_cast<bf16*>(out), (int)inter);
  return check_launch("swiglu");
}

extern "C" int fdk_slot_readout(const void* hidden, int hidden_is_fp32, const void* delta, int64_t hidden_size, const int32_t* slots,
                                const int32_t* nopts, int64_t num_slots, const void* final_norm_w, int weight_is_fp32,
                                const void* letters, int64_t num_letters, float eps, float temperature, float* probs,
                                float* logits, void* stream) {
  if (int st = check_device()) return st;
  if (!hidden || !slots || !nopts || !final_norm_w || !letters || !probs)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "slot_readout: null pointer");
  if (num_letters < 1 || num_letters > 16) return set_error(FDK_ERR_UNSUPPORTED, "slot_readout: 1..16 letters supported");
  if (hidden_size <= 0 || hidden_size > READOUT_MAX_H || num_slots < 0 || !(temperature > 0.f))
    return set_error(FDK_ERR_INVALID_ARGUMENT, "slot_readout: bad sizes (hidden_size <= %d)", READOUT_MAX_H);
  if (num_slots == 0) return FDK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto db = static_cast<const bf16*>(delta);
  auto lb = static_cast<const bf16*>(letters);
  const unsigned g = (unsigned)num_slots;
  const int H = (int)hidden_size, K = (int)num_letters;
  const int vec = (H % 8 == 0) && aligned16(hidden) && (!delta || aligned16(delta)) && aligned16(final_norm_w) &&
                  aligned16(letters);
  if (weight_is_fp32) {
    if (hidden_is_fp32) slot_readout_kernel<true, true><<<g, 256, 0, s>>>(hidden, db, H, slots, nopts, final_norm_w, lb, K, eps, temperature, probs, logits, vec);
    else slot_readout_kernel<true, false><<<g, 256, 0, s>>>(hidden, db, H, slots, nopts, final_norm_w, lb, K, eps, temperature, probs, logits, vec);
  } else {
    if (hidden_is_fp32) slot_readout_kernel<false, true><<<g, 256, 0, s>>>(hidden, db, H, slots, nopts, final_norm_w, lb, K, eps, temperature, probs, logits, vec);
    else slot_readout_kernel<false, false><<<g, 256, 0, s>>>(hidden, db, H, slots, nopts, final_norm_w, lb, K, eps, temperature, probs, logits, vec);
  }
  return check_launch("slot_readout");
}
