// Packed depthwise causal conv1d (width <= 4) + SiLU writing q/k/v in [tokens, H, D] layout.
//
// Each thread owns 8 consecutive channels (one 16-byte vector) and walks TT consecutive tokens,
// keeping the last three input rows of its channels in registers: every input byte is read
// once (plus a 3-row halo per TT-token tile) and every output byte written once, so the kernel
// runs at HBM speed.  A warp covers 256 contiguous channels, so loads and stores are fully
// coalesced 512-byte rows.  Segment starts (packed varlen) reset the history to zero.
#include "common.cuh"

namespace fdk {

constexpr int CONV_TT = 16;       // tokens per thread
constexpr int CONV_THREADS = 128;

__device__ __forceinline__ int64_t segment_start(const int32_t* cu, int nseg, int64_t t) {
  // largest cu[i] <= t
  int lo = 0, hi = nseg;  // cu[0] = 0 <= t
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return cu[lo];
}

__device__ __forceinline__ int64_t next_start(const int32_t* cu, int nseg, int64_t t) {
  // smallest cu[i] > t (or a sentinel past the end)
  int lo = 0, hi = nseg;
  if (cu[nseg] <= t) return INT64_MAX;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (cu[mid] > t) hi = mid; else lo = mid + 1;
  }
  return cu[lo];
}

template <int KW>
__global__ void __launch_bounds__(CONV_THREADS) packed_conv_silu_kernel(
    const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ w, int64_t ntok, int64_t period,
    const int32_t* __restrict__ cu, int nseg, int channels, int key_dim, bf16* __restrict__ q,
    bf16* __restrict__ k, bf16* __restrict__ v) {
  const int cvec = blockIdx.x * CONV_THREADS + threadIdx.x;  // 8-channel group
  if (cvec * 8 >= channels) return;
  const int c0 = cvec * 8;
  const int64_t t0 = (int64_t)blockIdx.y * CONV_TT;
  if (t0 >= ntok) return;
  const int64_t t1 = (t0 + CONV_TT < ntok) ? t0 + CONV_TT : ntok;

  // weights of my 8 channels, tap j multiplies x[t - (KW-1) + j]
  float wr[KW][8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const bf16* wc = w + (int64_t)(c0 + c) * KW;
#pragma unroll
    for (int j = 0; j < KW; ++j) wr[j][c] = __bfloat162float(wc[j]);
  }
  // destination: q / k / v region of this channel group (groups never straddle regions)
  bf16* dst;
  int64_t ldd;
  int cc;
  if (c0 < key_dim) { dst = q; ldd = key_dim; cc = c0; }
  else if (c0 < 2 * key_dim) { dst = k; ldd = key_dim; cc = c0 - key_dim; }
  else { dst = v; ldd = channels - 2 * key_dim; cc = c0 - 2 * key_dim; }

  int64_t seg0, nxt;
  if (cu != nullptr) {
    seg0 = segment_start(cu, nseg, t0);
    nxt = next_start(cu, nseg, t0);
  } else {
    seg0 = (t0 / period) * period;
    nxt = seg0 + period;
  }
  // history rows x[t0-3], x[t0-2], x[t0-1] (zero before the segment start)
  float hist[3][8];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int64_t t = t0 - 3 + j;
    if (t >= seg0) unpack8(ldg_stream(x + t * ldx + c0), hist[j]);
    else {
#pragma unroll
      for (int c = 0; c < 8; ++c) hist[j][c] = 0.f;
    }
  }
  uint4 raw[CONV_TT];
#pragma unroll
  for (int i = 0; i < CONV_TT; ++i) {
    const int64_t t = t0 + i;
    if (t < t1) raw[i] = ldg_stream(x + t * ldx + c0);
  }
#pragma unroll
  for (int i = 0; i < CONV_TT; ++i) {
    const int64_t t = t0 + i;
    if (t >= t1) break;
    if (t == nxt) {  // a new segment starts here: forget the history
#pragma unroll
      for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int c = 0; c < 8; ++c) hist[j][c] = 0.f;
      if (cu != nullptr) nxt = next_start(cu, nseg, t);
      else nxt += period;
    }
    float cur[8], y[8];
    unpack8(raw[i], cur);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float acc = wr[KW - 1][c] * cur[c];
      if (KW >= 2) acc = fmaf(wr[KW - 2][c], hist[2][c], acc);
      if (KW >= 3) acc = fmaf(wr[KW - 3][c], hist[1][c], acc);
      if (KW >= 4) acc = fmaf(wr[KW - 4][c], hist[0][c], acc);
      y[c] = silu(acc);
    }
    *reinterpret_cast<uint4*>(dst + t * ldd + cc) = pack8(y);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      hist[0][c] = hist[1][c];
      hist[1][c] = hist[2][c];
      hist[2][c] = cur[c];
    }
  }
}

}  // namespace fdk

using namespace fdk;

extern "C" int fdk_packed_conv_silu(const void* x, int64_t ld_x, const void* weight, int64_t batch, int64_t seqlen,
                                    int64_t channels, int kernel_width, const int32_t* cu_seqlens, int64_t num_segments,
                                    int64_t key_dim, int64_t value_dim, void* q, void* k, void* v, void* stream) {
  if (int st = check_device()) return st;
  if (!x || !weight || !q || !k || !v) return set_error(FDK_ERR_INVALID_ARGUMENT, "packed_conv: null pointer");
  if (batch < 0 || seqlen < 0 || channels <= 0 || key_dim <= 0 || value_dim <= 0 || channels != 2 * key_dim + value_dim)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "packed_conv: channels=%lld must equal 2*key_dim + value_dim", (long long)channels);
  if (kernel_width < 1 || kernel_width > 4)
    return set_error(FDK_ERR_UNSUPPORTED, "packed_conv: kernel_width=%d (1..4 supported)", kernel_width);
  if (key_dim % 8 || value_dim % 8) return set_error(FDK_ERR_UNSUPPORTED, "packed_conv: key/value dims must be multiples of 8");
  if (ld_x < channels) return set_error(FDK_ERR_INVALID_ARGUMENT, "packed_conv: ld_x < channels");
  if (!aligned16(x) || ld_x % 8 || !aligned16(q) || !aligned16(k) || !aligned16(v))
    return set_error(FDK_ERR_ALIGNMENT, "packed_conv: pointers and row stride must be 16-byte aligned");
  if (cu_seqlens && batch != 1) return set_error(FDK_ERR_INVALID_ARGUMENT, "packed_conv: cu_seqlens needs batch == 1");
  if (cu_seqlens && num_segments < 1) return set_error(FDK_ERR_INVALID_ARGUMENT, "packed_conv: num_segments < 1");
  const int64_t ntok = batch * seqlen;
  if (ntok == 0) return FDK_OK;
  const int64_t tiles = (ntok + CONV_TT - 1) / CONV_TT;
  if (tiles > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "packed_conv: too many tokens");
  dim3 grid((unsigned)((channels / 8 + CONV_THREADS - 1) / CONV_THREADS), (unsigned)tiles);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto xb = static_cast<const bf16*>(x);
  auto wb = static_cast<const bf16*>(weight);
  auto qb = static_cast<bf16*>(q);
  auto kb = static_cast<bf16*>(k);
  auto vb = static_cast<bf16*>(v);
  const int nseg = (int)num_segments;
  switch (kernel_width) {
    case 4: packed_conv_silu_kernel<4><<<grid, CONV_THREADS, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb); break;
    case 3: packed_conv_silu_kernel<3><<<grid, CONV_THREADS, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb); break;
    case 2: packed_conv_silu_kernel<2><<<grid, CONV_THREADS, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb); break;
    default: packed_conv_silu_kernel<1><<<grid, CONV_THREADS, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb); break;
  }
  return check_launch("packed_conv_silu");
}
