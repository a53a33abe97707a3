// Packed depthwise causal conv1d (width <= 4) + SiLU writing q/k/v in [tokens, H, D] layout.
//
// HBM-bound: every input byte is read once (plus a 3-row halo per 64-token tile, an L2 hit) and
// every output byte written once.  The [B, T, C] projection is read with 16-byte cp.async into
// shared-memory tiles that carry the causal halo, the 4 taps stay in registers, and q/k/v are
// written directly in the layout the delta rule reads.  Segment starts (packed varlen) reset the
// history to zero.
#include "common.cuh"

namespace fdk {

constexpr int CONV_THREADS = 128;

__device__ __forceinline__ int64_t segment_start(const int32_t* cu, int nseg, int64_t t) {
  int lo = 0, hi = nseg;  // largest cu[i] <= t (cu[0] = 0)
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return cu[lo];
}

__device__ __forceinline__ int64_t next_start(const int32_t* cu, int nseg, int64_t t) {
  if (cu[nseg] <= t) return INT64_MAX;  // smallest cu[i] > t
  int lo = 0, hi = nseg;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (cu[mid] > t) hi = mid; else lo = mid + 1;
  }
  return cu[lo];
}

// Shared-memory staged kernel: a CTA owns a 128-channel column block and `tpc` (1-4) consecutive
// 64-token tiles -- as many as keep every SM's six CTA slots busy in one wave (small inputs such
// as one 2048-token request get one or two tiles a CTA, so more loads are in flight at once).  Tile rows [t0 - 3, t0 + 64) (the 3-row causal halo included) stream
// into shared memory with cp.async, double-buffered, so the next tile's 16-byte loads are in flight
// while the current one is convolved.  Thread (cq, rg) computes 8 channels x 8 rows with the taps
// in registers (16-byte shared loads and global stores); a half-warp stores 256 contiguous bytes
// per row.  SiLU uses the one-MUFU tanh form: the MUFU pipe, not HBM, bounded the two-op form.
constexpr int CONV_CB = 128;            // channels per CTA
constexpr int CONV_ROWS = 64;           // tokens per tile
constexpr int CONV_HALO = 3;
constexpr int CONV_MAX_TILES_PER_CTA = 4;
constexpr int CONV_CTAS_PER_SM = 6;
constexpr int64_t CONV_DIRECT_MAX_TOKENS = 8192;  // up to this many tokens the direct kernel runs
constexpr int CONV_DIRECT_RPT = 8;  // tokens per thread of the direct kernel (16 measured slower: 14.2 vs 13.0 us at config 2)
constexpr int CONV_SROWS = CONV_ROWS + CONV_HALO;
constexpr int CONV_RPT = 8;             // rows per thread

template <int KW>
__global__ void __launch_bounds__(CONV_THREADS, 6) packed_conv_silu_smem_kernel(
    const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ w, int64_t ntok, int64_t period,
    const int32_t* __restrict__ cu, int nseg, int channels, int key_dim, bf16* __restrict__ q,
    bf16* __restrict__ k, bf16* __restrict__ v, int tpc) {
  __shared__ __align__(16) bf16 tile[2][CONV_SROWS][CONV_CB];
  __shared__ long long seg_info[CONV_ROWS / CONV_RPT][2];  // per row group: segment start, next start
  const int tid = threadIdx.x;
  const int cb0 = blockIdx.x * CONV_CB;
  const int cq = tid & 15, rg = tid >> 4;   // 8 channels, 8 rows
  const int c0 = cb0 + cq * 8;
  const int64_t first = (int64_t)blockIdx.y * tpc;
  const int64_t ntiles = (ntok + CONV_ROWS - 1) / CONV_ROWS;
  const int64_t last = (first + tpc < ntiles) ? first + tpc : ntiles;
  if (first >= last) return;

  auto issue = [&](int64_t ti, int b) {
    const int64_t base = ti * CONV_ROWS - CONV_HALO;
    for (int e = tid; e < CONV_SROWS * (CONV_CB / 8); e += CONV_THREADS) {
      const int r = e >> 4, ch = (e & 15) * 8;
      const int64_t t = base + r;
      const bool ok = t >= 0 && t < ntok && cb0 + ch < channels;
      const bf16* src = x + (ok ? t : 0) * ldx + (ok ? cb0 + ch : 0);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"((uint32_t)__cvta_generic_to_shared(&tile[b][r][ch])),
                   "l"(src), "r"(ok ? 16 : 0));
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };

  const bool active = c0 < channels;  // the last column block may be partial (threads still sync)
  float wr[KW][8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const bf16* wc = w + (int64_t)(active ? c0 + c : 0) * KW;
#pragma unroll
    for (int j = 0; j < KW; ++j) wr[j][c] = __bfloat162float(wc[j]);
  }
  bf16* dst;
  int64_t ldd;
  int cc;
  if (c0 < key_dim) { dst = q; ldd = key_dim; cc = c0; }
  else if (c0 < 2 * key_dim) { dst = k; ldd = key_dim; cc = c0 - key_dim; }
  else { dst = v; ldd = channels - 2 * key_dim; cc = c0 - 2 * key_dim; }

  issue(first, 0);
  for (int64_t ti = first; ti < last; ++ti) {
    const int b = (int)((ti - first) & 1);
    if (tid < CONV_ROWS / CONV_RPT) {  // segment bounds of the 8 row groups, found once per tile
      const int64_t rg0 = ti * CONV_ROWS + tid * CONV_RPT;
      if (rg0 < ntok) {
        if (cu != nullptr) {
          seg_info[tid][0] = segment_start(cu, nseg, rg0);
          seg_info[tid][1] = next_start(cu, nseg, rg0);
        } else {
          seg_info[tid][0] = (rg0 / period) * period;
          seg_info[tid][1] = seg_info[tid][0] + period;
        }
      }
    }
    if (ti + 1 < last) {
      issue(ti + 1, b ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();
    const int64_t r0 = ti * CONV_ROWS + rg * CONV_RPT;   // first output token of this thread
    if (active && r0 < ntok) {  // predicated, never around a barrier: every thread reaches both __syncthreads
      const int64_t seg0 = seg_info[rg][0];
      int64_t nxt = seg_info[rg][1];
      float hist[3][8];
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const int64_t t = r0 - 3 + j;
        if (t >= seg0) unpack8(*reinterpret_cast<const uint4*>(&tile[b][rg * CONV_RPT + j][cq * 8]), hist[j]);
        else {
#pragma unroll
          for (int c = 0; c < 8; ++c) hist[j][c] = 0.f;
        }
      }
      bf16* out = dst + r0 * ldd + cc;
      const bf16* srow = &tile[b][rg * CONV_RPT + CONV_HALO][cq * 8];
      // the 8 rows lie inside one segment and inside the batch: no per-row checks
      const bool plain = nxt >= r0 + CONV_RPT && r0 + CONV_RPT <= ntok;
#pragma unroll
      for (int i = 0; i < CONV_RPT; ++i) {
        const int64_t t = r0 + i;
        if (!plain) {
          if (t >= ntok) break;
          if (t == nxt) {
#pragma unroll
            for (int j = 0; j < 3; ++j)
#pragma unroll
              for (int c = 0; c < 8; ++c) hist[j][c] = 0.f;
            nxt = (cu != nullptr) ? next_start(cu, nseg, t) : nxt + period;
          }
        }
        float cur[8], y[8];
        unpack8(*reinterpret_cast<const uint4*>(srow + i * CONV_CB), cur);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float acc = wr[KW - 1][c] * cur[c];
          if (KW >= 2) acc = fmaf(wr[KW - 2][c], hist[2][c], acc);
          if (KW >= 3) acc = fmaf(wr[KW - 3][c], hist[1][c], acc);
          if (KW >= 4) acc = fmaf(wr[KW - 4][c], hist[0][c], acc);
          y[c] = silu_tanh(acc);
        }
        *reinterpret_cast<uint4*>(out + i * ldd) = pack8(y);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          hist[0][c] = hist[1][c];
          hist[1][c] = hist[2][c];
          hist[2][c] = cur[c];
        }
      }
    }
    __syncthreads();  // buffer b is refilled by the issue() two tiles ahead
  }
}

// Direct kernel for small inputs (a few thousand tokens: the staged kernel cannot fill the SMs'
// load pipes there).  Thread = 8 channels x 8 consecutive tokens; a warp covers 256 contiguous
// channels of one row group, a CTA four row groups.  All 11 rows a thread needs (the 3-row causal
// halo included; halo rows are L2 hits) are loaded with independent 16-byte loads before any
// arithmetic, so every thread has its whole input in flight at once.  Channel pairs use the packed
// fp32 pipe (fma.rn.f32x2): the same roundings per lane as the scalar chain of the staged kernel.
template <int KW, int RPT>
__global__ void __launch_bounds__(128) packed_conv_silu_direct_kernel(
    const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ w, int64_t ntok, int64_t period,
    const int32_t* __restrict__ cu, int nseg, int channels, int key_dim, bf16* __restrict__ q,
    bf16* __restrict__ k, bf16* __restrict__ v) {
  const int lane = threadIdx.x & 31, wg = threadIdx.x >> 5;
  const int c0 = (blockIdx.x * 32 + lane) * 8;
  const int64_t r0 = ((int64_t)blockIdx.y * 4 + wg) * RPT;
  if (c0 >= channels || r0 >= ntok) return;  // no barriers below
  int64_t seg0, nxt;
  if (cu != nullptr) {
    seg0 = segment_start(cu, nseg, r0);
    nxt = next_start(cu, nseg, r0);
  } else {
    seg0 = (r0 / period) * period;
    nxt = seg0 + period;
  }
  uint4 raw[RPT + CONV_HALO];
#pragma unroll
  for (int j = 0; j < RPT + CONV_HALO; ++j) {
    const int64_t t = r0 - CONV_HALO + j;
    raw[j] = (t >= seg0 && t < ntok) ? ldg_stream(x + t * ldx + c0) : make_uint4(0u, 0u, 0u, 0u);
  }
  float2 wr[KW][4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    if (KW == 4) {  // 2 channels x 4 taps = one aligned 16-byte load
      float f[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(w + (int64_t)(c0 + 2 * p) * KW)), f);
#pragma unroll
      for (int j = 0; j < KW; ++j) wr[j][p] = make_float2(f[j], f[KW + j]);
    } else {
#pragma unroll
      for (int j = 0; j < KW; ++j)
        wr[j][p] = make_float2(__bfloat162float(w[(int64_t)(c0 + 2 * p) * KW + j]),
                               __bfloat162float(w[(int64_t)(c0 + 2 * p + 1) * KW + j]));
    }
  }
  bf16* dst;
  int64_t ldd;
  int cc;
  if (c0 < key_dim) { dst = q; ldd = key_dim; cc = c0; }
  else if (c0 < 2 * key_dim) { dst = k; ldd = key_dim; cc = c0 - key_dim; }
  else { dst = v; ldd = channels - 2 * key_dim; cc = c0 - 2 * key_dim; }
  auto as2 = [](const uint4& u, int p) {
    const uint32_t b = p == 0 ? u.x : p == 1 ? u.y : p == 2 ? u.z : u.w;
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b));
  };
  const float2 half2 = make_float2(0.5f, 0.5f);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int64_t t = r0 + i;
    if (t >= ntok) break;
    if (t == nxt) {  // a segment starts inside this row group: earlier rows are not its history
#pragma unroll
      for (int j = 0; j < CONV_HALO + i; ++j) raw[j] = make_uint4(0u, 0u, 0u, 0u);
      nxt = (cu != nullptr) ? next_start(cu, nseg, t) : nxt + period;
    }
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float2 acc = __fmul2_rn(wr[KW - 1][p], as2(raw[CONV_HALO + i], p));
#pragma unroll
      for (int j = 1; j < KW; ++j) acc = __ffma2_rn(wr[KW - 1 - j][p], as2(raw[CONV_HALO + i - j], p), acc);
      const float2 hh = __fmul2_rn(half2, acc);  // silu(x) = h + h tanh(h), h = x / 2
      const float2 y = __ffma2_rn(hh, make_float2(tanh_approx(hh.x), tanh_approx(hh.y)), hh);
      o[p] = pack_bf16x2(y.x, y.y);
    }
    *reinterpret_cast<uint4*>(dst + t * ldd + cc) = out;
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
  const int64_t tiles = (ntok + CONV_ROWS - 1) / CONV_ROWS;
  const int64_t cblocks = (channels + CONV_CB - 1) / CONV_CB;
  const int64_t slots = (int64_t)sm_count() * CONV_CTAS_PER_SM;
  const int64_t want = (tiles * cblocks + slots - 1) / slots;  // tiles per CTA for one wave
  const int tpc = (int)(want < 1 ? 1 : want > CONV_MAX_TILES_PER_CTA ? CONV_MAX_TILES_PER_CTA : want);
  const int64_t groups = (tiles + tpc - 1) / tpc;
  if (groups > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "packed_conv: too many tokens");
  dim3 grid((unsigned)cblocks, (unsigned)groups);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto xb = static_cast<const bf16*>(x);
  auto wb = static_cast<const bf16*>(weight);
  auto qb = static_cast<bf16*>(q);
  auto kb = static_cast<bf16*>(k);
  auto vb = static_cast<bf16*>(v);
  const int nseg = (int)num_segments;
  static bool carveout_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !carveout_set[dev]) {
    // 34 KB of static shared memory per CTA: ask for the full carveout so six CTAs fit per SM
    cudaFuncSetAttribute(packed_conv_silu_smem_kernel<4>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(packed_conv_silu_smem_kernel<3>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(packed_conv_silu_smem_kernel<2>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(packed_conv_silu_smem_kernel<1>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (dev >= 0 && dev < 64) carveout_set[dev] = true;
  }
  if (ntok <= CONV_DIRECT_MAX_TOKENS) {
    constexpr int R = CONV_DIRECT_RPT;
    const dim3 dgrid((unsigned)((channels / 8 + 31) / 32), (unsigned)((ntok + 4 * R - 1) / (4 * R)));
    switch (kernel_width) {
      case 4: packed_conv_silu_direct_kernel<4, R><<<dgrid, 128, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb); break;
      case 3: packed_conv_silu_direct_kernel<3, R><<<dgrid, 128, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb); break;
      case 2: packed_conv_silu_direct_kernel<2, R><<<dgrid, 128, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb); break;
      default: packed_conv_silu_direct_kernel<1, R><<<dgrid, 128, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb); break;
    }
    return check_launch("packed_conv_silu");
  }
  switch (kernel_width) {
    case 4: packed_conv_silu_smem_kernel<4><<<grid, CONV_THREADS, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb, tpc); break;
    case 3: packed_conv_silu_smem_kernel<3><<<grid, CONV_THREADS, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb, tpc); break;
    case 2: packed_conv_silu_smem_kernel<2><<<grid, CONV_THREADS, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb, tpc); break;
    default: packed_conv_silu_smem_kernel<1><<<grid, CONV_THREADS, 0, s>>>(xb, ld_x, wb, ntok, seqlen, cu_seqlens, nseg, (int)channels, (int)key_dim, qb, kb, vb, tpc); break;
  }
  return check_launch("packed_conv_silu");
}
