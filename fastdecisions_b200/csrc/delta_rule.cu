// Chunked gated delta rule (Gated DeltaNet core), chunk = 64 tokens, dk = dv = 128.
//
// Restates transformers' torch_chunk_gated_delta_rule (models/qwen3_5/modeling_qwen3_5.py:234-311)
// for packed varlen input.  Three launches:
//   1. chunk_table_kernel   : per-segment chunk offsets (device side, graph-capturable).
//   2. delta_prep_kernel    : one CTA per (chunk, head), fully parallel.  l2-normalises q and k,
//      takes the in-chunk cumsum G of the log decay, forms KK^T and QK^T on the tensor cores,
//      inverts the unit-lower-triangular (I - L) in fp32 (16x16 diagonal blocks by forward
//      substitution, then block forward substitution), and produces
//        W  = T diag(beta e^G) K        U  = T diag(beta) V
//        Qg = q e^G                     Kg = k e^(G_last - G)       Aqk = (QK^T o decay), lower
//      into the caller's workspace (bf16), plus gamma = e^(G_last) per chunk.
//   3. delta_recur_kernel   : one CTA per (segment, head, 32-wide dv block), sequential over the
//      segment's chunks with the fp32 state S [128 x 32] in registers:
//        v_new = U - W S ;  o = Qg S + Aqk v_new ;  S = gamma S + Kg^T v_new
//      while the next chunk's tiles stream into shared memory with cp.async.
#include "common.cuh"
#include "mma_sm80.cuh"

namespace fdk {

constexpr int DR_C = 64;    // chunk length
constexpr int DR_D = 128;   // dk == dv
constexpr int DR_BV = 32;   // dv columns per recurrence CTA
constexpr int LD128 = DR_D + 8;  // padded smem row (bf16) for 128-wide tiles
constexpr int LD64 = DR_C + 8;   // padded smem row (bf16) for 64-wide tiles

// Per (chunk, head) workspace tile: W, U, Qg, Kg [64][128] bf16, Aqk [64][64] bf16, gamma f32.
constexpr size_t TILE128 = (size_t)DR_C * DR_D * 2;
constexpr size_t TILE64 = (size_t)DR_C * DR_C * 2;
constexpr size_t CH_BYTES = 4 * TILE128 + TILE64 + 16;

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct WsLayout {
  size_t off_table, off_tiles, total;
  int64_t max_chunks;
};

__host__ __device__ inline WsLayout ws_layout(int64_t tokens, int64_t nseg, int64_t heads) {
  WsLayout l;
  l.max_chunks = (tokens + DR_C - 1) / DR_C + nseg;
  l.off_table = 0;
  l.off_tiles = align256((size_t)(nseg + 1) * 4);
  l.total = l.off_tiles + align256((size_t)l.max_chunks * heads * CH_BYTES);
  return l;
}

__global__ void chunk_table_kernel(const int32_t* __restrict__ cu, int nseg, int32_t* __restrict__ table) {
  // single warp: exclusive scan of ceil(len / 64) over segments
  const int lane = threadIdx.x;
  int carry = 0;
  for (int base = 0; base < nseg; base += 32) {
    const int s = base + lane;
    int n = 0;
    if (s < nseg) {
      const int len = cu[s + 1] - cu[s];
      n = len > 0 ? (len + DR_C - 1) / DR_C : 0;
    }
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (s < nseg) table[s] = carry + incl - n;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) table[nseg] = carry;
}

struct PrepSmem {
  __nv_bfloat16 q[DR_C][LD128];
  __nv_bfloat16 k[DR_C][LD128];
  __nv_bfloat16 v[DR_C][LD128];
  __nv_bfloat16 tu[DR_C][LD64];   // bf16(T * beta_col)
  __nv_bfloat16 tw[DR_C][LD64];   // bf16(T * (beta e^G)_col)
  float L[DR_C][DR_C + 1];        // strictly lower L, then reused for the block solve
  float T[DR_C][DR_C + 1];
  float G[DR_C];
  float beta[DR_C];
  int info[3];
};

__global__ void __launch_bounds__(128) delta_prep_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, int64_t ldqk, const bf16* __restrict__ v, int64_t ldv,
    const float* __restrict__ g, const bf16* __restrict__ beta, const int32_t* __restrict__ cu, int nseg,
    const int32_t* __restrict__ table, int heads, float scale, uint8_t* __restrict__ tiles) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(smem_raw);
  const int ci = blockIdx.x;
  const int h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (ci >= table[nseg]) return;
  if (tid == 0) {
    int lo = 0, hi = nseg - 1;  // segment s with table[s] <= ci < table[s+1]
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (table[mid] <= ci) lo = mid; else hi = mid - 1;
    }
    // skip empty segments that share the same table value
    while (lo + 1 <= nseg - 1 && table[lo + 1] <= ci) ++lo;
    const int t0 = cu[lo] + (ci - table[lo]) * DR_C;
    sm.info[0] = t0;
    sm.info[1] = min(DR_C, cu[lo + 1] - t0);
  }
  __syncthreads();
  const int t0 = sm.info[0], len = sm.info[1];

  // 1. load q, k, v rows (zero past len), decay and beta
  for (int i = tid; i < DR_C * 16; i += 128) {
    const int r = i >> 4, c = (i & 15) * 8;
    uint4 zq = make_uint4(0, 0, 0, 0), zk = zq, zv = zq;
    if (r < len) {
      const int64_t t = t0 + r;
      zq = *reinterpret_cast<const uint4*>(q + t * ldqk + (int64_t)h * DR_D + c);
      zk = *reinterpret_cast<const uint4*>(k + t * ldqk + (int64_t)h * DR_D + c);
      zv = *reinterpret_cast<const uint4*>(v + t * ldv + (int64_t)h * DR_D + c);
    }
    *reinterpret_cast<uint4*>(&sm.q[r][c]) = zq;
    *reinterpret_cast<uint4*>(&sm.k[r][c]) = zk;
    *reinterpret_cast<uint4*>(&sm.v[r][c]) = zv;
  }
  if (warp == 0) {
    // inclusive cumsum of g over the chunk (padding rows contribute 0), 2 values per lane
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
    const int r0 = 2 * lane, r1 = 2 * lane + 1;
    if (r0 < len) { a0 = g[(int64_t)(t0 + r0) * heads + h]; b0 = __bfloat162float(beta[(int64_t)(t0 + r0) * heads + h]); }
    if (r1 < len) { a1 = g[(int64_t)(t0 + r1) * heads + h]; b1 = __bfloat162float(beta[(int64_t)(t0 + r1) * heads + h]); }
    float pair = a0 + a1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const float excl = incl - pair;
    sm.G[r0] = excl + a0;
    sm.G[r1] = excl + a0 + a1;
    sm.beta[r0] = b0;
    sm.beta[r1] = b1;
  }
  __syncthreads();

  // 2. l2 norm rows of q (times scale) and k in fp32, written back as bf16
  for (int r = warp; r < 2 * DR_C; r += 4) {
    __nv_bfloat16* row = (r < DR_C) ? sm.q[r] : sm.k[r - DR_C];
    float x[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = __bfloat162float(row[lane * 4 + j]);
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss + 1e-6f) * (r < DR_C ? scale : 1.0f);
#pragma unroll
    for (int j = 0; j < 4; ++j) row[lane * 4 + j] = __float2bfloat16_rn(x[j] * inv);
  }
  __syncthreads();

  // 3. KK^T and QK^T for rows [16w, 16w+16) on the tensor cores
  const int gq = lane >> 2, tq = lane & 3;
  float kk[8][4], qk[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int j = 0; j < 4; ++j) kk[n][j] = qk[n][j] = 0.f;
#pragma unroll
  for (int ks = 0; ks < DR_D; ks += 16) {
    uint32_t ak[4], aq[4];
    load_a(&sm.k[0][0], LD128, warp * 16, ks, ak);
    load_a(&sm.q[0][0], LD128, warp * 16, ks, aq);
#pragma unroll
    for (int n = 0; n < 8; n += 2) {
      uint32_t b[4];
      load_b_nk(&sm.k[0][0], LD128, n * 8, ks, b);
      mma_bf16_16816(kk[n], ak, b[0], b[1]);
      mma_bf16_16816(kk[n + 1], ak, b[2], b[3]);
      mma_bf16_16816(qk[n], aq, b[0], b[1]);
      mma_bf16_16816(qk[n + 1], aq, b[2], b[3]);
    }
  }
  uint8_t* tile = tiles + ((size_t)ci * heads + h) * CH_BYTES;
  __nv_bfloat16* wsW = reinterpret_cast<__nv_bfloat16*>(tile);
  __nv_bfloat16* wsU = reinterpret_cast<__nv_bfloat16*>(tile + TILE128);
  __nv_bfloat16* wsQg = reinterpret_cast<__nv_bfloat16*>(tile + 2 * TILE128);
  __nv_bfloat16* wsKg = reinterpret_cast<__nv_bfloat16*>(tile + 3 * TILE128);
  __nv_bfloat16* wsA = reinterpret_cast<__nv_bfloat16*>(tile + 4 * TILE128);
  float* wsGamma = reinterpret_cast<float*>(tile + 4 * TILE128 + TILE64);
#pragma unroll
  for (int n = 0; n < 8; ++n) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int i = warp * 16 + gq + hh * 8;
      const int j0 = n * 8 + 2 * tq;
      float l2[2], a2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = j0 + e;
        const float dec = (i >= j) ? expf(sm.G[i] - sm.G[j]) : 0.f;
        l2[e] = (i > j) ? -sm.beta[i] * kk[n][hh * 2 + e] * dec : 0.f;
        a2[e] = (i >= j) ? qk[n][hh * 2 + e] * dec : 0.f;
      }
      sm.L[i][j0] = l2[0];
      sm.L[i][j0 + 1] = l2[1];
      *reinterpret_cast<uint32_t*>(wsA + i * DR_C + j0) = pack_bf16x2(a2[0], a2[1]);
    }
  }
  __syncthreads();

  // 4. T = (I - L)^-1.  (a) diagonal 16x16 blocks by forward substitution, warp w -> block w.
  {
    const int b0 = warp * 16;
    const int c = lane & 15;
    const bool act = lane < 16;
    for (int r = 0; r < 16; ++r) {
      float val = 0.f;
      if (act) {
        if (c < r) {
          val = sm.L[b0 + r][b0 + c];
          for (int kx = c + 1; kx < r; ++kx) val = fmaf(sm.L[b0 + r][b0 + kx], sm.T[b0 + kx][b0 + c], val);
        } else {
          val = (c == r) ? 1.f : 0.f;
        }
      }
      __syncwarp();
      if (act) sm.T[b0 + r][b0 + c] = val;
      __syncwarp();
    }
  }
  __syncthreads();
  // (b) block rows 1..3: T_ij = T_ii * sum_{k=j}^{i-1} L_ik T_kj.  M is staged in sm.L's upper
  // triangle (unused there): block (j, i) of L holds M_ij.
  for (int bi = 1; bi < 4; ++bi) {
    const int nblk = bi;  // blocks j = 0..bi-1
    for (int e = tid; e < nblk * 256; e += 128) {
      const int bj = e >> 8, rr = (e >> 4) & 15, cc = e & 15;
      float m = 0.f;
      for (int bk = bj; bk < bi; ++bk)
        for (int x = 0; x < 16; ++x) m = fmaf(sm.L[bi * 16 + rr][bk * 16 + x], sm.T[bk * 16 + x][bj * 16 + cc], m);
      sm.L[bj * 16 + rr][bi * 16 + cc] = m;  // upper-triangle scratch
    }
    __syncthreads();
    for (int e = tid; e < nblk * 256; e += 128) {
      const int bj = e >> 8, rr = (e >> 4) & 15, cc = e & 15;
      float t = 0.f;
      for (int x = 0; x <= rr; ++x) t = fmaf(sm.T[bi * 16 + rr][bi * 16 + x], sm.L[bj * 16 + x][bi * 16 + cc], t);
      sm.T[bi * 16 + rr][bj * 16 + cc] = t;
    }
    __syncthreads();
  }
  // upper triangle of T is zero
  for (int e = tid; e < DR_C * DR_C; e += 128) {
    const int r = e >> 6, c = e & 63;
    if ((c >> 4) > (r >> 4)) sm.T[r][c] = 0.f;
  }
  __syncthreads();
  // 5. scaled bf16 copies of T for U and W
  for (int e = tid; e < DR_C * DR_C; e += 128) {
    const int r = e >> 6, c = e & 63;
    const float t = sm.T[r][c];
    sm.tu[r][c] = __float2bfloat16_rn(t * sm.beta[c]);
    sm.tw[r][c] = __float2bfloat16_rn(t * sm.beta[c] * expf(sm.G[c]));
  }
  __syncthreads();
  // 6. U = TU V, W = TW K  (rows [16w, 16w+16), 128 columns, K = 64)
  {
    float u[16][4], w[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) u[n][j] = w[n][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DR_C; ks += 16) {
      uint32_t au[4], aw[4];
      load_a(&sm.tu[0][0], LD64, warp * 16, ks, au);
      load_a(&sm.tw[0][0], LD64, warp * 16, ks, aw);
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        uint32_t bv[4], bk[4];
        load_b_kn(&sm.v[0][0], LD128, n * 8, ks, bv);
        load_b_kn(&sm.k[0][0], LD128, n * 8, ks, bk);
        mma_bf16_16816(u[n], au, bv[0], bv[1]);
        mma_bf16_16816(u[n + 1], au, bv[2], bv[3]);
        mma_bf16_16816(w[n], aw, bk[0], bk[1]);
        mma_bf16_16816(w[n + 1], aw, bk[2], bk[3]);
      }
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = warp * 16 + gq + hh * 8;
        const int j = n * 8 + 2 * tq;
        *reinterpret_cast<uint32_t*>(wsU + i * DR_D + j) = pack_bf16x2(u[n][hh * 2], u[n][hh * 2 + 1]);
        *reinterpret_cast<uint32_t*>(wsW + i * DR_D + j) = pack_bf16x2(w[n][hh * 2], w[n][hh * 2 + 1]);
      }
    }
  }
  // 7. Qg = q e^G, Kg = k e^(G_last - G); gamma = e^G_last
  const float glast = sm.G[DR_C - 1];
  for (int e = tid; e < DR_C * 16; e += 128) {
    const int r = e >> 4, c = (e & 15) * 8;
    const float eq = expf(sm.G[r]);
    const float ek = expf(glast - sm.G[r]);
    float xq[8], xk[8];
    unpack8(*reinterpret_cast<const uint4*>(&sm.q[r][c]), xq);
    unpack8(*reinterpret_cast<const uint4*>(&sm.k[r][c]), xk);
#pragma unroll
    for (int j = 0; j < 8; ++j) { xq[j] *= eq; xk[j] *= ek; }
    *reinterpret_cast<uint4*>(wsQg + r * DR_D + c) = pack8(xq);
    *reinterpret_cast<uint4*>(wsKg + r * DR_D + c) = pack8(xk);
  }
  if (tid == 0) *wsGamma = expf(glast);
}

struct RecurSmem {
  __nv_bfloat16 w[2][DR_C][LD128];
  __nv_bfloat16 qg[2][DR_C][LD128];
  __nv_bfloat16 kg[2][DR_C][LD128];
  __nv_bfloat16 a[2][DR_C][LD64];
  __nv_bfloat16 u[2][DR_C][DR_BV + 8];
  __nv_bfloat16 s[2][DR_D][DR_BV + 8];
  __nv_bfloat16 vn[DR_C][DR_BV + 8];
  float gamma[2];
};

__device__ __forceinline__ void recur_prefetch(RecurSmem& sm, int buf, const uint8_t* tile, int vb, int tid) {
  const __nv_bfloat16* W = reinterpret_cast<const __nv_bfloat16*>(tile);
  const __nv_bfloat16* U = reinterpret_cast<const __nv_bfloat16*>(tile + TILE128);
  const __nv_bfloat16* Qg = reinterpret_cast<const __nv_bfloat16*>(tile + 2 * TILE128);
  const __nv_bfloat16* Kg = reinterpret_cast<const __nv_bfloat16*>(tile + 3 * TILE128);
  const __nv_bfloat16* A = reinterpret_cast<const __nv_bfloat16*>(tile + 4 * TILE128);
  for (int e = tid; e < DR_C * 16; e += 128) {
    const int r = e >> 4, c = (e & 15) * 8;
    cp_async16(&sm.w[buf][r][c], W + r * DR_D + c);
    cp_async16(&sm.qg[buf][r][c], Qg + r * DR_D + c);
    cp_async16(&sm.kg[buf][r][c], Kg + r * DR_D + c);
  }
  for (int e = tid; e < DR_C * 8; e += 128) {
    const int r = e >> 3, c = (e & 7) * 8;
    cp_async16(&sm.a[buf][r][c], A + r * DR_C + c);
  }
  for (int e = tid; e < DR_C * (DR_BV / 8); e += 128) {
    const int r = e / (DR_BV / 8), c = (e % (DR_BV / 8)) * 8;
    cp_async16(&sm.u[buf][r][c], U + r * DR_D + vb * DR_BV + c);
  }
  cp_async_commit();
}

__global__ void __launch_bounds__(128) delta_recur_kernel(
    const int32_t* __restrict__ cu, int nseg, const int32_t* __restrict__ table, int heads,
    const uint8_t* __restrict__ tiles, const float* __restrict__ init_state, bf16* __restrict__ out,
    float* __restrict__ final_state) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  RecurSmem& sm = *reinterpret_cast<RecurSmem*>(smem_raw);
  const int s = blockIdx.x, h = blockIdx.y, vb = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int c0 = table[s], nch = table[s + 1] - c0;
  const int seg_t0 = cu[s], seg_len = cu[s + 1] - cu[s];

  // state S[dk][dv-block]: warp w owns dk rows [32w, 32w+32) as 2 m-tiles x 4 n-tiles
  float S[2][4][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float val = 0.f;
        if (init_state) {
          const int r = warp * 32 + mt * 16 + gq + (j >> 1) * 8;
          const int c = nt * 8 + 2 * tq + (j & 1);
          val = init_state[(((int64_t)s * heads + h) * DR_D + r) * DR_D + vb * DR_BV + c];
        }
        S[mt][nt][j] = val;
      }
  // bf16 copy of S for the first chunk
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int r = warp * 32 + mt * 16 + gq + hh * 8;
        const int c = nt * 8 + 2 * tq;
        *reinterpret_cast<uint32_t*>(&sm.s[0][r][c]) = pack_bf16x2(S[mt][nt][hh * 2], S[mt][nt][hh * 2 + 1]);
      }
  if (nch > 0) recur_prefetch(sm, 0, tiles + ((size_t)c0 * heads + h) * CH_BYTES, vb, tid);
  for (int c = 0; c < nch; ++c) {
    const int buf = c & 1;
    const uint8_t* tile = tiles + ((size_t)(c0 + c) * heads + h) * CH_BYTES;
    if (tid == 0) sm.gamma[buf] = *reinterpret_cast<const float*>(tile + 4 * TILE128 + TILE64);
    cp_async_wait<0>();
    __syncthreads();
    if (c + 1 < nch) recur_prefetch(sm, buf ^ 1, tile + (size_t)heads * CH_BYTES, vb, tid);
    // A. v_new = U - W S   (rows [16w, 16w+16), 32 cols, K = 128)
    float acc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[nt][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DR_D; ks += 16) {
      uint32_t a[4];
      load_a(&sm.w[buf][0][0], LD128, warp * 16, ks, a);
#pragma unroll
      for (int nt = 0; nt < 4; nt += 2) {
        uint32_t b[4];
        load_b_kn(&sm.s[buf][0][0], DR_BV + 8, nt * 8, ks, b);
        mma_bf16_16816(acc[nt], a, b[0], b[1]);
        mma_bf16_16816(acc[nt + 1], a, b[2], b[3]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int r = warp * 16 + gq + hh * 8;
        const int cc = nt * 8 + 2 * tq;
        const float2 uu = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.u[buf][r][cc]));
        *reinterpret_cast<uint32_t*>(&sm.vn[r][cc]) = pack_bf16x2(uu.x - acc[nt][hh * 2], uu.y - acc[nt][hh * 2 + 1]);
      }
    __syncthreads();
    // B. o = Qg S + Aqk v_new
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[nt][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DR_D; ks += 16) {
      uint32_t a[4];
      load_a(&sm.qg[buf][0][0], LD128, warp * 16, ks, a);
#pragma unroll
      for (int nt = 0; nt < 4; nt += 2) {
        uint32_t b[4];
        load_b_kn(&sm.s[buf][0][0], DR_BV + 8, nt * 8, ks, b);
        mma_bf16_16816(acc[nt], a, b[0], b[1]);
        mma_bf16_16816(acc[nt + 1], a, b[2], b[3]);
      }
    }
#pragma unroll
    for (int ks = 0; ks < DR_C; ks += 16) {
      uint32_t a[4];
      load_a(&sm.a[buf][0][0], LD64, warp * 16, ks, a);
#pragma unroll
      for (int nt = 0; nt < 4; nt += 2) {
        uint32_t b[4];
        load_b_kn(&sm.vn[0][0], DR_BV + 8, nt * 8, ks, b);
        mma_bf16_16816(acc[nt], a, b[0], b[1]);
        mma_bf16_16816(acc[nt + 1], a, b[2], b[3]);
      }
    }
    const int tok0 = seg_t0 + c * DR_C;
    const int len = min(DR_C, seg_len - c * DR_C);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int r = warp * 16 + gq + hh * 8;
        if (r < len) {
          const int cc = vb * DR_BV + nt * 8 + 2 * tq;
          *reinterpret_cast<uint32_t*>(out + ((int64_t)(tok0 + r) * heads + h) * DR_D + cc) =
              pack_bf16x2(acc[nt][hh * 2], acc[nt][hh * 2 + 1]);
        }
      }
    // C. S = gamma S + Kg^T v_new   (dk rows [32w, 32w+32), K = 64 tokens)
    const float gm = sm.gamma[buf];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) S[mt][nt][j] *= gm;
#pragma unroll
    for (int ks = 0; ks < DR_C; ks += 16) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t a[4];
        load_a_t(&sm.kg[buf][0][0], LD128, warp * 32 + mt * 16, ks, a);
#pragma unroll
        for (int nt = 0; nt < 4; nt += 2) {
          uint32_t b[4];
          load_b_kn(&sm.vn[0][0], DR_BV + 8, nt * 8, ks, b);
          mma_bf16_16816(S[mt][nt], a, b[0], b[1]);
          mma_bf16_16816(S[mt][nt + 1], a, b[2], b[3]);
        }
      }
    }
    // bf16 copy of the new state for the next chunk
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int r = warp * 32 + mt * 16 + gq + hh * 8;
          const int cc = nt * 8 + 2 * tq;
          *reinterpret_cast<uint32_t*>(&sm.s[buf ^ 1][r][cc]) = pack_bf16x2(S[mt][nt][hh * 2], S[mt][nt][hh * 2 + 1]);
        }
    __syncthreads();  // vn and s[buf] are rewritten by the next chunk
  }
  if (final_state) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = warp * 32 + mt * 16 + gq + (j >> 1) * 8;
          const int cc = nt * 8 + 2 * tq + (j & 1);
          final_state[(((int64_t)s * heads + h) * DR_D + r) * DR_D + vb * DR_BV + cc] = S[mt][nt][j];
        }
  }
}

}  // namespace fdk

using namespace fdk;

extern "C" size_t fdk_chunk_gated_delta_rule_workspace_size(int64_t tokens, int64_t num_segments, int64_t heads,
                                                            int64_t dk, int64_t dv) {
  if (tokens < 0 || num_segments < 1 || heads < 1 || dk != DR_D || dv != DR_D) return 0;
  return ws_layout(tokens, num_segments, heads).total;
}

extern "C" int fdk_chunk_gated_delta_rule_fwd(const void* q, const void* k, int64_t ld_qk, const void* v, int64_t ld_v,
                                              const float* g, const void* beta, const int32_t* cu_seqlens,
                                              int64_t num_segments, int64_t tokens, int64_t heads, int64_t dk, int64_t dv,
                                              float scale, const float* initial_state, void* out, float* final_state,
                                              void* workspace, size_t workspace_bytes, void* stream) {
  if (int st = check_device()) return st;
  if (!q || !k || !v || !g || !beta || !cu_seqlens || !out || !workspace)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "chunk_gated_delta_rule: null pointer");
  if (dk != DR_D || dv != DR_D)
    return set_error(FDK_ERR_UNSUPPORTED, "chunk_gated_delta_rule: dk=%lld dv=%lld (only 128 supported)", (long long)dk, (long long)dv);
  if (num_segments < 1 || tokens < 0 || heads < 1 || heads > 65535 || num_segments > 0x7fffffff)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "chunk_gated_delta_rule: bad sizes");
  if (ld_qk < heads * dk || ld_v < heads * dv) return set_error(FDK_ERR_INVALID_ARGUMENT, "chunk_gated_delta_rule: row stride too small");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || ld_qk % 8 || ld_v % 8 ||
      (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(FDK_ERR_ALIGNMENT, "chunk_gated_delta_rule: 16-byte tensors and a 256-byte aligned workspace required");
  const WsLayout lay = ws_layout(tokens, num_segments, heads);
  if (workspace_bytes < lay.total)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "chunk_gated_delta_rule: workspace %zu bytes < required %zu", workspace_bytes, lay.total);
  if (lay.max_chunks > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "chunk_gated_delta_rule: too many chunks");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* table = reinterpret_cast<int32_t*>(ws + lay.off_table);
  uint8_t* tiles = ws + lay.off_tiles;
  const int nseg = (int)num_segments;
  chunk_table_kernel<<<1, 32, 0, s>>>(cu_seqlens, nseg, table);
  if (int st = check_launch("chunk_gated_delta_rule/table")) return st;
  if (tokens == 0) return FDK_OK;
  static bool attr_set[64] = {};
  const int prep_smem = (int)sizeof(PrepSmem);
  const int recur_smem = (int)sizeof(RecurSmem);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaFuncSetAttribute(delta_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem);
    cudaFuncSetAttribute(delta_recur_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, recur_smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  delta_prep_kernel<<<dim3((unsigned)lay.max_chunks, (unsigned)heads), 128, prep_smem, s>>>(
      static_cast<const bf16*>(q), static_cast<const bf16*>(k), ld_qk, static_cast<const bf16*>(v), ld_v, g,
      static_cast<const bf16*>(beta), cu_seqlens, nseg, table, (int)heads, scale, tiles);
  if (int st = check_launch("chunk_gated_delta_rule/prep")) return st;
  delta_recur_kernel<<<dim3((unsigned)nseg, (unsigned)heads, DR_D / DR_BV), 128, recur_smem, s>>>(
      cu_seqlens, nseg, table, (int)heads, tiles, initial_state, static_cast<bf16*>(out), final_state);
  return check_launch("chunk_gated_delta_rule/recurrence");
}
