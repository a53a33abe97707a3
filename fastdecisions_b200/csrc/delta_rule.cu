// Chunked gated delta rule (Gated DeltaNet core), chunk = 64 tokens, dk = dv = 128.
//
// Restates transformers' torch_chunk_gated_delta_rule (models/qwen3_5/modeling_qwen3_5.py:234-311)
// for packed varlen input.  Three launches:
//   1. chunk_table_kernel : per-segment chunk offsets (device side, graph-capturable).
//   2. delta_prep_kernel  : one 256-thread CTA per (chunk, head), fully parallel.  l2-normalises q
//      and k, takes the in-chunk cumsum G of the log decay, forms KK^T and QK^T on the tensor
//      cores, inverts the unit-lower-triangular (I - L) in fp32 (16x16 diagonal blocks by forward
//      substitution with each column held in registers, then block forward substitution), and
//      writes into the caller's workspace (bf16)
//        W  = T diag(beta e^G) K      Ut = (T diag(beta) V)^T       Aqk = (QK^T o decay), lower
//        Qg = q e^G                   Kg = k e^(G_last - G)         gamma = e^G_last (fp32)
//   3. delta_recur_kernel : one CTA per (segment, head, dv slice), sequential over the segment's
//      chunks.  Each warp owns 16 dv rows of the TRANSPOSED state S^T [dv x dk] as fp32 mma
//      accumulators and never exchanges data with other warps:
//        v_new^T = U^T - S^T W^T ;  o^T = S^T Qg^T + v_new^T Aqk^T ;  S^T = gamma S^T + v_new^T Kg
//      An accumulator tile of one product is the A operand of the next (bf16-packed in
//      registers), so the state never round-trips through shared memory; the chunk tiles stream
//      in with cp.async, double-buffered, into XOR-swizzled (bank-conflict-free) shared memory.
#include "common.cuh"
#include "mma_sm80.cuh"

namespace fdk {

constexpr int DR_C = 64;    // chunk length
constexpr int DR_D = 128;   // dk == dv

// Per (chunk, head) workspace tile: W, Qg, Kg [64][128], Ut [128][64], Aqk [64][64] (bf16), gamma.
constexpr size_t TILE128 = (size_t)DR_C * DR_D * 2;
constexpr size_t TILE64 = (size_t)DR_C * DR_C * 2;
constexpr size_t OFF_W = 0, OFF_QG = TILE128, OFF_KG = 2 * TILE128, OFF_UT = 3 * TILE128, OFF_A = 4 * TILE128,
                 OFF_GAMMA = 4 * TILE128 + TILE64;
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

// XOR-swizzled row-major bf16 tiles: 16-byte chunk c of row r lives at chunk c ^ (r & 7).
template <int COLS>
__device__ __forceinline__ int swz(int r, int col) {
  return r * COLS + ((((col >> 3) ^ (r & 7))) << 3) + (col & 7);
}

// ldmatrix fragment loads from swizzled tiles (same conventions as mma_sm80.cuh).
template <int COLS>
__device__ __forceinline__ void lda_sw(const __nv_bfloat16* t, int r0, int c0, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31;
  ldsm_x4(smem_u32(t + swz<COLS>(r0 + (lane & 15), c0 + ((lane >> 4) << 3))), a[0], a[1], a[2], a[3]);
}
template <int COLS>  // B^T stored [n][k]
__device__ __forceinline__ void ldb_nk_sw(const __nv_bfloat16* t, int n0, int k0, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31, m = lane >> 3;
  ldsm_x4(smem_u32(t + swz<COLS>(n0 + (lane & 7) + ((m >> 1) << 3), k0 + ((m & 1) << 3))), b[0], b[1], b[2], b[3]);
}
template <int COLS>  // B stored [k][n]
__device__ __forceinline__ void ldb_kn_sw(const __nv_bfloat16* t, int n0, int k0, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31, m = lane >> 3;
  ldsm_x4_t(smem_u32(t + swz<COLS>(k0 + (lane & 7) + ((m & 1) << 3), n0 + ((m >> 1) << 3))), b[0], b[1], b[2], b[3]);
}

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(valid ? 16 : 0));
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

// ------------------------------------------------------------------------------------------ prep
constexpr int PREP_THREADS = 256;
constexpr int LDF = DR_C + 4;     // fp32 tile stride: conflict-free column solves and row reads
constexpr int UT_LD = DR_C + 8;   // padded row of the transposed U staging tile

struct PrepSmem {
  __nv_bfloat16 q[DR_C * DR_D];   // swizzled; TU / TW (2 x [64][64]) after QK^T; W staging last
  __nv_bfloat16 k[DR_C * DR_D];   // swizzled; with v: U^T staging [128][UT_LD] after U/W
  __nv_bfloat16 v[DR_C * DR_D];   // swizzled
  float L[DR_C][LDF];             // strictly lower L, then block-solve scratch
  float T[DR_C][LDF];
  float G[DR_C];
  float beta[DR_C];
  int info[2];
};

__global__ void __launch_bounds__(PREP_THREADS, 2) delta_prep_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, int64_t ldqk, const bf16* __restrict__ v, int64_t ldv,
    const float* __restrict__ g, const bf16* __restrict__ beta, const int32_t* __restrict__ cu, int nseg,
    const int32_t* __restrict__ table, int heads, float scale, uint8_t* __restrict__ tiles) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(smem_raw);
  const int ci = blockIdx.x;
  const int h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  if (ci >= table[nseg]) return;
  if (tid == 0) {
    int lo = 0, hi = nseg - 1;  // largest segment s with table[s] <= ci (empty segments skipped)
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (table[mid] <= ci) lo = mid; else hi = mid - 1;
    }
    const int t0 = cu[lo] + (ci - table[lo]) * DR_C;
    sm.info[0] = t0;
    sm.info[1] = min(DR_C, cu[lo + 1] - t0);
  }
  __syncthreads();
  const int t0 = sm.info[0], len = sm.info[1];
  uint8_t* tile = tiles + ((size_t)ci * heads + h) * CH_BYTES;

  // 1. q, k, v rows -> swizzled smem (zero-filled past len); decay cumsum and beta
  for (int e = tid; e < DR_C * 16; e += PREP_THREADS) {
    const int r = e >> 4, c = (e & 15) << 3;
    const bool ok = r < len;
    const int64_t t = t0 + (ok ? r : 0);
    cp_async16_zfill(&sm.q[swz<DR_D>(r, c)], q + t * ldqk + (int64_t)h * DR_D + c, ok);
    cp_async16_zfill(&sm.k[swz<DR_D>(r, c)], k + t * ldqk + (int64_t)h * DR_D + c, ok);
    cp_async16_zfill(&sm.v[swz<DR_D>(r, c)], v + t * ldv + (int64_t)h * DR_D + c, ok);
  }
  cp_async_commit();
  if (warp == 0) {
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
    const int r0 = 2 * lane, r1 = 2 * lane + 1;
    if (r0 < len) { a0 = g[(int64_t)(t0 + r0) * heads + h]; b0 = __bfloat162float(beta[(int64_t)(t0 + r0) * heads + h]); }
    if (r1 < len) { a1 = g[(int64_t)(t0 + r1) * heads + h]; b1 = __bfloat162float(beta[(int64_t)(t0 + r1) * heads + h]); }
    const float pair = a0 + a1;
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
  cp_async_wait<0>();
  __syncthreads();

  // 2. l2 norm of q (times scale) and k rows in fp32; Qg = q e^G and Kg = k e^(G_last - G) out
  {
    const float glast = sm.G[DR_C - 1];
    __nv_bfloat16* wsQg = reinterpret_cast<__nv_bfloat16*>(tile + OFF_QG);
    __nv_bfloat16* wsKg = reinterpret_cast<__nv_bfloat16*>(tile + OFF_KG);
    for (int rr = warp; rr < 2 * DR_C; rr += PREP_THREADS / 32) {
      const bool isq = rr < DR_C;
      const int r = isq ? rr : rr - DR_C;
      __nv_bfloat16* row = isq ? sm.q : sm.k;
      const int col = lane * 4;
      uint2 u = *reinterpret_cast<const uint2*>(&row[swz<DR_D>(r, col)]);
      float2 x01 = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.x));
      float2 x23 = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.y));
      float ss = x01.x * x01.x + x01.y * x01.y + x23.x * x23.x + x23.y * x23.y;
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss + 1e-6f) * (isq ? scale : 1.0f);
      x01.x *= inv; x01.y *= inv; x23.x *= inv; x23.y *= inv;
      uint2 o;
      o.x = pack_bf16x2(x01.x, x01.y);
      o.y = pack_bf16x2(x23.x, x23.y);
      *reinterpret_cast<uint2*>(&row[swz<DR_D>(r, col)]) = o;
      // decayed copies use the bf16-rounded normalised values (what the products see)
      const float2 n01 = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&o.x));
      const float2 n23 = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&o.y));
      const float f = isq ? expf(sm.G[r]) : expf(glast - sm.G[r]);
      uint2 d;
      d.x = pack_bf16x2(n01.x * f, n01.y * f);
      d.y = pack_bf16x2(n23.x * f, n23.y * f);
      *reinterpret_cast<uint2*>((isq ? wsQg : wsKg) + r * DR_D + col) = d;
    }
  }
  __syncthreads();

  // 3. KK^T and QK^T: warp w -> rows [16 (w%4), +16), cols [32 (w/4), +32); decay and masks
  {
    const int r0 = (warp & 3) * 16, n0 = (warp >> 2) * 32;
    float kk[4][4], qk[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) kk[n][j] = qk[n][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DR_D; ks += 16) {
      uint32_t ak[4], aq[4];
      lda_sw<DR_D>(sm.k, r0, ks, ak);
      lda_sw<DR_D>(sm.q, r0, ks, aq);
#pragma unroll
      for (int n = 0; n < 4; n += 2) {
        uint32_t b[4];
        ldb_nk_sw<DR_D>(sm.k, n0 + n * 8, ks, b);
        mma_bf16_16816(kk[n], ak, b[0], b[1]);
        mma_bf16_16816(kk[n + 1], ak, b[2], b[3]);
        mma_bf16_16816(qk[n], aq, b[0], b[1]);
        mma_bf16_16816(qk[n + 1], aq, b[2], b[3]);
      }
    }
    __nv_bfloat16* wsA = reinterpret_cast<__nv_bfloat16*>(tile + OFF_A);
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = r0 + gq + hh * 8;
        const int j0 = n0 + n * 8 + 2 * tq;
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

  // 4a. diagonal 16x16 blocks of T = (I - L)^-1: thread (b, c) solves column c of block b,
  //     keeping the column in registers (no cross-thread dependency).
  if (tid < 64) {
    const int b0 = (tid >> 4) * 16, c = tid & 15;
    float col[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float acc = 0.f;
      if (r == c) acc = 1.f;
      if (r > c) {
        acc = sm.L[b0 + r][b0 + c];
#pragma unroll
        for (int kx = 0; kx < r; ++kx)
          if (kx > c) acc = fmaf(sm.L[b0 + r][b0 + kx], col[kx], acc);
      }
      col[r] = acc;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) sm.T[b0 + r][b0 + c] = col[r];
  }
  __syncthreads();
  // 4b. block rows 1..3: T_ij = T_ii * sum_{k=j}^{i-1} L_ik T_kj (M staged in L's upper triangle)
  for (int bi = 1; bi < 4; ++bi) {
    for (int e = tid; e < bi * 256; e += PREP_THREADS) {
      const int bj = e >> 8, rr = (e >> 4) & 15, cc = e & 15;
      float m = 0.f;
      for (int x = bj * 16; x < bi * 16; ++x) m = fmaf(sm.L[bi * 16 + rr][x], sm.T[x][bj * 16 + cc], m);
      sm.L[bj * 16 + rr][bi * 16 + cc] = m;
    }
    __syncthreads();
    for (int e = tid; e < bi * 256; e += PREP_THREADS) {
      const int bj = e >> 8, rr = (e >> 4) & 15, cc = e & 15;
      float t = 0.f;
      for (int x = 0; x <= rr; ++x) t = fmaf(sm.T[bi * 16 + rr][bi * 16 + x], sm.L[bj * 16 + x][bi * 16 + cc], t);
      sm.T[bi * 16 + rr][bj * 16 + cc] = t;
    }
    __syncthreads();
  }

  // 5. TU = bf16(T diag(beta)), TW = bf16(T diag(beta e^G)) into q's space (upper triangle = 0)
  __nv_bfloat16* TU = sm.q;
  __nv_bfloat16* TW = sm.q + DR_C * DR_C;
  for (int e = tid; e < DR_C * 8; e += PREP_THREADS) {
    const int r = e & 63, c0 = (e >> 6) << 3;
    float t8[8], tu[8], tw[8];
    *reinterpret_cast<float4*>(&t8[0]) = *reinterpret_cast<const float4*>(&sm.T[r][c0]);
    *reinterpret_cast<float4*>(&t8[4]) = *reinterpret_cast<const float4*>(&sm.T[r][c0 + 4]);
    const bool live = (c0 >> 4) <= (r >> 4);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = c0 + j;
      const float t = live ? t8[j] : 0.f;
      tu[j] = t * sm.beta[c];
      tw[j] = t * sm.beta[c] * expf(sm.G[c]);
    }
    *reinterpret_cast<uint4*>(&TU[swz<DR_C>(r, c0)]) = pack8(tu);
    *reinterpret_cast<uint4*>(&TW[swz<DR_C>(r, c0)]) = pack8(tw);
  }
  __syncthreads();

  // 6. U = TU V and W = TW K: warp w -> rows [16 (w%4), +16), cols [64 (w/4), +64)
  {
    const int r0 = (warp & 3) * 16, n0 = (warp >> 2) * 64;
    float u[8][4], w[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) u[n][j] = w[n][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DR_C; ks += 16) {
      uint32_t au[4], aw[4];
      lda_sw<DR_C>(TU, r0, ks, au);
      lda_sw<DR_C>(TW, r0, ks, aw);
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t bv[4], bk[4];
        ldb_kn_sw<DR_D>(sm.v, n0 + n * 8, ks, bv);
        ldb_kn_sw<DR_D>(sm.k, n0 + n * 8, ks, bk);
        mma_bf16_16816(u[n], au, bv[0], bv[1]);
        mma_bf16_16816(u[n + 1], au, bv[2], bv[3]);
        mma_bf16_16816(w[n], aw, bk[0], bk[1]);
        mma_bf16_16816(w[n + 1], aw, bk[2], bk[3]);
      }
    }
    __syncthreads();  // every warp is done with TU/TW, k and v: stage W and U^T there
    __nv_bfloat16* Wst = sm.q;   // [64][128] plain row-major
    __nv_bfloat16* Ust = sm.k;   // [128][UT_LD] transposed, padded (spans k and v)
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = r0 + gq + hh * 8;
        const int j = n0 + n * 8 + 2 * tq;
        *reinterpret_cast<uint32_t*>(&Wst[i * DR_D + j]) = pack_bf16x2(w[n][hh * 2], w[n][hh * 2 + 1]);
        Ust[j * UT_LD + i] = __float2bfloat16_rn(u[n][hh * 2]);
        Ust[(j + 1) * UT_LD + i] = __float2bfloat16_rn(u[n][hh * 2 + 1]);
      }
  }
  __syncthreads();
  {
    const uint4* sW = reinterpret_cast<const uint4*>(sm.q);
    uint4* gW = reinterpret_cast<uint4*>(tile + OFF_W);
    __nv_bfloat16* gU = reinterpret_cast<__nv_bfloat16*>(tile + OFF_UT);
    for (int e = tid; e < (int)(TILE128 / 16); e += PREP_THREADS) {
      gW[e] = sW[e];
      const int j = e >> 3, c = (e & 7) << 3;
      *reinterpret_cast<uint4*>(gU + j * DR_C + c) = *reinterpret_cast<const uint4*>(sm.k + j * UT_LD + c);
    }
  }
  if (tid == 0) *reinterpret_cast<float*>(tile + OFF_GAMMA) = expf(sm.G[DR_C - 1]);
}

// ------------------------------------------------------------------------------------- recurrence
struct RecurStage {
  __nv_bfloat16 w[DR_C * DR_D];    // swizzled [tok][dk]
  __nv_bfloat16 qg[DR_C * DR_D];   // swizzled [tok][dk]
  __nv_bfloat16 kg[DR_C * DR_D];   // swizzled [tok][dk]
  __nv_bfloat16 a[DR_C * DR_C];    // swizzled [tok][tok']
  float gamma[4];                  // gamma = e^G_last (+ padding of the 16-byte copy)
};

template <int WARPS>
struct RecurSmem {
  RecurStage st[2];
  __nv_bfloat16 o[WARPS][DR_C][16];  // per-warp output staging [tok][16 dv]
};

__device__ __forceinline__ void recur_prefetch(RecurStage& s, const uint8_t* tile, int tid, int nthreads) {
  const __nv_bfloat16* W = reinterpret_cast<const __nv_bfloat16*>(tile + OFF_W);
  const __nv_bfloat16* Qg = reinterpret_cast<const __nv_bfloat16*>(tile + OFF_QG);
  const __nv_bfloat16* Kg = reinterpret_cast<const __nv_bfloat16*>(tile + OFF_KG);
  const __nv_bfloat16* A = reinterpret_cast<const __nv_bfloat16*>(tile + OFF_A);
  for (int e = tid; e < DR_C * 16; e += nthreads) {
    const int r = e >> 4, c = (e & 15) << 3;
    cp_async16(&s.w[swz<DR_D>(r, c)], W + r * DR_D + c);
    cp_async16(&s.qg[swz<DR_D>(r, c)], Qg + r * DR_D + c);
    cp_async16(&s.kg[swz<DR_D>(r, c)], Kg + r * DR_D + c);
  }
  for (int e = tid; e < DR_C * 8; e += nthreads) {
    const int r = e >> 3, c = (e & 7) << 3;
    cp_async16(&s.a[swz<DR_C>(r, c)], A + r * DR_C + c);
  }
  if (tid == 0) cp_async16(s.gamma, tile + OFF_GAMMA);
  cp_async_commit();
}

// U^T values of this thread for one chunk: rows dv (g, g+8), token pairs (8 nt + 2t, +1)
__device__ __forceinline__ void load_ut(const uint8_t* tile, int dv0, int gq, int tq, uint32_t (&u)[8][2]) {
  const __nv_bfloat16* Ut = reinterpret_cast<const __nv_bfloat16*>(tile + OFF_UT);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    u[nt][0] = __ldg(reinterpret_cast<const unsigned int*>(Ut + (dv0 + gq) * DR_C + nt * 8 + 2 * tq));
    u[nt][1] = __ldg(reinterpret_cast<const unsigned int*>(Ut + (dv0 + gq + 8) * DR_C + nt * 8 + 2 * tq));
  }
}

template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32) delta_recur_kernel(
    const int32_t* __restrict__ cu, int nseg, const int32_t* __restrict__ table, int heads,
    const uint8_t* __restrict__ tiles, const float* __restrict__ init_state, bf16* __restrict__ out,
    float* __restrict__ final_state) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  RecurSmem<WARPS>& sm = *reinterpret_cast<RecurSmem<WARPS>*>(smem_raw);
  constexpr int NT = WARPS * 32;
  const int s = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int dv0 = (blockIdx.z * WARPS + warp) * 16;  // this warp's 16 dv rows
  const int c0 = table[s], nch = table[s + 1] - c0;
  const int seg_t0 = cu[s], seg_len = cu[s + 1] - cu[s];
  const size_t hstride = (size_t)heads * CH_BYTES;

  // S^T [16 dv x 128 dk] as 16 accumulator tiles (rows dv0 + g (+8), cols 8 nt + 2t (+1))
  float st[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float val = 0.f;
      if (init_state) {
        const int dv = dv0 + gq + (j >> 1) * 8, dk = nt * 8 + 2 * tq + (j & 1);
        val = init_state[(((int64_t)s * heads + h) * DR_D + dk) * DR_D + dv];
      }
      st[nt][j] = val;
    }
  uint32_t ut[8][2];
  if (nch > 0) {
    const uint8_t* tile0 = tiles + ((size_t)c0 * heads + h) * CH_BYTES;
    recur_prefetch(sm.st[0], tile0, tid, NT);
    load_ut(tile0, dv0, gq, tq, ut);
  }
  for (int c = 0; c < nch; ++c) {
    const int buf = c & 1;
    const uint8_t* tile = tiles + ((size_t)(c0 + c) * heads + h) * CH_BYTES;
    cp_async_wait<0>();
    __syncthreads();
    uint32_t ut_next[8][2];
    if (c + 1 < nch) {
      recur_prefetch(sm.st[buf ^ 1], tile + hstride, tid, NT);
      load_ut(tile + hstride, dv0, gq, tq, ut_next);
    }
    const RecurStage& S = sm.st[buf];
    // S^T as bf16 A fragments (8 k-steps over dk)
    uint32_t sa[8][4];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      sa[kk][0] = pack_bf16x2(st[2 * kk][0], st[2 * kk][1]);
      sa[kk][1] = pack_bf16x2(st[2 * kk][2], st[2 * kk][3]);
      sa[kk][2] = pack_bf16x2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      sa[kk][3] = pack_bf16x2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
    }
    // 1. v_new^T = U^T - S^T W^T      [16 dv x 64 tok]
    float vn[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) vn[nt][j] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t b[4];
        ldb_nk_sw<DR_D>(S.w, nt * 8, kk * 16, b);
        mma_bf16_16816(vn[nt], sa[kk], b[0], b[1]);
        mma_bf16_16816(vn[nt + 1], sa[kk], b[2], b[3]);
      }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float2 u0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ut[nt][0]));
      const float2 u1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ut[nt][1]));
      vn[nt][0] = u0.x - vn[nt][0];
      vn[nt][1] = u0.y - vn[nt][1];
      vn[nt][2] = u1.x - vn[nt][2];
      vn[nt][3] = u1.y - vn[nt][3];
    }
    uint32_t va[4][4];  // v_new^T as A fragments (4 k-steps over tokens)
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) {
      va[kt][0] = pack_bf16x2(vn[2 * kt][0], vn[2 * kt][1]);
      va[kt][1] = pack_bf16x2(vn[2 * kt][2], vn[2 * kt][3]);
      va[kt][2] = pack_bf16x2(vn[2 * kt + 1][0], vn[2 * kt + 1][1]);
      va[kt][3] = pack_bf16x2(vn[2 * kt + 1][2], vn[2 * kt + 1][3]);
    }
    // 2. o^T = S^T Qg^T + v_new^T Aqk^T   [16 dv x 64 tok]  (old state)
    float ot[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) ot[nt][j] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t b[4];
        ldb_nk_sw<DR_D>(S.qg, nt * 8, kk * 16, b);
        mma_bf16_16816(ot[nt], sa[kk], b[0], b[1]);
        mma_bf16_16816(ot[nt + 1], sa[kk], b[2], b[3]);
      }
#pragma unroll
    for (int kt = 0; kt < 4; ++kt)
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t b[4];
        ldb_nk_sw<DR_C>(S.a, nt * 8, kt * 16, b);
        mma_bf16_16816(ot[nt], va[kt], b[0], b[1]);
        mma_bf16_16816(ot[nt + 1], va[kt], b[2], b[3]);
      }
    // 3. S^T = gamma S^T + v_new^T Kg     [16 dv x 128 dk]
    const float gm = S.gamma[0];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) st[nt][j] *= gm;
#pragma unroll
    for (int kt = 0; kt < 4; ++kt)
#pragma unroll
      for (int nt = 0; nt < 16; nt += 2) {
        uint32_t b[4];
        ldb_kn_sw<DR_D>(S.kg, nt * 8, kt * 16, b);
        mma_bf16_16816(st[nt], va[kt], b[0], b[1]);
        mma_bf16_16816(st[nt + 1], va[kt], b[2], b[3]);
      }
    // output: stage o^T as [tok][16 dv] and write 32-byte row pieces
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int tk = nt * 8 + 2 * tq;
      sm.o[warp][tk][gq] = __float2bfloat16_rn(ot[nt][0]);
      sm.o[warp][tk + 1][gq] = __float2bfloat16_rn(ot[nt][1]);
      sm.o[warp][tk][gq + 8] = __float2bfloat16_rn(ot[nt][2]);
      sm.o[warp][tk + 1][gq + 8] = __float2bfloat16_rn(ot[nt][3]);
    }
    __syncwarp();
    const int tok0 = seg_t0 + c * DR_C;
    const int len = min(DR_C, seg_len - c * DR_C);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lane + i * 32;  // 128 pieces of 16 B: row e/2, half e%2
      const int r = e >> 1, half = e & 1;
      if (r < len)
        *reinterpret_cast<uint4*>(out + ((int64_t)(tok0 + r) * heads + h) * DR_D + dv0 + half * 8) =
            *reinterpret_cast<const uint4*>(&sm.o[warp][r][half * 8]);
    }
    if (c + 1 < nch) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) { ut[nt][0] = ut_next[nt][0]; ut[nt][1] = ut_next[nt][1]; }
    }
    __syncthreads();  // stage buf is refilled by the prefetch two chunks ahead; o staging reused
  }
  if (final_state) {
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int dv = dv0 + gq + (j >> 1) * 8, dk = nt * 8 + 2 * tq + (j & 1);
        final_state[(((int64_t)s * heads + h) * DR_D + dk) * DR_D + dv] = st[nt][j];
      }
  }
}

template <int WARPS>
static int launch_recur(int nseg, int heads, cudaStream_t s, const int32_t* cu, const int32_t* table,
                        const uint8_t* tiles, const float* init, bf16* out, float* fin) {
  const int smem = (int)sizeof(RecurSmem<WARPS>);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaFuncSetAttribute(delta_recur_kernel<WARPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  delta_recur_kernel<WARPS><<<dim3((unsigned)nseg, (unsigned)heads, DR_D / (16 * WARPS)), WARPS * 32, smem, s>>>(
      cu, nseg, table, heads, tiles, init, out, fin);
  return check_launch("chunk_gated_delta_rule/recurrence");
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
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaFuncSetAttribute(delta_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  delta_prep_kernel<<<dim3((unsigned)lay.max_chunks, (unsigned)heads), PREP_THREADS, prep_smem, s>>>(
      static_cast<const bf16*>(q), static_cast<const bf16*>(k), ld_qk, static_cast<const bf16*>(v), ld_v, g,
      static_cast<const bf16*>(beta), cu_seqlens, nseg, table, (int)heads, scale, tiles);
  if (int st = check_launch("chunk_gated_delta_rule/prep")) return st;
  // Few (segment, head) pairs: one warp per 16 dv rows spreads the sequential chains over more
  // SMs; many pairs: 4 warps share each chunk tile read.
  const int64_t pairs = (int64_t)nseg * heads;
  auto o = static_cast<bf16*>(out);
  if (pairs * 8 <= 2 * (int64_t)sm_count())
    return launch_recur<1>(nseg, (int)heads, s, cu_seqlens, table, tiles, initial_state, o, final_state);
  if (pairs * 4 <= 2 * (int64_t)sm_count())
    return launch_recur<2>(nseg, (int)heads, s, cu_seqlens, table, tiles, initial_state, o, final_state);
  return launch_recur<4>(nseg, (int)heads, s, cu_seqlens, table, tiles, initial_state, o, final_state);
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant: the scratch is a file-scope device array instead of a caller-owned
// workspace.  For callers that reach this library only through the C ABI and own no device
// allocator (a cgo / JNI / ctypes host without a CUDA framework), or that must not call
// cudaMalloc / cudaFree on their request path (those calls synchronise the device).
// ---------------------------------------------------------------------------------------------
#include <mutex>

namespace fdk {

// 32 MiB: enough for one 1536-token request with 16 heads (config 4).  Every GPU that loads this
// library holds the array until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
static __device__ __align__(256) uint8_t g_delta_noalloc_scratch[kNoAllocScratchBytes];

// Host code cannot pass the array's symbol to a kernel (it names a host-side stand-in), so the
// device address is looked up once per device, with that device current, and cached.
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64];

static int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return set_error(FDK_ERR_DEVICE, "chunk_gated_delta_rule_fwd_noalloc: no usable current device");
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_delta_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return set_error(FDK_ERR_DEVICE, "chunk_gated_delta_rule_fwd_noalloc: cudaGetSymbolAddress failed on device %d: %s",
                       dev, cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return FDK_OK;
}

}  // namespace fdk

extern "C" int fdk_chunk_gated_delta_rule_fwd_noalloc(const void* q, const void* k, int64_t ld_qk, const void* v,
                                                      int64_t ld_v, const float* g, const void* beta,
                                                      const int32_t* cu_seqlens, int64_t num_segments, int64_t tokens,
                                                      int64_t heads, int64_t dk, int64_t dv, float scale,
                                                      const float* initial_state, void* out, float* final_state,
                                                      void* stream) {
  using namespace fdk;
  if (int st = check_device()) return st;
  const size_t need = fdk_chunk_gated_delta_rule_workspace_size(tokens, num_segments, heads, dk, dv);
  if (need == 0)
    return set_error(FDK_ERR_UNSUPPORTED, "chunk_gated_delta_rule_fwd_noalloc: unsupported sizes (dk = dv = 128, "
                     "num_segments >= 1, heads >= 1, tokens >= 0)");
  if (need > kNoAllocScratchBytes)
    return set_error(FDK_ERR_UNSUPPORTED,
                     "chunk_gated_delta_rule_fwd_noalloc: this call needs %zu bytes of scratch but the built-in scratch "
                     "holds %zu (32 MiB); pass a workspace to fdk_chunk_gated_delta_rule_fwd instead",
                     need, kNoAllocScratchBytes);
  void* ws = nullptr;
  if (int st = noalloc_scratch(&ws)) return st;
  return fdk_chunk_gated_delta_rule_fwd(q, k, ld_qk, v, ld_v, g, beta, cu_seqlens, num_segments, tokens, heads, dk, dv,
                                        scale, initial_state, out, final_state, ws, kNoAllocScratchBytes, stream);
}
