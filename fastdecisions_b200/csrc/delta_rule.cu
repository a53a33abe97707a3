// Chunked gated delta rule (Gated DeltaNet core), chunk = 64 tokens, dk = dv = 128.
//
// Restates transformers' torch_chunk_gated_delta_rule (models/qwen3_5/modeling_qwen3_5.py:234-311)
// for packed varlen input.  Three launches (four with final states):
//   1. chunk_table_kernel : per-segment chunk offsets and per-chunk (first token, length, segment
//      start), device side and graph-capturable.
//   2. delta_prep_kernel  : one 256-thread CTA per (chunk, head), fully parallel, three CTAs per
//      SM.  TMA brings the raw q / k rows (or, fused, the raw projection columns, which the CTA
//      convolves itself, computing the gates from the projection too), the CTA l2-normalises
//      them, takes the in-chunk cumsum G of the log decay, forms [K;Q] K^T as one M=128 tcgen05
//      MMA, inverts the unit-lower-triangular (I - L) in fp32 (diagonal 16x16 blocks by row
//      substitution in registers, then off-diagonal blocks by 16x16 block products on mma.sync
//      tf32 with the 3xTF32 split), and forms U^T and W^T as two more tcgen05 MMAs (V and K as
//      MN-major A operands).  It writes into the caller's workspace (bf16)
//        W^T = (T diag(beta e^G) K)^T   U^T = (T diag(beta) V)^T     Aqk = (QK^T o decay), lower
//        Qg  = q e^G                    Kg  = k e^(G_last - G)       gamma = e^G_last (fp32)
//   3. delta_recur_tc_kernel : persistent; each CTA takes (segment, head) chains from a work
//      counter and runs them chunk by chunk with the state S^T [dv x dk] resident in TMEM:
//        v_new^T = U^T - S^T W^T ;  o^T = S^T Qg^T + v_new^T Aqk^T ;  S^T = gamma S^T + v_new^T Kg
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "common.cuh"
#include "sm100.cuh"

// Phase stamps of the prep (a profiling build only: `python -m fastdecisions_b200.build
// --phase-stamps` compiles this file with FDK_PHASE_STAMPS into a separate libfdk_phases.so).
// Thread 0 of every prep tile adds the SM cycles of each phase to g_phase[k]; g_phase[15] counts
// tiles; fdk_phase_stamps_read copies and clears them.
#ifdef FDK_PHASE_STAMPS
__device__ unsigned long long g_phase[16];
#define PHASE_START()                                   \
  unsigned long long t_phase = clock64();               \
  if (threadIdx.x == 0) atomicAdd(&g_phase[15], 1ull)
#define PHASE(k)                                                   \
  do {                                                             \
    if (threadIdx.x == 0) {                                        \
      const unsigned long long t_ = clock64();                     \
      atomicAdd(&g_phase[k], t_ - t_phase);                        \
      t_phase = t_;                                                \
    }                                                              \
  } while (0)
extern "C" int fdk_phase_stamps_read(unsigned long long* out) {
  if (cudaMemcpyFromSymbol(out, g_phase, sizeof(g_phase)) != cudaSuccess) return 1;
  unsigned long long z[16] = {};
  return cudaMemcpyToSymbol(g_phase, z, sizeof(z)) == cudaSuccess ? 0 : 1;
}
#else
#define PHASE_START() do {} while (0)
#define PHASE(k) do {} while (0)
#endif

namespace fdk {

constexpr int DR_C = 64;    // chunk length
constexpr int DR_D = 128;   // dk == dv

// Per (chunk, head) workspace tile: W^T [128][64], Qg, Kg [64][128], U^T [128][64], Aqk [64][64]
// (bf16), gamma (fp32).
constexpr size_t TILE128 = (size_t)DR_C * DR_D * 2;
constexpr size_t TILE64 = (size_t)DR_C * DR_C * 2;
constexpr size_t OFF_W = 0, OFF_QG = TILE128, OFF_KG = 2 * TILE128, OFF_UT = 3 * TILE128, OFF_A = 4 * TILE128,
                 OFF_GAMMA = 4 * TILE128 + TILE64;
constexpr size_t CH_BYTES = 4 * TILE128 + TILE64 + 16;

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct WsLayout {
  size_t off_table, off_info, off_tiles, off_ready, total;
  int64_t max_chunks;
};

// chunk table [nseg + 1] + recurrence work counter + prep tile counter, chunk info (first token,
// length, segment start) [max_chunks], tiles [max_chunks][heads], tile-ready flags [max_chunks][heads]
__host__ __device__ inline WsLayout ws_layout(int64_t tokens, int64_t nseg, int64_t heads) {
  WsLayout l;
  l.max_chunks = (tokens + DR_C - 1) / DR_C + nseg;
  l.off_table = 0;
  l.off_info = align256((size_t)(nseg + 3) * 4);
  l.off_tiles = l.off_info + align256((size_t)l.max_chunks * 16);
  l.off_ready = l.off_tiles + align256((size_t)l.max_chunks * heads * CH_BYTES);
  l.total = l.off_ready + align256((size_t)l.max_chunks * heads * 4);
  return l;
}

__device__ int g_delta_error = 0;  // bit 0: a bounded wait ran out; bit 1: cu_seqlens rejected on the device

// One CTA of 256 threads: exclusive scan of ceil(len / 64) over segments (table[s] = first chunk
// of segment s, table[nseg] = chunk count), each chunk's (first token, length, segment start), the zeroed
// work counters of the recurrence (table[nseg + 1]) and of the pipelined prep (table[nseg + 2]), and
// the zeroed tile-ready flags (`ready`, n_ready of them).
// cu_seqlens lives on the device, so the host cannot check it: this kernel does.  Unless
// cu[0] == 0, cu is non-decreasing and cu[nseg] == tokens (which bounds the chunk count by
// max_chunks, the size the workspace was laid out for), it writes an all-zero table -- every
// segment empty, so the prep and the recurrence touch no tile and no output row -- and sets bit 1
// of the delta-rule error word.
__global__ void __launch_bounds__(256) chunk_table_kernel(const int32_t* __restrict__ cu, int nseg, int64_t tokens,
                                                          int64_t max_chunks, int32_t* __restrict__ table,
                                                          int4* __restrict__ info, int32_t* __restrict__ ready,
                                                          int64_t n_ready) {
  __shared__ int warp_sums[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t i = tid; i < n_ready; i += 256) ready[i] = 0;
  bool bad = false;
  for (int s = tid; s < nseg; s += 256) bad |= cu[s + 1] < cu[s];
  if (tid == 0) bad |= cu[0] != 0 || (int64_t)cu[nseg] != tokens;
  if (__syncthreads_or(bad)) {
    for (int s = tid; s <= nseg + 2; s += 256) table[s] = 0;
    if (tid == 0) atomicOr(&g_delta_error, 2);
    return;
  }
  (void)max_chunks;  // sum of ceil(len / 64) <= tokens / 64 + nseg == max_chunks once cu is valid
  int carry = 0;
  for (int base = 0; base < nseg; base += 256) {
    const int s = base + tid;
    int n = 0, t0 = 0, len = 0;
    if (s < nseg) {
      t0 = cu[s];
      len = cu[s + 1] - t0;
      n = len > 0 ? (len + DR_C - 1) / DR_C : 0;
    }
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    int woff = 0, total = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      woff += w < warp ? warp_sums[w] : 0;
      total += warp_sums[w];
    }
    const int first = carry + woff + incl - n;
    if (s < nseg) {
      table[s] = first;
      for (int c = 0; c < n; ++c) info[first + c] = make_int4(t0 + c * DR_C, min(DR_C, len - c * DR_C), t0, 0);
    }
    carry += total;
    __syncthreads();  // warp_sums is rewritten by the next pass
  }
  if (tid == 0) {
    table[nseg] = carry;
    table[nseg + 1] = 0;  // work counter of the recurrence
    table[nseg + 2] = 0;  // tile counter of the pipelined prep
  }
}

// byte offset of 16-byte chunk `c16` of row `r` in a [c16 / 8][rows][128 B] 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128_off(int r, int c16, int rows) {
  return (uint32_t)(c16 >> 3) * (uint32_t)(rows * 128) + (uint32_t)r * 128u + ((uint32_t)((c16 & 7) ^ (r & 7)) << 4);
}

// warp-uniform bounded wait: every lane polls, the warp proceeds only if all lanes saw the phase
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  const bool ok = sm100::mbar_wait(bar, parity, abort_flag);
  return __all_sync(0xffffffffu, ok ? 1 : 0) != 0;
}

// ---- 16x16 fp32 block products on the tensor cores: mma.sync m16n8k8 tf32 with the 3xTF32 split
//      (x = hi + lo, both tf32; x*y ~ hi*hi + hi*lo + lo*hi), accurate to about fp32.  One warp per
//      product; blocks are row-major in shared memory with row stride ld floats.
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
  const float r = x - __uint_as_float(hi);
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(r));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// acc = C (or 0 when C is null), in the m16n8 accumulator layout of two 8-column tiles
__device__ __forceinline__ void bmm16_init(float (&acc)[2][4], const float* C, int ld) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    acc[nt][0] = C ? C[g * ld + nt * 8 + 2 * t] : 0.f;
    acc[nt][1] = C ? C[g * ld + nt * 8 + 2 * t + 1] : 0.f;
    acc[nt][2] = C ? C[(g + 8) * ld + nt * 8 + 2 * t] : 0.f;
    acc[nt][3] = C ? C[(g + 8) * ld + nt * 8 + 2 * t + 1] : 0.f;
  }
}
// acc += X Y (16x16 each).  The three split terms and the two k halves accumulate into
// independent partial tiles, so the dependent mma chain is two deep instead of twelve.
__device__ __forceinline__ void bmm16_acc(float (&acc)[2][4], const float* X, const float* Y, int ld) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float part[2][3][2][4];
#pragma unroll
  for (int k = 0; k < 2; ++k)
#pragma unroll
    for (int q = 0; q < 3; ++q)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) part[k][q][nt][e] = 0.f;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int k0 = 8 * k;
    uint32_t ah[4], al[4];
    tf32_split(X[g * ld + k0 + t], ah[0], al[0]);
    tf32_split(X[(g + 8) * ld + k0 + t], ah[1], al[1]);
    tf32_split(X[g * ld + k0 + t + 4], ah[2], al[2]);
    tf32_split(X[(g + 8) * ld + k0 + t + 4], ah[3], al[3]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      uint32_t bh0, bl0, bh1, bl1;
      tf32_split(Y[(k0 + t) * ld + nt * 8 + g], bh0, bl0);
      tf32_split(Y[(k0 + t + 4) * ld + nt * 8 + g], bh1, bl1);
      mma_tf32(part[k][0][nt], al, bh0, bh1);
      mma_tf32(part[k][1][nt], ah, bl0, bl1);
      mma_tf32(part[k][2][nt], ah, bh0, bh1);
    }
  }
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      acc[nt][e] += ((part[0][0][nt][e] + part[1][0][nt][e]) + (part[0][1][nt][e] + part[1][1][nt][e])) +
                    (part[0][2][nt][e] + part[1][2][nt][e]);
}
__device__ __forceinline__ void bmm16_store(const float (&acc)[2][4], float* C, int ld) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    *reinterpret_cast<float2*>(C + g * ld + nt * 8 + 2 * t) = make_float2(acc[nt][0], acc[nt][1]);
    *reinterpret_cast<float2*>(C + (g + 8) * ld + nt * 8 + 2 * t) = make_float2(acc[nt][2], acc[nt][3]);
  }
}

// ------------------------------------------------------------------------------------------ prep
namespace dprep {
using namespace sm100;

constexpr int THREADS = 256;
constexpr int LDF = DR_C + 4;                 // fp32 tile stride: conflict-free column solves and row stores
constexpr uint32_t A1 = 0;                    // [2 dk halves][128 rows][128 B]: rows 0-63 k^, 64-127 q^ then V
constexpr uint32_t LF = 32768;                // fp32 L [64][LDF]; after the solve TU and TW (8 KB each)
constexpr uint32_t TU_OFF = LF, TW_OFF = LF + 8192;
constexpr uint32_t TF = LF + 64 * LDF * 4;    // fp32 T [64][LDF]
constexpr uint32_t VEC = TF + 64 * LDF * 4;   // G * log2(e), beta, beta e^G, -G * log2(e): [4][64] fp32
constexpr uint32_t BARS = VEC + 4 * 64 * 4;
enum { B_QK = 0, B_MMA1, B_V, B_MMA2, B_DRAIN, NBAR };
constexpr uint32_t SMEM_BYTES = BARS + 8 * NBAR + 16 + 1024;
constexpr uint32_t TM_D1 = 0, TM_U = 64, TM_W = 0, TM_COLS = 128;
constexpr float LOG2E = 1.4426950408889634f;
constexpr long long DRAIN_BUDGET = 2000000000LL;

// Inputs of the prep.  Plain: q / k / v through the tensor maps, g (fp32) and beta (bf16) [T, H].
// CONV (the fused GDN prologue): the [T, >= C] projection itself -- q / k / v come from the
// depthwise causal conv (width 4) + SiLU of its first C = 2 key_dim + value_dim columns, g and
// beta from its a / b columns (g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)), with
// the same arithmetic and bf16 roundings as the packed-conv and gate kernels.
struct PrepIn {
  const float* g;
  const bf16* beta;
  const bf16* proj;
  int64_t ld;
  const bf16* conv_w;  // [C][4]
  int key_dim;
  int a_col, b_col;
  const float* A_log;
  const float* dt_bias;
  int64_t tokens;
};

// conv + SiLU of one 8-channel group for ROWS consecutive tokens, from a raw projection box in
// shared memory ([67 rows][64 channels] bf16, row r = token t0 - 3 + r, rows past the tokens
// zero-filled by TMA), written as bf16 into a 128-byte-swizzled row of A1 (row srow0 + i, 16-byte
// chunk c16).  Raw rows below `first_valid` precede the segment start and read as zero.
template <int ROWS>
__device__ __forceinline__ void conv_rows(const uint8_t* box, int row0, int chunk, int first_valid, const bf16* wcol,
                                          uint8_t* a1, int srow0, int c16) {
  // Channel pairs run on the packed fp32 pipe (fma.rn.f32x2): per lane the same roundings as
  // the scalar mul / fma chain of the packed-conv kernel.
  float2 w[4][4];
  {
    const uint4* wp = reinterpret_cast<const uint4*>(wcol);  // 8 channels x 4 taps, contiguous
    float f[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      unpack8(__ldg(wp + q), f);  // channels 2q, 2q+1, taps 0..3 each
#pragma unroll
      for (int t = 0; t < 4; ++t) w[t][q] = make_float2(f[t], f[4 + t]);
    }
  }
  auto ld_row = [&](int r, float2 (&f)[4]) {
    if (r >= first_valid) {
      const uint4 u = *reinterpret_cast<const uint4*>(box + r * 128 + chunk * 16);
      f[0] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      f[1] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
      f[2] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.z));
      f[3] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.w));
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) f[c] = make_float2(0.f, 0.f);
    }
  };
  const float2 half2 = make_float2(0.5f, 0.5f);
  float2 h0[4], h1[4], h2[4];
  ld_row(row0, h0);
  ld_row(row0 + 1, h1);
  ld_row(row0 + 2, h2);
#pragma unroll
  for (int i = 0; i < ROWS; ++i) {
    float2 cur[4];
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
    ld_row(row0 + 3 + i, cur);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float2 acc = __fmul2_rn(w[3][c], cur[c]);
      acc = __ffma2_rn(w[2][c], h2[c], acc);
      acc = __ffma2_rn(w[1][c], h1[c], acc);
      acc = __ffma2_rn(w[0][c], h0[c], acc);
      const float2 hh = __fmul2_rn(half2, acc);  // silu(x) = h + h tanh(h), h = x / 2
      const float2 y = __ffma2_rn(hh, make_float2(tanh_approx(hh.x), tanh_approx(hh.y)), hh);
      o[c] = pack_bf16x2(y.x, y.y);
    }
    *reinterpret_cast<uint4*>(a1 + sw128_off(srow0 + i, c16, 128)) = out;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      h0[c] = h1[c];
      h1[c] = h2[c];
      h2[c] = cur[c];
    }
  }
}
constexpr uint32_t RAW_BOX = 67 * 128;  // one raw projection box: 67 rows x 64 bf16

// Block-wide barrier of the prep: the whole CTA (standalone kernel), or named barrier 1 over the
// 256 prep threads of a pipelined CTA (its other warps never take part in a prep tile).
template <bool PIPE>
__device__ __forceinline__ void prep_sync() {
  if constexpr (PIPE) asm volatile("bar.sync 1, 256;\n" ::: "memory");
  else __syncthreads();
}
template <bool PIPE>
__device__ __forceinline__ bool prep_sync_and(bool v) {
  if constexpr (PIPE) {
    uint32_t r;
    asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 256, p;\n selp.u32 %0, 1, 0, q;\n}\n"
                 : "=r"(r) : "r"((uint32_t)v) : "memory");
    return r != 0;
  } else {
    return __syncthreads_and(v) != 0;
  }
}

// One (chunk ci, head h) tile of the prep by 256 threads (tid 0-255).  Shared memory at `base`
// (1024-byte aligned; `sb` its generic address) with this file's prep layout and its barriers
// initialised; `tmem` holds TM_COLS allocated columns; `par` is the phase parity of this tile on
// every barrier (each completes once per tile).  Returns false if a bounded wait ran out.
template <bool CONV, bool PIPE>
__device__ __forceinline__ bool prep_tile(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                                          const CUtensorMap& mw_st, const CUtensorMap& mut_st,
                                          const PrepIn& in, const int4* __restrict__ info, int heads, float scale,
                                          uint8_t* __restrict__ tiles, int ci, int h, uint32_t base, uint8_t* sb,
                                          uint32_t tmem, uint32_t par) {
  float* G2 = reinterpret_cast<float*>(sb + VEC);  // G * log2(e)
  float* bet = G2 + 64;                            // beta (0 past the chunk's length)
  float* fw = G2 + 128;                            // beta e^G
  float* nG2 = G2 + 192;                           // -G * log2(e)
  float* Lf = reinterpret_cast<float*>(sb + LF);
  float* Tf = reinterpret_cast<float*>(sb + TF);
  const uint32_t bar0 = base + BARS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sb + BARS + 8 * NBAR);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int4 inf = info[ci];
  const int t0 = inf.x, len = inf.y, seg_start = inf.z;
  uint8_t* tile = tiles + ((size_t)ci * heads + h) * CH_BYTES;
  PHASE_START();
  bool issued_v = false, issued_mma = false;

  // 1. raw k rows -> A1 rows 0-63, raw q rows -> rows 64-127 (TMA, 128-byte swizzle; rows past
  //    the end of the tokens read as zero, rows of the next segment are masked below).
  //    CONV: the projection's raw k and q columns of this head, 3 history rows included, land in
  //    the L / T area (free until the solve) as four [67][64] boxes: k0 k1 q0 q1.
  if (CONV && tid == 0) {
    prefetch_tmap(&mq);
    mbar_expect_tx(bar0 + 8 * B_QK, 4 * RAW_BOX);
#pragma unroll
    for (int bx = 0; bx < 4; ++bx) {
      const int col = (bx < 2 ? in.key_dim : 0) + h * DR_D + (bx & 1) * 64;
      tma_load_2d(base + LF + bx * RAW_BOX, &mq, bar0 + 8 * B_QK, col, t0 - 3);
    }
  }
  if (!CONV && tid == 0) {
    prefetch_tmap(&mq);
    prefetch_tmap(&mk);
    prefetch_tmap(&mv);
    mbar_expect_tx(bar0 + 8 * B_QK, 4 * 8192);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      tma_load_2d(base + A1 + hf * 16384, &mk, bar0 + 8 * B_QK, h * DR_D + hf * 64, t0);
      tma_load_2d(base + A1 + hf * 16384 + 8192, &mq, bar0 + 8 * B_QK, h * DR_D + hf * 64, t0);
    }
  }
  // decay cumsum (log2 domain), beta and the column factors of TU / TW
  if (warp == 1) {
    const int r0 = 2 * lane, r1 = 2 * lane + 1;
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
    if (CONV) {  // gates from the projection's a / b columns
      const float el = -expf(in.A_log[h]), dtb = in.dt_bias[h];
      if (r0 < len) {
        const bf16* row = in.proj + (int64_t)(t0 + r0) * in.ld;
        a0 = el * softplusf_(__bfloat162float(row[in.a_col + h]) + dtb);
        b0 = round_bf16(sigmoidf_(__bfloat162float(row[in.b_col + h])));
      }
      if (r1 < len) {
        const bf16* row = in.proj + (int64_t)(t0 + r1) * in.ld;
        a1 = el * softplusf_(__bfloat162float(row[in.a_col + h]) + dtb);
        b1 = round_bf16(sigmoidf_(__bfloat162float(row[in.b_col + h])));
      }
    } else {
      if (r0 < len) { a0 = in.g[(int64_t)(t0 + r0) * heads + h]; b0 = __bfloat162float(in.beta[(int64_t)(t0 + r0) * heads + h]); }
      if (r1 < len) { a1 = in.g[(int64_t)(t0 + r1) * heads + h]; b1 = __bfloat162float(in.beta[(int64_t)(t0 + r1) * heads + h]); }
    }
    const float pair = a0 + a1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const float G0 = incl - pair + a0, G1 = incl;  // natural-log cumsum at r0, r1
    G2[r0] = G0 * LOG2E;
    G2[r1] = G1 * LOG2E;
    nG2[r0] = -(G0 * LOG2E);
    nG2[r1] = -(G1 * LOG2E);
    bet[r0] = b0;
    bet[r1] = b1;
    fw[r0] = b0 * expf(G0);
    fw[r1] = b1 * expf(G1);
    if (lane == 31) *reinterpret_cast<float*>(tile + OFF_GAMMA) = expf(G1);
  }
  bool ok = mbar_wait(bar0 + 8 * B_QK, par, abort_flag);
  if (CONV && ok) {  // q (A1 rows 64-127) and k (rows 0-63): thread = 8 channels x 8 tokens
    const int g8 = tid & 31, rs = tid >> 5;
    const bool isk = g8 >= 16;
    const int c16 = g8 & 15;
    const int first_valid = max(0, seg_start - (t0 - 3));
    const bf16* wcol = in.conv_w + ((isk ? in.key_dim : 0) + (int64_t)h * DR_D + c16 * 8) * 4;
    const uint8_t* box = sb + LF + ((isk ? 0 : 2) + (c16 >> 3)) * RAW_BOX;
    conv_rows<8>(box, rs * 8, c16 & 7, first_valid, wcol, sb + A1, (isk ? 0 : 64) + rs * 8, c16);
    fence_proxy_async_smem();  // the raw boxes are refilled by TMA (V) below
  }
  PHASE(1);
  ok = prep_sync_and<PIPE>(ok);  // also publishes G2 / beta / fw
  if (CONV && ok && tid == 0) {  // raw v columns -> the T area, landing while k / q are normalised
    mbar_expect_tx(bar0 + 8 * B_V, 2 * RAW_BOX);
    tma_load_2d(base + TF, &mq, bar0 + 8 * B_V, 2 * in.key_dim + h * DR_D, t0 - 3);
    tma_load_2d(base + TF + RAW_BOX, &mq, bar0 + 8 * B_V, 2 * in.key_dim + h * DR_D + 64, t0 - 3);
    issued_v = true;
  }

  if (ok) {
    // 2. l2-normalise k and q rows (q also times scale) in place, zero rows past the length;
    //    decayed copies Kg = k e^(G_last - G), Qg = q e^G out (from the bf16-rounded normalised
    //    values the products see).  Four threads per row; thread `part` takes the 16-byte chunks
    //    part, part + 4, part + 8, part + 12, so each warp store writes 64 contiguous bytes a row.
    const int row = tid >> 2, part = tid & 3;
    const bool valid = row < len;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int srow = rr * 64 + row;
      uint4 u[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) u[j] = *reinterpret_cast<const uint4*>(sb + A1 + sw128_off(srow, part + 4 * j, 128));
      // packed fp32 pipe (f32x2) for the sum of squares and both scalings
      float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&u[j]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(hp[e]);
          ss2 = __ffma2_rn(f, f, ss2);
        }
      }
      float ss = ss2.x + ss2.y;
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      const float inv = valid ? rsqrtf(ss + 1e-6f) * (rr ? scale : 1.0f) : 0.f;
      const float dec = rr ? exp2f(G2[row]) : exp2f(G2[63] - G2[row]);
      const float2 inv2 = make_float2(inv, inv), dec2 = make_float2(dec, dec);
      uint4* gout = reinterpret_cast<uint4*>(tile + (rr ? OFF_QG : OFF_KG) + (size_t)row * 256);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&u[j]);
        uint4 nb, db;
        uint32_t* np = reinterpret_cast<uint32_t*>(&nb);
        uint32_t* dp = reinterpret_cast<uint32_t*>(&db);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __fmul2_rn(__bfloat1622float2(hp[e]), inv2);
          np[e] = pack_bf16x2(f.x, f.y);
          const float2 d = __fmul2_rn(__bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&np[e])), dec2);
          dp[e] = pack_bf16x2(d.x, d.y);
        }
        *reinterpret_cast<uint4*>(sb + A1 + sw128_off(srow, part + 4 * j, 128)) = nb;
        gout[part + 4 * j] = db;
      }
    }
    fence_proxy_async_smem();
  }
  prep_sync<PIPE>();

  PHASE(2);
  // 3. D1 = [K^; Q^] K^T  (M128 N64 K128; B is A's first 64 rows)
  if (ok && tid == 0) {
    tc_fence_after();
    constexpr uint32_t ID = idesc_bf16(128, 64, false, false);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint64_t d = sdesc_sw128(base + A1 + (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u, 16, 1024);
      umma_ss(tmem + TM_D1, d, d, ID, kk > 0 ? 1u : 0u);
    }
    umma_commit(bar0 + 8 * B_MMA1);
    issued_mma = true;
  }
  if (ok) ok = warp_wait(bar0 + 8 * B_MMA1, par, abort_flag);
  if (ok) tc_fence_after();
  // V rows -> A1 rows 64-127 (q^ is no longer read), landing while the solve runs
  PHASE(3);
  if (CONV && ok) ok = warp_wait(bar0 + 8 * B_V, par, abort_flag);
  if (CONV && ok) {  // v by conv into A1 rows 64-127: thread = 8 channels x 4 tokens
    const int g8 = tid & 15, rs = tid >> 4;
    const int first_valid = max(0, seg_start - (t0 - 3));
    const bf16* wcol = in.conv_w + (2 * (int64_t)in.key_dim + (int64_t)h * DR_D + g8 * 8) * 4;
    conv_rows<4>(sb + TF + (g8 >> 3) * RAW_BOX, rs * 4, g8 & 7, first_valid, wcol, sb + A1, 64 + rs * 4, g8);
    fence_proxy_async_smem();
  }
  if (!CONV && ok && tid == 0) {
    mbar_expect_tx(bar0 + 8 * B_V, 2 * 8192);
    tma_load_2d(base + A1 + 8192, &mv, bar0 + 8 * B_V, h * DR_D, t0);
    tma_load_2d(base + A1 + 16384 + 8192, &mv, bar0 + 8 * B_V, h * DR_D + 64, t0);
    issued_v = true;
  }

  PHASE(4);
  // 4. rows of D1: L = -beta_i (KK^T)_ij e^(G_i - G_j) (j < i) -> smem; Aqk = (QK^T)_ij e^(G_i - G_j)
  //    (j <= i) -> workspace.  Warp w reads TMEM lane quarter w % 4, column half w / 4.
  if (ok) {
    const int q4 = warp & 3, chh = warp >> 2;
    uint32_t v[32];
    tmem_ld32(tmem + ((uint32_t)(q4 * 32) << 16) + TM_D1 + chh * 32, v);
    tmem_ld_wait();
    const int i = (q4 & 1) * 32 + lane;
    const float g2i = G2[i];
    const float2 g2i2 = make_float2(g2i, g2i);
    // decay e^(G_i - G_j) for the row's 32 columns j, pairs on the packed fp32 pipe
    // (g2i + (-G_j) is the same rounding as g2i - G_j)
    auto decay8 = [&](int j8, float2 (&e2)[4]) {
      const float4 na = *reinterpret_cast<const float4*>(nG2 + chh * 32 + j8 * 8);
      const float4 nc = *reinterpret_cast<const float4*>(nG2 + chh * 32 + j8 * 8 + 4);
      const float2 d[4] = {__fadd2_rn(g2i2, make_float2(na.x, na.y)), __fadd2_rn(g2i2, make_float2(na.z, na.w)),
                           __fadd2_rn(g2i2, make_float2(nc.x, nc.y)), __fadd2_rn(g2i2, make_float2(nc.z, nc.w))};
#pragma unroll
      for (int p = 0; p < 4; ++p) e2[p] = make_float2(ex2(d[p].x), ex2(d[p].y));
    };
    if (q4 < 2) {
      const float nb = -bet[i];
      const float2 nb2 = make_float2(nb, nb);
      float* dst = Lf + i * LDF + chh * 32;
#pragma unroll
      for (int j8 = 0; j8 < 4; ++j8) {
        float2 e2[4];
        decay8(j8, e2);
        float l[8];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 vv = make_float2(__uint_as_float(v[j8 * 8 + 2 * p]), __uint_as_float(v[j8 * 8 + 2 * p + 1]));
          const float2 y = __fmul2_rn(__fmul2_rn(nb2, vv), e2[p]);
          const int j = chh * 32 + j8 * 8 + 2 * p;
          l[2 * p] = j < i ? y.x : 0.f;
          l[2 * p + 1] = j + 1 < i ? y.y : 0.f;
        }
        *reinterpret_cast<float4*>(dst + j8 * 8) = make_float4(l[0], l[1], l[2], l[3]);
        *reinterpret_cast<float4*>(dst + j8 * 8 + 4) = make_float4(l[4], l[5], l[6], l[7]);
      }
    } else {
      uint4* dst = reinterpret_cast<uint4*>(tile + OFF_A + (size_t)i * 128 + chh * 64);
#pragma unroll
      for (int j8 = 0; j8 < 4; ++j8) {
        float2 e2[4];
        decay8(j8, e2);
        uint4 out;
        uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 vv = make_float2(__uint_as_float(v[j8 * 8 + 2 * p]), __uint_as_float(v[j8 * 8 + 2 * p + 1]));
          const float2 y = __fmul2_rn(vv, e2[p]);
          const int j = chh * 32 + j8 * 8 + 2 * p;
          o[p] = pack_bf16x2(j <= i ? y.x : 0.f, j + 1 <= i ? y.y : 0.f);
        }
        dst[j8] = out;
      }
    }
  }
  tc_fence_before();
  prep_sync<PIPE>();

  PHASE(5);
  // 5. T = (I - L)^-1 in fp32.
  //    Level 0 (warps 0-1, thread = one column k of one diagonal block b): forward substitution
  //    down the column, x_r = d_rk + sum_{j<r} N_rj x_j with the FMAs in increasing j (the
  //    reference's row-by-row update order); rows of N are shared-memory broadcasts within the
  //    block's 16 threads and x stays in registers.
  //    Levels 1-3: 16x16 block products on the tensor cores (mma.sync tf32, 3xTF32 split,
  //    fp32-accurate): T_10 = T_11 L_10 T_00 and T_32 = T_33 L_32 T_22; then the 32x32 corner
  //    T_[23][01] = T_[23][23] (L_[23][01] T_[01][01]) as X = L T then Y = T X, four blocks each.
  //    Scratch: the unused upper blocks of L.
  if (ok && warp < 2) {
    const int b = tid >> 4, k = tid & 15;
    const float* nb = Lf + (16 * b) * LDF + 16 * b;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float n[16];
#pragma unroll
      for (int j4 = 0; j4 < (r + 3) / 4; ++j4) {
        const float4 q = *reinterpret_cast<const float4*>(nb + r * LDF + 4 * j4);
        n[4 * j4] = q.x;
        n[4 * j4 + 1] = q.y;
        n[4 * j4 + 2] = q.z;
        n[4 * j4 + 3] = q.w;
      }
      float acc = r == k ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) acc = fmaf(n[j], x[j], acc);
      x[r] = acc;
    }
    float* tcol = Tf + (16 * b) * LDF + 16 * b + k;
#pragma unroll
    for (int r = 0; r < 16; ++r) tcol[r * LDF] = x[r];
  }
  prep_sync<PIPE>();
  auto blk = [&](float* base_, int bi, int bj) { return base_ + (16 * bi) * LDF + 16 * bj; };
  PHASE(6);
  // level 1: warp 0 -> T_10, warp 1 -> T_32
  if (ok && warp < 2) {
    const int j = 2 * warp, i = j + 1;
    float acc[2][4];
    bmm16_init(acc, nullptr, 0);
    bmm16_acc(acc, blk(Lf, i, j), blk(Tf, j, j), LDF);
    float* M = blk(Lf, j, i);
    bmm16_store(acc, M, LDF);
    __syncwarp();
    bmm16_init(acc, nullptr, 0);
    bmm16_acc(acc, blk(Tf, i, i), M, LDF);
    bmm16_store(acc, blk(Tf, i, j), LDF);
  }
  prep_sync<PIPE>();
  PHASE(7);
  // level 2: X_ij (i in {2,3}, j in {0,1}) = L_i0 T_0j + L_i1 T_1j (T_01 = 0) into L's block (j, i)
  if (ok && warp < 4) {
    const int i = 2 + (warp >> 1), j = warp & 1;
    float acc[2][4];
    bmm16_init(acc, nullptr, 0);
    if (j == 0) bmm16_acc(acc, blk(Lf, i, 0), blk(Tf, 0, 0), LDF);
    bmm16_acc(acc, blk(Lf, i, 1), blk(Tf, 1, j), LDF);
    bmm16_store(acc, blk(Lf, j, i), LDF);
  }
  prep_sync<PIPE>();
  PHASE(8);
  // level 3: T_ij = T_i2 X_2j + T_i3 X_3j (T_23 = 0)
  if (ok && warp < 4) {
    const int i = 2 + (warp >> 1), j = warp & 1;
    float acc[2][4];
    bmm16_init(acc, nullptr, 0);
    bmm16_acc(acc, blk(Tf, i, 2), blk(Lf, j, 2), LDF);
    if (i == 3) bmm16_acc(acc, blk(Tf, 3, 3), blk(Lf, j, 3), LDF);
    bmm16_store(acc, blk(Tf, i, j), LDF);
  }
  prep_sync<PIPE>();

  PHASE(9);
  // 6. TU = bf16(T diag(beta)), TW = bf16(T diag(beta e^G)) as K-major swizzled B tiles (over L)
  if (ok) {
    for (int e = tid; e < 64 * 8; e += THREADS) {
      const int r = e & 63, c8 = e >> 6;
      float t8[8], tu[8], tw[8];
      *reinterpret_cast<float4*>(&t8[0]) = *reinterpret_cast<const float4*>(Tf + r * LDF + c8 * 8);
      *reinterpret_cast<float4*>(&t8[4]) = *reinterpret_cast<const float4*>(Tf + r * LDF + c8 * 8 + 4);
      const bool live = (c8 >> 1) <= (r >> 4);  // block-lower part of T (its upper blocks are unset)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float t = live ? t8[j] : 0.f;
        tu[j] = t * bet[c8 * 8 + j];
        tw[j] = t * fw[c8 * 8 + j];
      }
      const uint32_t off = (uint32_t)r * 128u + ((uint32_t)(c8 ^ (r & 7)) << 4);
      *reinterpret_cast<uint4*>(sb + TU_OFF + off) = pack8(tu);
      *reinterpret_cast<uint4*>(sb + TW_OFF + off) = pack8(tw);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  prep_sync<PIPE>();

  PHASE(10);
  // 7. U^T = V^T TU^T and W^T = K^T TW^T  (M128 N64 K64; A = V / K^ MN-major, B = TU / TW K-major)
  if (ok && tid == 0) {
    if (CONV || mbar_wait(bar0 + 8 * B_V, par, abort_flag)) {
      tc_fence_after();
      constexpr uint32_t ID = idesc_bf16(128, 64, true, false);
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        umma_ss(tmem + TM_U, sdesc_sw128(base + A1 + 8192 + kt * 2048, 16384, 1024),
                sdesc_sw128(base + TU_OFF + kt * 32, 16, 1024), ID, kt > 0 ? 1u : 0u);
        umma_ss(tmem + TM_W, sdesc_sw128(base + A1 + kt * 2048, 16384, 1024),
                sdesc_sw128(base + TW_OFF + kt * 32, 16, 1024), ID, kt > 0 ? 1u : 0u);
      }
      umma_commit(bar0 + 8 * B_MMA2);
    }
  }
  if (ok) ok = warp_wait(bar0 + 8 * B_MMA2, par, abort_flag);
  PHASE(11);
  // 8. U^T rows (warps 0-3) and W^T rows (warps 4-7) -> workspace, one 128-byte row per thread
  if (ok) {
    tc_fence_after();
    const int q4 = warp & 3, which = warp >> 2;
    const int r = q4 * 32 + lane;
    uint32_t v[2][32];
    const uint32_t ta = tmem + ((uint32_t)(q4 * 32) << 16) + (which ? TM_W : TM_U);
    tmem_ld32(ta, v[0]);
    tmem_ld32(ta + 32, v[1]);
    tmem_ld_wait();
    // staged 128-byte-swizzled in A1 (free: the second MMA has completed) and written as one
    // [128][64] TMA box a tile (16-byte row pieces from 32 rows at once would be half sectors)
    uint8_t* dst = sb + A1 + which * 16384 + r * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[j >> 2][(j & 3) * 8 + e]);
      *reinterpret_cast<uint4*>(dst + ((j ^ (r & 7)) << 4)) = pack8(f);
    }
    fence_proxy_async_smem();
  }
  ok = prep_sync_and<PIPE>(ok);
  if (ok && tid == 0) {
    const int z = ci * heads + h;
    tma_store_3d(&mut_st, base + A1, 0, 0, z);
    tma_store_3d(&mw_st, base + A1 + 16384, 0, 0, z);
    bulk_commit();
    bulk_wait<0>();  // complete (not just read) before the tile is published or A1 is reused
  }
  PHASE(12);
  // teardown: on a bounded-wait failure, let in-flight copies and MMAs land before TMEM and
  // shared memory are released
  if (tid == 0 && *abort_flag) {
    volatile int never = 0;
    mbar_wait(bar0 + 8 * B_QK, par, &never, DRAIN_BUDGET);
    if (issued_v) mbar_wait(bar0 + 8 * B_V, par, &never, DRAIN_BUDGET);
    if (issued_mma) {  // every MMA this thread issued has completed
      umma_commit(bar0 + 8 * B_DRAIN);
      mbar_wait(bar0 + 8 * B_DRAIN, 0, &never, DRAIN_BUDGET);
    }
    atomicOr(&g_delta_error, 1);
  }
  return *abort_flag == 0;
}

template <bool CONV>
__global__ void __launch_bounds__(THREADS, 3) delta_prep_kernel(
    const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
    const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mw_st,
    const __grid_constant__ CUtensorMap mut_st, const PrepIn in, const int4* __restrict__ info,
    const int32_t* __restrict__ table, int nseg, int heads, float scale, uint8_t* __restrict__ tiles) {
  extern __shared__ uint8_t smem_raw[];
  const int ci = blockIdx.x, h = blockIdx.y;
  if (ci >= table[nseg]) return;  // CTA-uniform, before any barrier or TMEM use
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sb = smem_raw + (base - raw);
  const uint32_t bar0 = base + BARS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sb + BARS + 8 * NBAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sb + BARS + 8 * NBAR + 4);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(bar0 + 8 * i, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  prep_tile<CONV, false>(mq, mk, mv, mw_st, mut_st, in, info, heads, scale, tiles, ci, h, base, sb, tmem, 0);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

}  // namespace dprep

// ------------------------------------------------------------------------------------- recurrence
// tcgen05 recurrence, persistent: each CTA takes (segment, head) chains from an atomic work counter
// and runs them chunk by chunk; the tile ring runs ahead across chain boundaries.
//   TMEM (512 columns of fp32; lane = dv row): S^T [0,128), vn [128,192), o^T [192,256) and
//   [256,320) (double-buffered so the output epilogue leaves the critical path).
//   Per chunk n (tiles W^T, Qg, Kg, Aqk, U^T of the chunk in a 2-stage TMA ring, 128-byte swizzle):
//     state warps : S^T -> bf16 A tile in SMEM; S^T *= gamma in TMEM
//     MMA thread  : vn = S^T W^T (M128 N64 K128); then o^T = S^T Qg^T
//     state warps : v_new^T = U^T - vn -> bf16 A tile in SMEM; then o^T of chunk n-1 -> out
//     MMA thread  : S^T += v_new^T Kg (M128 N128 K64, Kg MN-major); then o^T += v_new^T Aqk^T
//   Warps: 0 TMA producer (and work counter), 1 TMEM allocator + single-thread MMA issuer, 2-9
//   state warps (two per TMEM lane quarter, each owning half of a dv row's columns).  Every mbarrier wait is bounded; a wait that
//   runs out sets the device error word, and the CTA drains its copies and MMAs, frees TMEM and
//   returns.
namespace drtc {
using namespace sm100;

constexpr uint32_t KM_HALF = 64 * 128;  // [64 rows][128 B] swizzled block (one TMA box)
constexpr uint32_t ST_W = 0, ST_QG = 2 * KM_HALF, ST_KG = 4 * KM_HALF, ST_A = 6 * KM_HALF, ST_UT = 7 * KM_HALF,
                   ST_BYTES = 9 * KM_HALF;           // U^T: [128 dv][128 B]
constexpr uint32_t OFF_SA = 2 * ST_BYTES;            // S^T bf16 A tile: [2 dk halves][128 dv][128 B]
constexpr uint32_t OFF_VA = OFF_SA + 2 * 128 * 128;  // v_new^T bf16 A tile: [128 dv][128 B]
constexpr uint32_t OFF_OST = OFF_VA + 128 * 128;     // o staging: per state warp [32 tok][32 dv] bf16
constexpr uint32_t OFF_META = OFF_OST + 4 * 64 * 32 * 2;
constexpr uint32_t OFF_BAR = OFF_META + 2 * 32;
enum { B_FULL0 = 0, B_FULL1, B_EMPTY0, B_EMPTY1, B_SA, B_VN, B_VNEW, B_SDONE, B_ODONE0, B_ODONE1, B_DRAIN, NBAR };
constexpr uint32_t SMEM_BYTES = OFF_BAR + 8 * NBAR + 16 + 1024;
constexpr int THREADS = 320;
constexpr uint32_t TM_S = 0, TM_VN = 128, TM_O = 192, TM_COLS = 512;
constexpr long long DRAIN_BUDGET = 2000000000LL;

struct RParams {
  const int32_t* cu;
  const int32_t* table;
  int32_t* work_counter;  // zeroed by the chunk-table kernel of the same call
  int nseg, heads;
  const uint8_t* tiles;   // gamma is read from here directly
  const float* init_state;
  bf16* out;
  float* final_state;
  const int* tile_ready;  // pipelined launch: per (chunk, head) tile, set once the prep has written it
};

// Bounded wait until *flag != 0 (acquire), then a proxy fence so the TMA loads that follow see the
// tile the flag publishes.  Gives up after ~budget SM cycles, raising *abort.
__device__ __forceinline__ bool wait_tile_ready(const int* flag, volatile int* abort, long long budget = 4000000000LL) {
  auto ld = [&]() {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(flag) : "memory");
    return v;
  };
  if (!ld()) {
    const long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
      if (ld()) break;
      __nanosleep(64);
      if ((i & 63) == 0 && (*abort || clock64() - t0 > budget)) {
        *abort = 1;
        return false;
      }
    }
  }
  asm volatile("fence.proxy.async.global;\n" ::: "memory");
  return true;
}

struct StageMeta {  // written by the producer before the stage's expect_tx arrive
  int s, h, c, nch;
  float gamma;
  int half;  // SPLIT == 2: which 64 dv rows of the head this chain carries
  int pad[2];
};

// SPLIT == 1: a chain is one (segment, head); the state S^T is 128 dv rows (M = 128 MMAs).
// SPLIT == 2: every dv row of S^T evolves on its own (v_new, o and the update of row r read only
// row r of S^T, U^T and vn), so a (segment, head) is run as two chains of 64 dv rows each on two
// CTAs: twice the chains when there are fewer chains than SMs (batch 1 has 16), with M = 64 MMAs
// (accumulator rows in lanes 0-15 of each TMEM lane quarter) and only that half of U^T loaded.
// PIPE: the tiles are produced during this launch by other CTAs (gdn_pipe_kernel): the producer
// acquires each tile's ready flag before loading it and reads gamma coherently.
template <int SPLIT, bool PIPE>
__device__ __forceinline__ void recur_body(const CUtensorMap& mw, const CUtensorMap& mqg, const CUtensorMap& mkg,
                                           const CUtensorMap& ma, const CUtensorMap& mut, const RParams& p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + OFF_BAR;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * NBAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + 8 * NBAR + 4);
  volatile StageMeta* meta = reinterpret_cast<volatile StageMeta*>(gbase + OFF_META);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = p.heads;

  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(bar0 + 8 * i, (i == B_SA || i == B_VNEW) ? 256u : 1u);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&mw);
      prefetch_tmap(&mqg);
      prefetch_tmap(&mkg);
      prefetch_tmap(&ma);
      prefetch_tmap(&mut);
      const int items = p.nseg * H * SPLIT;
      constexpr uint32_t stage_tx = SPLIT == 1 ? ST_BYTES : ST_BYTES - KM_HALF;  // U^T: 128 or 64 dv rows
      int n = 0;  // real chunks pushed into the ring by this CTA
      bool closed = false;
      while (true) {
        const int item = atomicAdd(p.work_counter, 1);
        if (item >= items) {  // closing stage: s = -1, no tiles
          const int st = n & 1;
          if (n >= 2 && !mbar_wait(bar0 + 8 * (B_EMPTY0 + st), ((n >> 1) - 1) & 1, abort_flag)) break;
          meta[st].s = -1;
          mbar_arrive(bar0 + 8 * (B_FULL0 + st));
          closed = true;
          break;
        }
        const int s = item / (H * SPLIT), rem = item - s * (H * SPLIT), h = rem / SPLIT, half = rem - h * SPLIT;
        const int c0 = __ldg(p.table + s), nch = __ldg(p.table + s + 1) - c0;
        bool ok = true;
        for (int c = 0; c < nch; ++c, ++n) {
          const int st = n & 1;
          if (n >= 2 && !mbar_wait(bar0 + 8 * (B_EMPTY0 + st), ((n >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
          const int z = (c0 + c) * H + h;
          if constexpr (PIPE) {
            if (!wait_tile_ready(p.tile_ready + z, abort_flag)) { ok = false; break; }
          }
          meta[st].s = s;
          meta[st].h = h;
          meta[st].c = c;
          meta[st].nch = nch;
          meta[st].half = half;
          const float* gp = reinterpret_cast<const float*>(p.tiles + (size_t)z * CH_BYTES + OFF_GAMMA);
          meta[st].gamma = PIPE ? *reinterpret_cast<const volatile float*>(gp) : __ldg(gp);
          const uint32_t sb = base + st * ST_BYTES;
          const uint32_t fb = bar0 + 8 * (B_FULL0 + st);
          mbar_expect_tx(fb, stage_tx);
          tma_load_3d(sb + ST_W, &mw, fb, 0, 0, z);
          tma_load_3d(sb + ST_QG, &mqg, fb, 0, 0, z);
          tma_load_3d(sb + ST_QG + KM_HALF, &mqg, fb, 64, 0, z);
          tma_load_3d(sb + ST_KG, &mkg, fb, 0, 0, z);
          tma_load_3d(sb + ST_KG + KM_HALF, &mkg, fb, 64, 0, z);
          tma_load_3d(sb + ST_A, &ma, fb, 0, 0, z);
          tma_load_3d(sb + ST_UT, &mut, fb, 0, 64 * half, z);  // SPLIT == 2: the map's box is 64 rows
        }
        if (!ok) break;
      }
      // Before the CTA exits every issued copy has landed.  Real chunk m's phase is the newest of
      // its FULL barrier unless the closing stage followed on the same barrier, which it only did
      // after chunk m's tiles were consumed.
      volatile int never = 0;
      for (int m = n > 2 ? n - 2 : 0; m < n; ++m)
        if (!(closed && ((m ^ n) & 1) == 0))
          mbar_wait(bar0 + 8 * (B_FULL0 + (m & 1)), (m >> 1) & 1, &never, DRAIN_BUDGET);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr int MR = 128 / SPLIT;  // dv rows of the chain: the MMAs' M
      constexpr uint32_t A_KHALF = (uint32_t)MR * 128u;  // bytes of one 64-wide dk half of the S^T A tile
      constexpr uint32_t ID_N64 = idesc_bf16(MR, 64, false, false);
      constexpr uint32_t ID_N64_BMN = idesc_bf16(MR, 64, false, true);
      constexpr uint32_t ID_N128_BMN = idesc_bf16(MR, 128, false, true);
      const uint64_t dSA = sdesc_sw128(base + OFF_SA, 16, 1024), dVA = sdesc_sw128(base + OFF_VA, 16, 1024);
      for (int n = 0;; ++n) {
        const int st = n & 1;
        const uint32_t sb = base + st * ST_BYTES;
        if (!mbar_wait(bar0 + 8 * (B_FULL0 + st), (n >> 1) & 1, abort_flag)) break;
        if (meta[st].s < 0) break;
        if (!mbar_wait(bar0 + 8 * B_SA, n & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t tO = tmem + TM_O + 64u * (uint32_t)st;
        // Descriptors are built once per stage; a k step adds its byte offset / 16 to the start
        // address field (shared-memory addresses stay below 2^18, so the field never carries).
        const uint64_t dW = sdesc_sw128(sb + ST_W, KM_HALF, 1024), dQG = sdesc_sw128(sb + ST_QG, 16, 1024),
                       dKG = sdesc_sw128(sb + ST_KG, KM_HALF, 1024), dA = sdesc_sw128(sb + ST_A, 16, 1024);
        // vn = S^T W^T  (K = 128 dk: 2 swizzle halves x 4 steps of 16; W^T [dk][tok] is MN-major)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t aoff = (uint32_t)(kk >> 2) * A_KHALF + (uint32_t)(kk & 3) * 32u;
          umma_ss(tmem + TM_VN, dSA + (aoff >> 4), dW + ((uint32_t)kk * 2048u >> 4), ID_N64_BMN, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar0 + 8 * B_VN);
        // o^T = S^T Qg^T
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t aoff = (uint32_t)(kk >> 2) * A_KHALF + (uint32_t)(kk & 3) * 32u;
          const uint32_t boff = (uint32_t)(kk >> 2) * KM_HALF + (uint32_t)(kk & 3) * 32u;
          umma_ss(tO, dSA + (aoff >> 4), dQG + (boff >> 4), ID_N64, kk > 0 ? 1u : 0u);
        }
        if (!mbar_wait(bar0 + 8 * B_VNEW, n & 1, abort_flag)) break;
        tc_fence_after();
        // S^T += v_new^T Kg  (Kg MN-major: [2 dk halves][64 tok][128 B]; K = 64 tokens in 4 steps)
#pragma unroll
        for (int kt = 0; kt < 4; ++kt)
          umma_ss(tmem + TM_S, dVA + (uint32_t)(kt * 32 >> 4), dKG + (uint32_t)(kt * 2048 >> 4), ID_N128_BMN, 1u);
        umma_commit(bar0 + 8 * B_SDONE);
        // o^T += v_new^T Aqk^T
#pragma unroll
        for (int kt = 0; kt < 4; ++kt)
          umma_ss(tO, dVA + (uint32_t)(kt * 32 >> 4), dA + (uint32_t)(kt * 32 >> 4), ID_N64, 1u);
        umma_commit(bar0 + 8 * (B_ODONE0 + st));
        umma_commit(bar0 + 8 * (B_EMPTY0 + st));
      }
      // every MMA issued above has completed before TMEM is freed
      volatile int never = 0;
      umma_commit(bar0 + 8 * B_DRAIN);
      mbar_wait(bar0 + 8 * B_DRAIN, 0, &never, DRAIN_BUDGET);
    }
  } else {
    // ---------------------------------------------------------------- state warps (256 threads)
    // Two warps per TMEM lane quarter; warp half `hf` owns half of every row's columns: S^T
    // columns [64 hf, +64), vn / o columns (tokens) [32 hf, +32).
    // SPLIT == 1: thread = dv row (TMEM lane) and all of its warp half's columns.
    // SPLIT == 2: thread = chain row 16 q4 + (lane & 15) (TMEM lanes 0-15 of the quarter, the M = 64
    //   accumulator layout) and column part sub = lane >> 4 of its warp half's columns: S^T
    //   columns [64 hf + 32 sub, +32), vn / o columns [32 hf + 16 sub, +16) (16x32bx2 accesses).
    constexpr int MR = 128 / SPLIT;   // dv rows of a chain
    const int q4 = warp & 3;          // the TMEM lane quarter this warp may access
    const int hf = (warp - 2) >> 2;   // 0 for warps 2-5, 1 for warps 6-9
    const int sub = SPLIT == 2 ? lane >> 4 : 0;
    const int r = SPLIT == 1 ? q4 * 32 + lane : q4 * 16 + (lane & 15);  // row of the chain's S^T
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    const uint32_t tS = tmem + lane_addr + TM_S + 64 * hf, tVN = tmem + lane_addr + TM_VN + 32 * hf,
                   tO = tmem + lane_addr + TM_O + 32 * hf;
    uint8_t* sa = gbase + OFF_SA;
    uint8_t* va = gbase + OFF_VA;
    // o staging per state warp: [32 tok][32 dv] (SPLIT 1) or [32 tok][16 dv] (SPLIT 2) bf16
    bf16* ost = reinterpret_cast<bf16*>(gbase + OFF_OST) + (hf * 4 + q4) * (32 * 32);
    constexpr int NCB = SPLIT == 1 ? 2 : 1;  // 32-column S^T pieces per thread
    auto scol = [&](int cb) { return 64 * hf + 32 * (SPLIT == 1 ? cb : sub); };  // first dk column of piece cb
    auto s_ld = [&](int cb, uint32_t (&v)[32]) {
      if constexpr (SPLIT == 1) tmem_ld32(tS + cb * 32, v); else tmem_ld16x2_x32(tS, v);
    };
    auto s_st = [&](int cb, const uint32_t (&v)[32]) {
      if constexpr (SPLIT == 1) tmem_st32(tS + cb * 32, v); else tmem_st16x2_x32(tS, v);
    };

    // o^T of chunk (s, h, c) (complete in TMEM buffer b) -> out[token][h][dv]
    auto o_epilogue = [&](int b, int s, int h, int c, int half) {
      const int tok0 = p.cu[s] + c * DR_C + 32 * hf;
      const int len = min(32, p.cu[s + 1] - tok0);
      if constexpr (SPLIT == 1) {
        uint32_t o[32];
        tmem_ld32(tO + 64 * b, o);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) ost[t * 32 + lane] = __float2bfloat16_rn(__uint_as_float(o[t]));
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // 64-byte pieces
          const int e = lane + i * 32, tr = e >> 2, ch = e & 3;
          if (tr < len)
            *reinterpret_cast<uint4*>(p.out + ((int64_t)(tok0 + tr) * H + h) * DR_D + q4 * 32 + ch * 8) =
                *reinterpret_cast<const uint4*>(ost + tr * 32 + ch * 8);
        }
      } else {
        uint32_t o[16];
        tmem_ld16x2_x16(tO + 64 * b, o);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 16; ++t) ost[(16 * sub + t) * 16 + (lane & 15)] = __float2bfloat16_rn(__uint_as_float(o[t]));
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 2; ++i) {  // 32-byte pieces
          const int e = lane + i * 32, tr = e >> 1, ch = e & 1;
          if (tr < len)
            *reinterpret_cast<uint4*>(p.out + ((int64_t)(tok0 + tr) * H + h) * DR_D + 64 * half + q4 * 16 + ch * 8) =
                *reinterpret_cast<const uint4*>(ost + tr * 16 + ch * 8);
        }
      }
      __syncwarp();
    };
    // final_state[s][h][dk][dv] = S^T[dv][dk]; dv = MR * half + r
    auto write_final = [&](int s, int h, int half) {
      if (!p.final_state) return;
      const int64_t sh = (int64_t)s * H + h;
#pragma unroll
      for (int cb = 0; cb < NCB; ++cb) {
        uint32_t v[32];
        s_ld(cb, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          p.final_state[(sh * DR_D + scol(cb) + i) * DR_D + MR * half + r] = __uint_as_float(v[i]);
      }
    };

    int ps = -1, ph = 0, pc = 0, phalf = 0;  // the previous chunk (its output is written one chunk late)
    for (int n = 0;; ++n) {
      const int st = n & 1;
      if (!warp_wait(bar0 + 8 * (B_FULL0 + st), (n >> 1) & 1, abort_flag)) break;
      const int s = meta[st].s, h = meta[st].h, c = meta[st].c, half = SPLIT == 1 ? 0 : meta[st].half;
      const float gam = meta[st].gamma;
      if (n > 0) {  // S^T of the previous chunk is complete
        if (!warp_wait(bar0 + 8 * B_SDONE, (n - 1) & 1, abort_flag)) break;
        tc_fence_after();
      }
      if (s < 0 || c == 0) {  // chain boundary
        if (ps >= 0) write_final(ps, ph, phalf);
        if (s < 0) {  // closing stage: output of the last chunk, then done
          if (ps >= 0 && warp_wait(bar0 + 8 * (B_ODONE0 + (st ^ 1)), ((n - 1) >> 1) & 1, abort_flag)) {
            tc_fence_after();
            o_epilogue(st ^ 1, ps, ph, pc, phalf);
          }
          break;
        }
        const int64_t sh = (int64_t)s * H + h;
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {  // S^T[r][dk] = initial_state[dk][MR * half + r]
          uint32_t v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i)
            v[i] = __float_as_uint(p.init_state ? p.init_state[(sh * DR_D + scol(cb) + i) * DR_D + MR * half + r] : 0.f);
          s_st(cb, v);
        }
        tmem_st_wait();
      }
      // S^T -> bf16 A tile; S^T *= gamma in TMEM (this chunk's MMAs read the A tile)
#pragma unroll
      for (int cb = 0; cb < NCB; ++cb) {
        uint32_t v[32];
        s_ld(cb, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(v[j * 8 + i]);
          *reinterpret_cast<uint4*>(sa + sw128_off(r, scol(cb) / 8 + j, MR)) = pack8(f);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * gam);
        s_st(cb, v);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar0 + 8 * B_SA);
      // v_new^T = U^T - vn -> bf16 A tile
      if (!warp_wait(bar0 + 8 * B_VN, n & 1, abort_flag)) break;
      tc_fence_after();
      {
        const uint8_t* ut = gbase + st * ST_BYTES + ST_UT;  // the chain's MR rows of U^T
        constexpr int NV = 32 / SPLIT;                     // vn columns per thread
        uint32_t v[32];
        if constexpr (SPLIT == 1) {
          tmem_ld32(tVN, v);
        } else {
          uint32_t w[16];
          tmem_ld16x2_x16(tVN, w);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = w[i];
        }
        tmem_ld_wait();
        const int c16_0 = (32 * hf + 16 * sub) / 8;
#pragma unroll
        for (int j = 0; j < NV / 8; ++j) {
          float u[8], f[8];
          unpack8(*reinterpret_cast<const uint4*>(ut + sw128_off(r, c16_0 + j, MR)), u);
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = u[i] - __uint_as_float(v[j * 8 + i]);
          *reinterpret_cast<uint4*>(va + sw128_off(r, c16_0 + j, MR)) = pack8(f);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar0 + 8 * B_VNEW);
      // output of the previous chunk (its o^T buffer is reused by the next chunk's MMAs)
      if (ps >= 0) {
        if (!warp_wait(bar0 + 8 * (B_ODONE0 + (st ^ 1)), ((n - 1) >> 1) & 1, abort_flag)) break;
        tc_fence_after();
        o_epilogue(st ^ 1, ps, ph, pc, phalf);
      }
      ps = s;
      ph = h;
      pc = c;
      phalf = half;
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
  if (tid == 0 && *abort_flag) atomicOr(&g_delta_error, 1);
}

template <int SPLIT>
__global__ void __launch_bounds__(THREADS, 1)
delta_recur_tc_kernel(const __grid_constant__ CUtensorMap mw, const __grid_constant__ CUtensorMap mqg,
                      const __grid_constant__ CUtensorMap mkg, const __grid_constant__ CUtensorMap ma,
                      const __grid_constant__ CUtensorMap mut, const RParams p) {
  recur_body<SPLIT, false>(mw, mqg, mkg, ma, mut, p);
}

// Final state of empty segments (their chains never enter the recurrence): the initial state, or 0.
__global__ void empty_state_kernel(const int32_t* __restrict__ table, int heads, const float* __restrict__ init,
                                   float* __restrict__ fin) {
  const int s = blockIdx.x, h = blockIdx.y;
  if (table[s + 1] > table[s]) return;
  const int64_t off = ((int64_t)s * heads + h) * DR_D * DR_D;
  for (int e = threadIdx.x * 4; e < DR_D * DR_D; e += blockDim.x * 4) {
    float4 v = init ? *reinterpret_cast<const float4*>(init + off + e) : make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(fin + off + e) = v;
  }
}

using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
    cudaGetLastError();
  }
  return fn;
}

// 3-D map over one operand of every workspace tile: [n_tiles][rows][cols] bf16, tile stride
// CH_BYTES, box 64 x box_rows x 1 (box_rows = rows unless given), 128-byte swizzle.
static int tile_map(CUtensorMap* m, const uint8_t* tiles, size_t off, int cols, int rows, int64_t n_tiles,
                    int box_rows = 0) {
  EncodeFn enc = encode_fn();
  if (!enc) return set_error(FDK_ERR_DEVICE, "chunk_gated_delta_rule: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)n_tiles};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)CH_BYTES};
  cuuint32_t box[3] = {64, (cuuint32_t)(box_rows ? box_rows : rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint8_t*>(tiles + off), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "chunk_gated_delta_rule: tensor map encode failed (%d)", (int)r);
  return FDK_OK;
}

// 2-D map over a [tokens, >= heads * 128] bf16 activation (row stride ld elements), box 64 x 64,
// 128-byte swizzle: one (chunk, head) tile is two boxes.
static int act_map(CUtensorMap* m, const void* ptr, int64_t tokens, int64_t heads, int64_t ld) {
  EncodeFn enc = encode_fn();
  if (!enc) return set_error(FDK_ERR_DEVICE, "chunk_gated_delta_rule: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)(heads * DR_D), (cuuint64_t)tokens};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "chunk_gated_delta_rule: tensor map encode failed (%d)", (int)r);
  return FDK_OK;
}

// 2-D map over the first `cols` columns of a [tokens, ld] bf16 projection, box 64 x 67 (one
// 64-token chunk plus 3 history rows), no swizzle: the fused prologue's raw conv input.
static int raw_map(CUtensorMap* m, const void* ptr, int64_t tokens, int64_t cols, int64_t ld) {
  EncodeFn enc = encode_fn();
  if (!enc) return set_error(FDK_ERR_DEVICE, "gdn_fused_delta_rule: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)tokens};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, 67};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gdn_fused_delta_rule: tensor map encode failed (%d)", (int)r);
  return FDK_OK;
}

}  // namespace drtc

// ------------------------------------------------------------------------------------ pipelined
// Prep and recurrence in ONE launch, for few chains (batch-1 decisions: 16 heads of one request).
// Two back-to-back launches leave the recurrence waiting for every tile although it needs chunk c
// only at its c-th step; here they overlap chunk by chunk.  Grid = one CTA per SM (the recurrence's
// shared memory allows one), so every CTA is resident: CTAs [0, rec_ctas) run the recurrence (two
// 64-row halves per (segment, head), as delta_recur_tc_kernel<2>); the others take prep tiles in
// chunk-major order from an atomic counter (tile t = chunk * heads + head) and, once a tile is in
// the workspace, set its ready flag (release).  The recurrence's producer acquires that flag (a
// bounded wait) before its TMA loads of the tile.  A tile is only ever waited on after some running
// CTA has claimed it or will claim it, so every wait has a producer making progress.
namespace dpipe {

template <bool CONV>
__global__ void __launch_bounds__(drtc::THREADS, 1)
gdn_pipe_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mw,
                const __grid_constant__ CUtensorMap mqg, const __grid_constant__ CUtensorMap mkg,
                const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mut,
                const __grid_constant__ CUtensorMap mw_st, const __grid_constant__ CUtensorMap mut_st,
                const dprep::PrepIn in, const int4* __restrict__ info, const int32_t* __restrict__ table, int nseg,
                int heads, float scale, uint8_t* __restrict__ tiles, const drtc::RParams rp, int rec_ctas,
                int32_t* __restrict__ ready, int32_t* __restrict__ prep_counter, int n_tiles) {
  if ((int)blockIdx.x < rec_ctas) {
    drtc::recur_body<2, true>(mw, mqg, mkg, ma, mut, rp);
    return;
  }
  using namespace dprep;
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sb = smem_raw + (base - raw);
  const uint32_t bar0 = base + BARS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sb + BARS + 8 * NBAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sb + BARS + 8 * NBAR + 4);
  volatile int* claim = reinterpret_cast<volatile int*>(sb + BARS + 8 * NBAR + 8);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(bar0 + 8 * i, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp < THREADS / 32) {  // the 256 prep threads; the other warps wait at the final barrier
    const int nchunks = table[nseg];
    for (uint32_t local = 0;; ++local) {
      if (tid == 0) *claim = atomicAdd(prep_counter, 1);
      prep_sync<true>();
      const int t = *claim;  // every thread reads it before the barrier that ends this iteration
      const int ci = t / heads, h = t - (t / heads) * heads;
      if (t >= n_tiles || ci >= nchunks) break;  // uniform
      bool ok = prep_tile<CONV, true>(mq, mk, mv, mw_st, mut_st, in, info, heads, scale, tiles, ci, h, base, sb, tmem,
                                      local & 1);
      // the tile's global stores before the flag that publishes them to TMA readers; this tile's
      // shared-memory writes and TMEM loads before the next tile's TMA writes and MMAs
      asm volatile("fence.proxy.async.global;\n" ::: "memory");
      fence_proxy_async_smem();
      tc_fence_before();
      ok = prep_sync_and<true>(ok);  // all of the tile's stores are done (and the claim slot was read)
      tc_fence_after();
      if (!ok) break;
      if (tid == 0) {
        __threadfence();
        asm volatile("st.release.gpu.global.b32 [%0], %1;\n" ::"l"(ready + t), "r"(1) : "memory");
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

}  // namespace dpipe

int delta_take_device_error() {
  int h = 0;
  if (cudaMemcpyFromSymbol(&h, g_delta_error, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (h) {
    int zero = 0;
    cudaMemcpyToSymbol(g_delta_error, &zero, sizeof(int));
  }
  return h;
}

static int launch_recur(int nseg, int heads, int64_t n_tiles, cudaStream_t s, const int32_t* cu, const int32_t* table,
                        int32_t* counter, const uint8_t* tiles, const float* init, bf16* out, float* fin) {
  using namespace drtc;
  if (fin) {
    empty_state_kernel<<<dim3((unsigned)nseg, (unsigned)heads), 256, 0, s>>>(table, heads, init, fin);
    if (int st = check_launch("chunk_gated_delta_rule/empty segments")) return st;
  }
  CUtensorMap mw, mqg, mkg, ma, mut;
  if (int st = tile_map(&mw, tiles, OFF_W, DR_C, DR_D, n_tiles)) return st;
  if (int st = tile_map(&mqg, tiles, OFF_QG, DR_D, DR_C, n_tiles)) return st;
  if (int st = tile_map(&mkg, tiles, OFF_KG, DR_D, DR_C, n_tiles)) return st;
  if (int st = tile_map(&ma, tiles, OFF_A, DR_C, DR_C, n_tiles)) return st;
  // Fewer (segment, head) chains than half the SMs (batch-1 decisions: 16): run each as two chains
  // of 64 dv rows on two CTAs; otherwise every SM already has a whole chain to run.
  const int64_t chains = (int64_t)nseg * heads;
  const bool split = 2 * chains <= sm_count();
  if (int st = tile_map(&mut, tiles, OFF_UT, DR_C, DR_D, n_tiles, split ? DR_D / 2 : DR_D)) return st;
  const RParams prm{cu, table, counter, nseg, heads, tiles, init, out, fin};
  const void* fn = split ? (const void*)delta_recur_tc_kernel<2> : (const void*)delta_recur_tc_kernel<1>;
  if (int st = ensure_smem_attr(fn, (int)SMEM_BYTES, "chunk_gated_delta_rule/recurrence")) return st;
  const int64_t items = chains * (split ? 2 : 1);
  const unsigned grid = (unsigned)(items < sm_count() ? items : sm_count());
  if (split)
    delta_recur_tc_kernel<2><<<grid, THREADS, SMEM_BYTES, s>>>(mw, mqg, mkg, ma, mut, prm);
  else
    delta_recur_tc_kernel<1><<<grid, THREADS, SMEM_BYTES, s>>>(mw, mqg, mkg, ma, mut, prm);
  return check_launch("chunk_gated_delta_rule/recurrence");
}

}  // namespace fdk

using namespace fdk;

extern "C" size_t fdk_chunk_gated_delta_rule_workspace_size(int64_t tokens, int64_t num_segments, int64_t heads,
                                                            int64_t dk, int64_t dv) {
  if (tokens < 0 || num_segments < 1 || heads < 1 || dk != DR_D || dv != DR_D) return 0;
  return ws_layout(tokens, num_segments, heads).total;
}

// Table, prep (plain or with the fused conv + gate prologue) and recurrence.  `q / k / v` are used
// by the plain prep only; the caller has validated everything.
static int run_pipelined(bool conv, const void* q, const void* k, int64_t ld_qk, const void* v, int64_t ld_v,
                         const dprep::PrepIn& in, const WsLayout& lay, const int32_t* cu, int nseg, int64_t tokens,
                         int64_t heads, float scale, const float* init, bf16* out, float* fin, uint8_t* ws,
                         cudaStream_t s) {
  int32_t* table = reinterpret_cast<int32_t*>(ws + lay.off_table);
  const int4* info = reinterpret_cast<const int4*>(ws + lay.off_info);
  uint8_t* tiles = ws + lay.off_tiles;
  int32_t* ready = reinterpret_cast<int32_t*>(ws + lay.off_ready);
  const int64_t n_tiles = lay.max_chunks * heads;
  if (fin) {
    drtc::empty_state_kernel<<<dim3((unsigned)nseg, (unsigned)heads), 256, 0, s>>>(table, (int)heads, init, fin);
    if (int st = check_launch("chunk_gated_delta_rule/empty segments")) return st;
  }
  CUtensorMap mq, mk, mv, mw, mqg, mkg, ma, mut;
  if (conv) {
    memset(&mk, 0, sizeof(mk));
    memset(&mv, 0, sizeof(mv));
    if (int st = drtc::raw_map(&mq, in.proj, tokens, 3 * (int64_t)in.key_dim, in.ld)) return st;
  } else {
    if (int st = drtc::act_map(&mq, q, tokens, heads, ld_qk)) return st;
    if (int st = drtc::act_map(&mk, k, tokens, heads, ld_qk)) return st;
    if (int st = drtc::act_map(&mv, v, tokens, heads, ld_v)) return st;
  }
  if (int st = drtc::tile_map(&mw, tiles, OFF_W, DR_C, DR_D, n_tiles)) return st;
  if (int st = drtc::tile_map(&mqg, tiles, OFF_QG, DR_D, DR_C, n_tiles)) return st;
  if (int st = drtc::tile_map(&mkg, tiles, OFF_KG, DR_D, DR_C, n_tiles)) return st;
  if (int st = drtc::tile_map(&ma, tiles, OFF_A, DR_C, DR_C, n_tiles)) return st;
  if (int st = drtc::tile_map(&mut, tiles, OFF_UT, DR_C, DR_D, n_tiles, DR_D / 2)) return st;
  CUtensorMap mut_st;  // the prep writes whole U^T tiles (the recurrence halves read 64 rows)
  if (int st = drtc::tile_map(&mut_st, tiles, OFF_UT, DR_C, DR_D, n_tiles)) return st;
  drtc::RParams rp{cu, table, table + nseg + 1, nseg, (int)heads, tiles, init, out, fin, ready};
  const void* fn = conv ? (const void*)dpipe::gdn_pipe_kernel<true> : (const void*)dpipe::gdn_pipe_kernel<false>;
  if (int st = ensure_smem_attr(fn, (int)drtc::SMEM_BYTES, "chunk_gated_delta_rule/pipelined")) return st;
  const int rec_ctas = (int)(2 * (int64_t)nseg * heads);
  const unsigned grid = (unsigned)sm_count();
  if (conv)
    dpipe::gdn_pipe_kernel<true><<<grid, drtc::THREADS, drtc::SMEM_BYTES, s>>>(
        mq, mk, mv, mw, mqg, mkg, ma, mut, mw, mut_st, in, info, table, nseg, (int)heads, scale, tiles, rp, rec_ctas,
        ready,
        table + nseg + 2, (int)n_tiles);
  else
    dpipe::gdn_pipe_kernel<false><<<grid, drtc::THREADS, drtc::SMEM_BYTES, s>>>(
        mq, mk, mv, mw, mqg, mkg, ma, mut, mw, mut_st, in, info, table, nseg, (int)heads, scale, tiles, rp, rec_ctas,
        ready,
        table + nseg + 2, (int)n_tiles);
  return check_launch("chunk_gated_delta_rule/pipelined");
}

static int run_delta_rule(bool conv, const void* q, const void* k, int64_t ld_qk, const void* v, int64_t ld_v,
                          const dprep::PrepIn& in, const int32_t* cu_seqlens, int64_t num_segments, int64_t tokens,
                          int64_t heads, float scale, const float* initial_state, void* out, float* final_state,
                          void* workspace, size_t workspace_bytes, cudaStream_t s) {
  const WsLayout lay = ws_layout(tokens, num_segments, heads);
  if (workspace_bytes < lay.total)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "chunk_gated_delta_rule: workspace %zu bytes < required %zu", workspace_bytes, lay.total);
  if (lay.max_chunks > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "chunk_gated_delta_rule: too many chunks");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* table = reinterpret_cast<int32_t*>(ws + lay.off_table);
  int4* info = reinterpret_cast<int4*>(ws + lay.off_info);
  uint8_t* tiles = ws + lay.off_tiles;
  const int nseg = (int)num_segments;
  int32_t* ready = reinterpret_cast<int32_t*>(ws + lay.off_ready);
  chunk_table_kernel<<<1, 256, 0, s>>>(cu_seqlens, nseg, tokens, lay.max_chunks, table, info, ready,
                                       lay.max_chunks * heads);
  if (int st = check_launch("chunk_gated_delta_rule/table")) return st;
  if (tokens == 0 && !final_state) return FDK_OK;
  // One request (batch-1 decisions) with few heads: prep and recurrence pipelined in one launch (at
  // most half the SMs run chains, at least as many make tiles).  Measured: config 4 (1536 tokens, 16
  // heads) 85 -> 76 us, one 8192-token request ~390 -> 264 us; with two or more requests the prep,
  // one tile at a time per SM here (each tile ~16 us of latency), becomes the bound and the two
  // launches are faster.
  const int64_t chains = num_segments * heads;
  if (tokens > 0 && num_segments == 1 && 4 * chains <= sm_count())
    return run_pipelined(conv, q, k, ld_qk, v, ld_v, in, lay, cu_seqlens, nseg, tokens, heads, scale, initial_state,
                         static_cast<bf16*>(out), final_state, ws, s);
  if (tokens > 0) {
    CUtensorMap mq, mk, mv;
    if (conv) {  // the fused prologue reads the projection through one map (passed as mq)
      memset(&mk, 0, sizeof(mk));
      memset(&mv, 0, sizeof(mv));
      if (int st = drtc::raw_map(&mq, in.proj, tokens, 3 * (int64_t)in.key_dim, in.ld)) return st;
    } else {
      if (int st = drtc::act_map(&mq, q, tokens, heads, ld_qk)) return st;
      if (int st = drtc::act_map(&mk, k, tokens, heads, ld_qk)) return st;
      if (int st = drtc::act_map(&mv, v, tokens, heads, ld_v)) return st;
    }
    if (int st = ensure_smem_attr(conv ? (const void*)dprep::delta_prep_kernel<true> : (const void*)dprep::delta_prep_kernel<false>,
                                  (int)dprep::SMEM_BYTES, "chunk_gated_delta_rule/prep"))
      return st;
    CUtensorMap mw_st, mut_st;  // the prep writes its U^T / W^T tiles through these
    if (int st = drtc::tile_map(&mw_st, tiles, OFF_W, DR_C, DR_D, lay.max_chunks * heads)) return st;
    if (int st = drtc::tile_map(&mut_st, tiles, OFF_UT, DR_C, DR_D, lay.max_chunks * heads)) return st;
    const dim3 grid((unsigned)lay.max_chunks, (unsigned)heads);
    if (conv)
      dprep::delta_prep_kernel<true><<<grid, dprep::THREADS, dprep::SMEM_BYTES, s>>>(mq, mk, mv, mw_st, mut_st, in, info, table, nseg,
                                                                                   (int)heads, scale, tiles);
    else
      dprep::delta_prep_kernel<false><<<grid, dprep::THREADS, dprep::SMEM_BYTES, s>>>(mq, mk, mv, mw_st, mut_st, in, info, table, nseg,
                                                                                    (int)heads, scale, tiles);
    if (int st = check_launch("chunk_gated_delta_rule/prep")) return st;
  }
  return launch_recur(nseg, (int)heads, lay.max_chunks * heads, s, cu_seqlens, table, table + nseg + 1, tiles,
                      initial_state, static_cast<bf16*>(out), final_state);
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
  dprep::PrepIn in{};
  in.g = g;
  in.beta = static_cast<const bf16*>(beta);
  return run_delta_rule(false, q, k, ld_qk, v, ld_v, in, cu_seqlens, num_segments, tokens, heads, scale, initial_state,
                        out, final_state, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int fdk_gdn_fused_delta_rule_fwd(const void* proj, int64_t ld_proj, const void* conv_weight, int kernel_width,
                                            int64_t key_dim, int64_t value_dim, int64_t a_col, int64_t b_col,
                                            const float* A_log, const float* dt_bias, const int32_t* cu_seqlens,
                                            int64_t num_segments, int64_t tokens, int64_t heads, float scale,
                                            const float* initial_state, void* out, float* final_state, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  if (int st = check_device()) return st;
  if (!proj || !conv_weight || !A_log || !dt_bias || !cu_seqlens || !out || !workspace)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gdn_fused_delta_rule: null pointer");
  if (kernel_width != 4) return set_error(FDK_ERR_UNSUPPORTED, "gdn_fused_delta_rule: kernel_width=%d (4 supported)", kernel_width);
  if (num_segments < 1 || tokens < 0 || heads < 1 || heads > 65535 || num_segments > 0x7fffffff)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gdn_fused_delta_rule: bad sizes");
  if (key_dim != heads * DR_D || value_dim != heads * DR_D)
    return set_error(FDK_ERR_UNSUPPORTED, "gdn_fused_delta_rule: key_dim and value_dim must be heads x 128");
  const int64_t C = 2 * key_dim + value_dim;
  if (a_col < C || b_col < C || a_col + heads > ld_proj || b_col + heads > ld_proj || ld_proj < C)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gdn_fused_delta_rule: a / b columns outside the projection row");
  if (!aligned16(proj) || ld_proj % 8 || !aligned16(conv_weight) || !aligned16(out) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(FDK_ERR_ALIGNMENT, "gdn_fused_delta_rule: 16-byte tensors and a 256-byte aligned workspace required");
  dprep::PrepIn in{};
  in.proj = static_cast<const bf16*>(proj);
  in.ld = ld_proj;
  in.conv_w = static_cast<const bf16*>(conv_weight);
  in.key_dim = (int)key_dim;
  in.a_col = (int)a_col;
  in.b_col = (int)b_col;
  in.A_log = A_log;
  in.dt_bias = dt_bias;
  in.tokens = tokens;
  return run_delta_rule(true, nullptr, nullptr, 0, nullptr, 0, in, cu_seqlens, num_segments, tokens, heads, scale,
                        initial_state, out, final_state, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
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
