// Native GQA causal attention for sm_100a: tcgen05 tensor cores, TMEM accumulators, TMA loads.
//
// One CTA computes a 128-query tile of TWO query heads that share one KV head (GQA pairs), so
// every K/V tile brought into shared memory feeds two heads.  Warp roles (320 threads):
//   warps 0-3  softmax of head A (thread = query row = TMEM lane)
//   warps 4-7  softmax of head B
//   warp  8    TMA producer: Q (once), K and V rings of 2 stages each
//   warp  9    TMEM allocator + single-thread tcgen05.mma issuer
// TMEM (512 columns): S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512), fp32.
// The issuer runs S_A = Q_A K_0^T and S_B = Q_B K_0^T, then per KV block j: O_A += P_A V_j once
// the head-A softmax has written P_A (bf16 pairs over the first 64 columns of S_A: the PV MMA
// takes A from TMEM), S_A = Q_A K_{j+1}^T, O_B += P_B V_j, S_B = Q_B K_{j+1}^T.  Head A's
// softmax of block j+1 thus overlaps head B's of block j, and the tensor core always has the
// other head's work queued; MMAs of one thread execute in issue order, so S_A(j+1) overwrites
// P_A(j) only after the PV that reads it.
// Softmax is online in fp32 in the exp2 domain with lazy rescaling of O (only when the running
// max grows by more than 2^8).  The causal mask is applied only on the diagonal block; rows of a
// tile past the end of its segment are computed but never stored.  Varlen: cu_seqlens gives
// each segment's token range; nothing attends across segments.
//
// Every mbarrier wait is bounded (clock64 budget): on timeout the CTA raises an abort flag, all
// roles leave their loops, in-flight MMAs and TMA loads are drained (bounded), TMEM is freed and
// a device-side error word is set (read with fdk_poll_device_error).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "common.cuh"
#include "sm100.cuh"

namespace fdk {
namespace attn {
using namespace sm100;

constexpr int BM = 128, BN = 128, HD = 128;
constexpr uint32_t HALF = 128 * 128;  // 128 rows x 128 B (64 bf16): one swizzle-128B box
constexpr uint32_t TILE = 2 * HALF;   // 128 x 128 bf16
constexpr uint32_t OFF_QA = 0, OFF_QB = TILE, OFF_K0 = 2 * TILE, OFF_K1 = 3 * TILE, OFF_V0 = 4 * TILE,
                   OFF_V1 = 5 * TILE, OFF_BAR = 6 * TILE;
enum { B_Q = 0, B_KF0, B_KF1, B_KE0, B_KE1, B_VF0, B_VF1, B_VE0, B_VE1, B_SA, B_SB, B_PA, B_PB, B_O, NBAR };
constexpr uint32_t SMEM_BYTES = OFF_BAR + 8 * NBAR + 16 + 1024;  // + slack for 1024-B alignment
constexpr int NUM_THREADS = 320;
constexpr uint32_t TM_SA = 0, TM_SB = 128, TM_OA = 256, TM_OB = 384, TM_COLS = 512;
// head_dim 128 runs one query head a CTA when (segments x head pairs x query tiles) is at most this.
// Measured (16 q / 4 kv heads): one 1536 segment 41.0 -> 29.3 us, one 2048 segment 49.1 -> 37.7 us;
// at one 4096 segment (256 pair-tiles) 82.9 vs 92.9 us and on packed config-5 batches the two-head
// kernel is faster.
constexpr int64_t ONE_HEAD_MAX_PAIR_TILES = 148;
constexpr long long DRAIN_BUDGET = 2000000000LL;

__device__ int g_device_error = 0;

struct Params {
  const int32_t* cu;
  int64_t tokens;  // rows of q / out: stores past them are skipped (cu_seqlens is not checked on the host)
  int hq, hkv;
  float sl2;  // softmax scale * log2(e)
  bf16* out;
  const bf16* gate;
  int64_t ld_gate;
  int gate_hstride;
};

__device__ __forceinline__ bool drain(uint32_t bar, uint32_t parity) {
  volatile int never = 0;
  return mbar_wait(bar, parity, &never, DRAIN_BUDGET);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
gqa_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + OFF_BAR;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * NBAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + 8 * NBAR + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // grid: x = (segment, head pair) with the pair fastest, y = query tile from the last one down.
  // Blocks are dispatched x-fastest, so every segment's longest (causal: most KV blocks) tiles go
  // first across all heads -- longest-processing-time order over the whole grid.
  const int npairs = p.hq / 2;
  const int seg = (int)blockIdx.x / npairs, pair = (int)blockIdx.x - seg * npairs;
  const int seg0 = p.cu[seg];
  const int L = p.cu[seg + 1] - seg0;
  const int mblk = (int)gridDim.y - 1 - (int)blockIdx.y;
  const int m0 = mblk * BM;
  if (m0 >= L) return;  // uniform early exit: this tile lies past the segment
  const int ha = pair * 2, hb = ha + 1;
  const int hk = ha / (p.hq / p.hkv);
  const int n_kv = mblk + 1;

  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(bar0 + 8 * i, (i == B_PA || i == B_PB) ? 128u : 1u);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      mbar_expect_tx(bar0 + 8 * B_Q, 2 * TILE);
      tma_load_2d(base + OFF_QA, &tq, bar0 + 8 * B_Q, ha * HD, seg0 + m0);
      tma_load_2d(base + OFF_QA + HALF, &tq, bar0 + 8 * B_Q, ha * HD + 64, seg0 + m0);
      tma_load_2d(base + OFF_QB, &tq, bar0 + 8 * B_Q, hb * HD, seg0 + m0);
      tma_load_2d(base + OFF_QB + HALF, &tq, bar0 + 8 * B_Q, hb * HD + 64, seg0 + m0);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int ks = j & 1;
        if (j >= 2 && !mbar_wait(bar0 + 8 * (B_KE0 + ks), ((j >> 1) - 1) & 1, abort_flag)) break;
        const uint32_t kdst = base + (ks ? OFF_K1 : OFF_K0);
        mbar_expect_tx(bar0 + 8 * (B_KF0 + ks), TILE);
        tma_load_2d(kdst, &tk, bar0 + 8 * (B_KF0 + ks), hk * HD, seg0 + j * BN);
        tma_load_2d(kdst + HALF, &tk, bar0 + 8 * (B_KF0 + ks), hk * HD + 64, seg0 + j * BN);
        issued_k = j + 1;
        if (j >= 2 && !mbar_wait(bar0 + 8 * (B_VE0 + ks), ((j >> 1) - 1) & 1, abort_flag)) break;
        const uint32_t vdst = base + (ks ? OFF_V1 : OFF_V0);
        mbar_expect_tx(bar0 + 8 * (B_VF0 + ks), TILE);
        tma_load_2d(vdst, &tv, bar0 + 8 * (B_VF0 + ks), hk * HD, seg0 + j * BN);
        tma_load_2d(vdst + HALF, &tv, bar0 + 8 * (B_VF0 + ks), hk * HD + 64, seg0 + j * BN);
        issued_v = j + 1;
      }
      // drain: every issued load must have landed before shared memory is released
      drain(bar0 + 8 * B_Q, 0);
      for (int j = (issued_k > 2 ? issued_k - 2 : 0); j < issued_k; ++j) drain(bar0 + 8 * (B_KF0 + (j & 1)), (j >> 1) & 1);
      for (int j = (issued_v > 2 ? issued_v - 2 : 0); j < issued_v; ++j) drain(bar0 + 8 * (B_VF0 + (j & 1)), (j >> 1) & 1);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_QK = idesc_bf16(128, 128, false, false);
      constexpr uint32_t ID_PV = idesc_bf16(128, 128, false, true);  // V is MN-major (D contiguous)
      // Issue order per KV block j: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1).  Softmax A starts on
      // block j+1 while softmax B is still on block j, so the two row groups overlap each other
      // and the tensor pipe instead of taking turns.  Each S commit also covers the PV of the
      // same head issued before it (O rescale and P-tile reuse rely on that).
      // descriptors built once; a k step adds its byte offset / 16 to the start-address field
      // (shared-memory addresses stay below 2^18, so the field never carries)

      auto issue_s = [&](int j, uint32_t q_off, uint32_t tm, uint32_t bar) {
        const uint64_t dq = sdesc_sw128(base + q_off, 16, 1024);
        const uint64_t dk = sdesc_sw128(base + ((j & 1) ? OFF_K1 : OFF_K0), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = ((kk >> 2) * HALF + (kk & 3) * 32) >> 4;
          umma_ss(tmem + tm, dq + off, dk + off, ID_QK, kk > 0);
        }
        umma_commit(bar);
      };
      // O += P V with P (bf16, packed two per column) in the first 64 TMEM columns of the head's S
      // region: the softmax overwrote S with P; the next S MMA of the head is issued after this one
      auto issue_pv = [&](int j, uint32_t tm_p, uint32_t tm) {
        const uint64_t dV = sdesc_sw128(base + ((j & 1) ? OFF_V1 : OFF_V0), HALF, 1024);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + tm, tmem + tm_p + 8 * kk, dV + (uint32_t)(kk * 2048 >> 4), ID_PV, (j > 0 || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(bar0 + 8 * B_Q, 0, abort_flag) && mbar_wait(bar0 + 8 * B_KF0, 0, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_s(0, OFF_QA, TM_SA, bar0 + 8 * B_SA);
        issue_s(0, OFF_QB, TM_SB, bar0 + 8 * B_SB);
        umma_commit(bar0 + 8 * B_KE0);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const bool more = j + 1 < n_kv;
        if (!mbar_wait(bar0 + 8 * (B_VF0 + (j & 1)), (j >> 1) & 1, abort_flag)) break;
        if (!mbar_wait(bar0 + 8 * B_PA, j & 1, abort_flag)) break;
        tc_fence_after();
        issue_pv(j, TM_SA, TM_OA);
        if (more) {
          if (!mbar_wait(bar0 + 8 * (B_KF0 + ((j + 1) & 1)), ((j + 1) >> 1) & 1, abort_flag)) break;
          tc_fence_after();
          issue_s(j + 1, OFF_QA, TM_SA, bar0 + 8 * B_SA);
        }
        if (!mbar_wait(bar0 + 8 * B_PB, j & 1, abort_flag)) break;
        tc_fence_after();
        issue_pv(j, TM_SB, TM_OB);
        umma_commit(bar0 + 8 * (B_VE0 + (j & 1)));
        if (more) {
          issue_s(j + 1, OFF_QB, TM_SB, bar0 + 8 * B_SB);
          umma_commit(bar0 + 8 * (B_KE0 + ((j + 1) & 1)));
        }
      }
      umma_commit(bar0 + 8 * B_O);  // arrives when every MMA above has completed
      drain(bar0 + 8 * B_O, 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax (2 warpgroups)
    const int wg = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + (wg ? TM_SB : TM_SA);
    const uint32_t tO = tmem + lane_base + (wg ? TM_OB : TM_OA);
    const uint32_t bS = bar0 + 8 * (wg ? B_SB : B_SA);
    const uint32_t bP = bar0 + 8 * (wg ? B_PB : B_PA);
    const float sl2 = p.sl2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      // warp-uniform: the tcgen05.ld below is warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(bS, j & 1, abort_flag) ? 1 : 0)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, sr[c]);
      tmem_ld_wait();
      if (j == n_kv - 1) {  // diagonal block: causal mask (the only block that needs one)
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i > row) sr[c][i] = __float_as_uint(-INFINITY);
      }
      // row max with 8 independent accumulators (a 128-long fmax chain would serialise the warp)
      float mx8[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mx8[a] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(sr[c][i]));
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float m_new = fmaxf(m_run, mx * sl2);
      float alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_run = m_new;
      } else if (m_new > m_run + 8.0f) {
        alpha = ex2(m_run - m_new);
        m_run = m_new;
        rescale = true;
      }
      // P = exp2(S * scale * log2e - m_run) as bf16 pairs over the first 64 columns of this row's
      // S (the PV MMA reads A from TMEM); the row sum in 8 independent partial sums
      float sum8[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) sum8[a] = 0.f;
      uint32_t pk[2][32];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float e0 = ex2(fmaf(__uint_as_float(sr[(2 * c) >> 5][(2 * c) & 31]), sl2, -m_run));
        const float e1 = ex2(fmaf(__uint_as_float(sr[(2 * c + 1) >> 5][(2 * c + 1) & 31]), sl2, -m_run));
        sum8[(2 * c) & 7] += e0;
        sum8[(2 * c + 1) & 7] += e1;
        pk[c >> 5][c & 31] = pack_bf16x2(e0, e1);
      }
      tmem_st32(tS, pk[0]);
      tmem_st32(tS + 32, pk[1]);
      const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      l_run = l_run * alpha + sum;
      if (rescale) {  // O row *= alpha (PV of block j-1 has completed: S_j's commit covers it)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bP);
    }
    // ------------------------------------------------------------------ epilogue
    // Warp-uniform condition: every thread of the warp saw the same waits succeed or fail.
    if (ok && __all_sync(0xffffffffu, mbar_wait(bar0 + 8 * B_O, 0, abort_flag) ? 1 : 0)) {
      tc_fence_after();
      const int qpos = m0 + row;
      const bool valid = qpos < L && (int64_t)seg0 + qpos < p.tokens;
      const int h = wg ? hb : ha;
      const float inv_l = 1.0f / l_run;
      const int64_t tok = (int64_t)seg0 + qpos;
      bf16* orow = p.out + (tok * p.hq + h) * HD;
      const bf16* grow = p.gate ? p.gate + tok * p.ld_gate + (int64_t)h * p.gate_hstride : nullptr;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            float y[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = __uint_as_float(o[v8 * 8 + i]) * inv_l;
            if (grow) {
              float gv[8];
              unpack8(*reinterpret_cast<const uint4*>(grow + c * 32 + v8 * 8), gv);
#pragma unroll
              for (int i = 0; i < 8; ++i) y[i] *= sigmoidf_(gv[i]);
            }
            *reinterpret_cast<uint4*>(orow + c * 32 + v8 * 8) = pack8(y);
          }
        }
      }
    }
  }
  // ------------------------------------------------------------------ teardown
  __syncwarp();  // lane 0 of the producer / MMA warps rejoins its warp before the aligned barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
  if (tid == 0 && *abort_flag) atomicExch(&g_device_error, 1);
}

// ---------------------------------------------------------------------------------------------
// One query head a CTA.  Used for head_dim 256 (the reference op's own shape:
// native_gqa_kernel.py:132-133 accepts only D = 256, run with 8 query / 2 KV heads), where S and O
// of two heads would not fit 512 TMEM columns, with 64-key KV blocks: Q 64 KB, K and V two stages of
// 32 KB each -- 192 KB of shared memory; and for head_dim 128 when the two-head kernel's grid would
// leave SMs idle (short segments), with 128-key blocks: 160 KB.  TMEM: S ping-pong [0, BN) and
// [BN, 2 BN), O [256, 256 + D).  Warps 0-3 softmax (thread = query row = TMEM lane), warp 4 TMA
// producer, warp 5 TMEM allocator + MMA issuer.  The issuer keeps one S block ahead of the softmax:
//     S(0), S(1); then per block j: [P(j) ready] O += P(j) V(j); S(j+2) into P(j)'s buffer
// (MMAs of one thread run in issue order, so S(j+2) overwrites P(j) only after the PV reading it),
// so the tensor core runs PV(j) and S(j+2) while the softmax works on S(j+1).  A lazy O rescale at
// block j waits for PV(j-1) on its own barrier: S(j)'s commit covers PV(j-2), and PV(j) needs P(j),
// so that barrier has completed j-1 or j times.
namespace onehead {
// Geometry of one instantiation: head_dim HD_ (128 or 256) and BN_ keys a KV block (128 or 64).
// Shared memory: Q [HD/64 boxes][128 rows][128 B], K and V two stages of [HD/64][BN][128 B] each.
// TMEM: S ping-pong [0, BN) and [BN, 2 BN), O [256, 256 + HD).
template <int HD_, int BN_>
struct Geo {
  static constexpr int BM = 128, BN = BN_, HD = HD_, NBX = HD_ / 64;
  static constexpr uint32_t QBOX = 128 * 128, KBOX = (uint32_t)BN_ * 128;
  static constexpr uint32_t QT = NBX * QBOX, KT = NBX * KBOX;
  static constexpr uint32_t OFF_Q = 0, OFF_K0 = QT, OFF_K1 = QT + KT, OFF_V0 = QT + 2 * KT, OFF_V1 = QT + 3 * KT,
                            OFF_BAR = QT + 4 * KT;
};
enum { B_Q = 0, B_KF0, B_KF1, B_KE0, B_KE1, B_VF0, B_VF1, B_VE0, B_VE1, B_S0, B_S1, B_P0, B_P1, B_PV, B_O, NBAR };
template <int HD_, int BN_>
constexpr uint32_t smem_bytes() { return Geo<HD_, BN_>::OFF_BAR + 8 * NBAR + 16 + 1024; }
constexpr int NUM_THREADS = 192;
constexpr uint32_t TM_S = 0, TM_O = 256, TM_COLS = 512;

template <int HD_, int BN_>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gqa_fwd_1head_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, const Params p) {
  using G = Geo<HD_, BN_>;
  constexpr int BM = G::BM, BN = G::BN, HD = G::HD, NBX = G::NBX;
  constexpr uint32_t QBOX = G::QBOX, KBOX = G::KBOX, QT = G::QT, KT = G::KT;
  constexpr uint32_t OFF_Q = G::OFF_Q, OFF_K0 = G::OFF_K0, OFF_K1 = G::OFF_K1, OFF_V0 = G::OFF_V0,
                     OFF_V1 = G::OFF_V1, OFF_BAR = G::OFF_BAR;
  static_assert(2 * BN <= (int)TM_O && (int)TM_O + HD <= (int)TM_COLS, "TMEM layout");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + OFF_BAR;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * NBAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + 8 * NBAR + 4);
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // grid: x = (segment, query head) with the head fastest, y = query tile from the last one down
  const int seg = (int)blockIdx.x / p.hq, h = (int)blockIdx.x - seg * p.hq;
  const int seg0 = p.cu[seg];
  const int L = p.cu[seg + 1] - seg0;
  const int mblk = (int)gridDim.y - 1 - (int)blockIdx.y;
  const int m0 = mblk * BM;
  if (m0 >= L) return;  // uniform early exit: this tile lies past the segment
  const int hk = h / (p.hq / p.hkv);
  const int n_kv = (min(m0 + BM, L) + BN - 1) / BN;  // keys up to the tile's last valid query

  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(bar(i), (i == B_P0 || i == B_P1) ? 128u : 1u);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      mbar_expect_tx(bar(B_Q), QT);
#pragma unroll
      for (int b = 0; b < NBX; ++b) tma_load_2d(base + OFF_Q + b * QBOX, &tq, bar(B_Q), h * HD + 64 * b, seg0 + m0);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int ks = j & 1;
        if (j >= 2 && !mbar_wait(bar(B_KE0 + ks), ((j >> 1) - 1) & 1, abort_flag)) break;
        const uint32_t kdst = base + (ks ? OFF_K1 : OFF_K0);
        mbar_expect_tx(bar(B_KF0 + ks), KT);
#pragma unroll
        for (int b = 0; b < NBX; ++b) tma_load_2d(kdst + b * KBOX, &tk, bar(B_KF0 + ks), hk * HD + 64 * b, seg0 + j * BN);
        issued_k = j + 1;
        if (j >= 2 && !mbar_wait(bar(B_VE0 + ks), ((j >> 1) - 1) & 1, abort_flag)) break;
        const uint32_t vdst = base + (ks ? OFF_V1 : OFF_V0);
        mbar_expect_tx(bar(B_VF0 + ks), KT);
#pragma unroll
        for (int b = 0; b < NBX; ++b) tma_load_2d(vdst + b * KBOX, &tv, bar(B_VF0 + ks), hk * HD + 64 * b, seg0 + j * BN);
        issued_v = j + 1;
      }
      // drain: every issued load must have landed before shared memory is released
      drain(bar(B_Q), 0);
      for (int j = (issued_k > 2 ? issued_k - 2 : 0); j < issued_k; ++j) drain(bar(B_KF0 + (j & 1)), (j >> 1) & 1);
      for (int j = (issued_v > 2 ? issued_v - 2 : 0); j < issued_v; ++j) drain(bar(B_VF0 + (j & 1)), (j >> 1) & 1);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_QK = idesc_bf16(128, BN, false, false);
      constexpr uint32_t ID_PV = idesc_bf16(128, HD, false, true);  // V is MN-major (d contiguous)
      const uint64_t dq = sdesc_sw128(base + OFF_Q, 16, 1024);
      // S(j) = Q K_j^T into S buffer j & 1: K = D in D / 16 steps of 16 (4 per swizzle box)
      auto issue_s = [&](int j) {
        const uint64_t dk = sdesc_sw128(base + ((j & 1) ? OFF_K1 : OFF_K0), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t qoff = ((kk >> 2) * QBOX + (kk & 3) * 32) >> 4;
          const uint32_t koff = ((kk >> 2) * KBOX + (kk & 3) * 32) >> 4;
          umma_ss(tmem + TM_S + (uint32_t)BN * (uint32_t)(j & 1), dq + qoff, dk + koff, ID_QK, kk > 0);
        }
        umma_commit(bar(B_S0 + (j & 1)));
        umma_commit(bar(B_KE0 + (j & 1)));
      };
      // O += P(j) V(j): P as bf16 pairs in the first BN / 2 columns of S buffer j & 1; V's 64-wide d
      // groups are KBOX apart (lbo), its 8-key atoms 1024 B apart (sbo); K = BN keys in steps of 16
      auto issue_pv = [&](int j) {
        const uint64_t dv = sdesc_sw128(base + ((j & 1) ? OFF_V1 : OFF_V0), KBOX, 1024);
        const uint32_t tp = tmem + TM_S + (uint32_t)BN * (uint32_t)(j & 1);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_ts(tmem + TM_O, tp + 8 * kk, dv + (uint32_t)(kk * 2048 >> 4), ID_PV, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bar(B_PV));
        umma_commit(bar(B_VE0 + (j & 1)));
      };
      bool ok = mbar_wait(bar(B_Q), 0, abort_flag) && mbar_wait(bar(B_KF0), 0, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        if (n_kv > 1) {
          ok = mbar_wait(bar(B_KF1), 0, abort_flag);
          if (ok) {
            tc_fence_after();
            issue_s(1);
          }
        }
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (!mbar_wait(bar(B_VF0 + (j & 1)), (j >> 1) & 1, abort_flag)) break;
        if (!mbar_wait(bar(B_P0 + (j & 1)), (j >> 1) & 1, abort_flag)) break;
        tc_fence_after();
        issue_pv(j);
        if (j + 2 < n_kv) {
          if (!mbar_wait(bar(B_KF0 + (j & 1)), ((j + 2) >> 1) & 1, abort_flag)) break;
          tc_fence_after();
          issue_s(j + 2);
        }
      }
      umma_commit(bar(B_O));  // arrives when every MMA above has completed
      drain(bar(B_O), 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax (warps 0-3)
    const int row = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t tO = tmem + lane_base + TM_O;
    const float sl2 = p.sl2;
    const int qpos = m0 + row;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const uint32_t tS = tmem + lane_base + TM_S + (uint32_t)BN * (uint32_t)(j & 1);
      if (!__all_sync(0xffffffffu, mbar_wait(bar(B_S0 + (j & 1)), (j >> 1) & 1, abort_flag) ? 1 : 0)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[BN / 32][32];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + c * 32, sr[c]);
      tmem_ld_wait();
      const int lim = qpos - j * BN;  // key column c is visible when c <= lim
      if (lim < BN - 1) {             // a block that crosses the diagonal: causal mask
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i > lim) sr[c][i] = __float_as_uint(-INFINITY);
      }
      float mx8[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mx8[a] = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(sr[c][i]));
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float m_new = fmaxf(m_run, mx * sl2);
      float alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_run = m_new;
      } else if (m_new > m_run + 8.0f) {
        alpha = ex2(m_run - m_new);
        m_run = m_new;
        rescale = true;
      }
      float sum8[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) sum8[a] = 0.f;
      uint32_t pk[BN / 64][32];
#pragma unroll
      for (int c = 0; c < BN / 2; ++c) {
        const float e0 = ex2(fmaf(__uint_as_float(sr[(2 * c) >> 5][(2 * c) & 31]), sl2, -m_run));
        const float e1 = ex2(fmaf(__uint_as_float(sr[(2 * c + 1) >> 5][(2 * c + 1) & 31]), sl2, -m_run));
        sum8[(2 * c) & 7] += e0;
        sum8[(2 * c + 1) & 7] += e1;
        pk[c >> 5][c & 31] = pack_bf16x2(e0, e1);
      }
#pragma unroll
      for (int c = 0; c < BN / 64; ++c) tmem_st32(tS + c * 32, pk[c]);
      const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      l_run = l_run * alpha + sum;
      // O row *= alpha once PV(j-1) has completed (warp-uniform: the TMEM accesses are collective)
      if (__any_sync(0xffffffffu, rescale)) {
        if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PV), (j - 1) & 1, abort_flag) ? 1 : 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(B_P0 + (j & 1)));
    }
    // ------------------------------------------------------------------ epilogue
    if (ok && __all_sync(0xffffffffu, mbar_wait(bar(B_O), 0, abort_flag) ? 1 : 0)) {
      tc_fence_after();
      const bool valid = qpos < L && (int64_t)seg0 + qpos < p.tokens;
      const float inv_l = 1.0f / l_run;
      const int64_t tok = (int64_t)seg0 + qpos;
      bf16* orow = p.out + (tok * p.hq + h) * HD;
      const bf16* grow = p.gate ? p.gate + tok * p.ld_gate + (int64_t)h * p.gate_hstride : nullptr;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            float y[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = __uint_as_float(o[v8 * 8 + i]) * inv_l;
            if (grow) {
              float gv[8];
              unpack8(*reinterpret_cast<const uint4*>(grow + c * 32 + v8 * 8), gv);
#pragma unroll
              for (int i = 0; i < 8; ++i) y[i] *= sigmoidf_(gv[i]);
            }
            *reinterpret_cast<uint4*>(orow + c * 32 + v8 * 8) = pack8(y);
          }
        }
      }
    }
  }
  // ------------------------------------------------------------------ teardown
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
  if (tid == 0 && *abort_flag) atomicExch(&g_device_error, 1);
}
}  // namespace onehead

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

// 2-D map over [rows, cols] bf16 (row stride ld elements), box 64 x box_rows, 128-byte swizzle.
static int make_map(CUtensorMap* m, const void* ptr, int64_t cols, int64_t rows, int64_t ld, int box_rows = 128) {
  EncodeFn enc = encode_fn();
  if (!enc) return set_error(FDK_ERR_DEVICE, "gqa_fwd: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FDK_ERR_INVALID_ARGUMENT, "gqa_fwd: tensor map encode failed (%d)", (int)r);
  return FDK_OK;
}

}  // namespace attn
}  // namespace fdk

using namespace fdk;

extern "C" int fdk_gqa_fwd(const void* q, int64_t ld_q, const void* k, int64_t ld_k, const void* v, int64_t ld_v,
                           const int32_t* cu_seqlens, int64_t num_segments, int64_t max_seqlen, int64_t tokens,
                           int64_t hq, int64_t hkv, int64_t head_dim, float scale, const void* gate, int64_t ld_gate,
                           int gate_interleaved, void* out, void* stream) {
  using namespace fdk::attn;
  if (int st = check_device()) return st;
  if (!q || !k || !v || !cu_seqlens || !out) return set_error(FDK_ERR_INVALID_ARGUMENT, "gqa_fwd: null pointer");
  if (head_dim != 128 && head_dim != 256)
    return set_error(FDK_ERR_UNSUPPORTED, "gqa_fwd: head_dim=%lld (128 and 256 supported)", (long long)head_dim);
  const int64_t HD = head_dim;
  if (hq <= 0 || hkv <= 0 || hq % hkv) return set_error(FDK_ERR_INVALID_ARGUMENT, "gqa_fwd: hq must be a multiple of hkv");
  if (HD == 128 && (hq / hkv) % 2)
    return set_error(FDK_ERR_UNSUPPORTED, "gqa_fwd: with head_dim 128 the query heads per KV head must be even");
  if (num_segments < 1 || num_segments > 65535 || tokens < 0 || max_seqlen < 0)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gqa_fwd: bad segment count or sizes");
  if (ld_q < hq * HD || ld_k < hkv * HD || ld_v < hkv * HD || (gate && ld_gate < hq * HD))
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gqa_fwd: row stride too small");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || ld_q % 8 || ld_k % 8 || ld_v % 8 ||
      (gate && (!aligned16(gate) || ld_gate % 8)))
    return set_error(FDK_ERR_ALIGNMENT, "gqa_fwd: pointers and strides must be 16-byte aligned");
  if (tokens == 0 || max_seqlen == 0) return FDK_OK;
  // head_dim 128: two query heads a CTA, unless that grid would leave SMs idle (short segments, e.g.
  // one 1536-token request: 96 CTAs for 148 SMs) -- then one head a CTA, twice the CTAs
  const int64_t mtiles = (max_seqlen + BM - 1) / BM;
  const bool one_head = HD == 256 || num_segments * (hq / 2) * mtiles <= (int64_t)ONE_HEAD_MAX_PAIR_TILES;
  const int kv_rows = HD == 256 ? 64 : 128;
  CUtensorMap mq, mk, mv;
  if (int st = make_map(&mq, q, hq * HD, tokens, ld_q)) return st;
  if (int st = make_map(&mk, k, hkv * HD, tokens, ld_k, kv_rows)) return st;
  if (int st = make_map(&mv, v, hkv * HD, tokens, ld_v, kv_rows)) return st;
  Params prm;
  prm.cu = cu_seqlens;
  prm.tokens = tokens;
  prm.hq = (int)hq;
  prm.hkv = (int)hkv;
  prm.sl2 = scale * 1.4426950408889634f;
  prm.out = static_cast<bf16*>(out);
  prm.gate = static_cast<const bf16*>(gate);
  prm.ld_gate = ld_gate;
  prm.gate_hstride = (int)(gate_interleaved ? 2 * HD : HD);
  if (one_head) {
    if (mtiles > 65535 || num_segments * hq > 0x7fffffff)
      return set_error(FDK_ERR_UNSUPPORTED, "gqa_fwd: too many query tiles or segments");
    dim3 grid((unsigned)(num_segments * hq), (unsigned)mtiles);
    cudaStream_t st_ = static_cast<cudaStream_t>(stream);
    if (HD == 256) {
      constexpr uint32_t sm = onehead::smem_bytes<256, 64>();
      if (int st = ensure_smem_attr((const void*)onehead::gqa_fwd_1head_kernel<256, 64>, (int)sm, "gqa_fwd")) return st;
      onehead::gqa_fwd_1head_kernel<256, 64><<<grid, onehead::NUM_THREADS, sm, st_>>>(mq, mk, mv, prm);
    } else {
      constexpr uint32_t sm = onehead::smem_bytes<128, 128>();
      if (int st = ensure_smem_attr((const void*)onehead::gqa_fwd_1head_kernel<128, 128>, (int)sm, "gqa_fwd")) return st;
      onehead::gqa_fwd_1head_kernel<128, 128><<<grid, onehead::NUM_THREADS, sm, st_>>>(mq, mk, mv, prm);
    }
    return check_launch("gqa_fwd (one head a CTA)");
  }
  if (int st = ensure_smem_attr((const void*)gqa_fwd_kernel, (int)SMEM_BYTES, "gqa_fwd")) return st;
  if (mtiles > 65535 || num_segments * (hq / 2) > 0x7fffffff)
    return set_error(FDK_ERR_UNSUPPORTED, "gqa_fwd: too many query tiles or segments");
  dim3 grid((unsigned)(num_segments * (hq / 2)), (unsigned)mtiles);
  gqa_fwd_kernel<<<grid, NUM_THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(mq, mk, mv, prm);
  return check_launch("gqa_fwd");
}

namespace fdk {
namespace attn {
// One warp waits on an mbarrier that nothing arrives on, through the same bounded wait every
// kernel here uses; the wait runs out after `budget` SM cycles and bit 2 of the error word is set.
__global__ void bounded_wait_probe_kernel(long long budget) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const bool ok = mbar_wait(smem_u32(&bar), 0, &abort_flag, budget);
  if (__all_sync(0xffffffffu, ok ? 1 : 0) == 0 && threadIdx.x == 0) atomicOr(&g_device_error, 4);
}
}  // namespace attn
}  // namespace fdk

extern "C" int fdk_selftest_bounded_wait(int64_t budget_cycles, void* stream) {
  if (budget_cycles <= 0 || budget_cycles > 4000000000LL)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "selftest_bounded_wait: budget_cycles must be in (0, 4e9]");
  fdk::attn::bounded_wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>((long long)budget_cycles);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FDK_ERR_LAUNCH, cudaGetErrorString(e));
  return FDK_OK;
}

extern "C" int fdk_poll_device_error(int* code) {
  int h = 0;
  if (cudaMemcpyFromSymbol(&h, fdk::attn::g_device_error, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return set_error(FDK_ERR_DEVICE, "poll_device_error: cannot read the device error word");
  }
  if (h) {
    int zero = 0;
    cudaMemcpyToSymbol(fdk::attn::g_device_error, &zero, sizeof(int));
  }
  const int d = fdk::delta_take_device_error();
  if (d < 0) return set_error(FDK_ERR_DEVICE, "poll_device_error: cannot read the device error word");
  h |= ((d & 1) << 1) | ((d & 2) << 2);  // 2: a delta-rule wait ran out; 8: cu_seqlens rejected
  const int gm = fdk::gemm_take_device_error();
  if (gm < 0) return set_error(FDK_ERR_DEVICE, "poll_device_error: cannot read the device error word");
  if (gm) h |= 16;  // a GEMM wait ran out
  if (code) *code = h;
  return FDK_OK;
}
