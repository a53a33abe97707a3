// Projection / MLP GEMMs for sm_100a: C = A B^T (bf16 in, fp32 accumulate) on tcgen05 with TMEM
// accumulators fed by TMA, with the epilogue the decision forward needs fused in.
//
// Persistent kernel, one CTA per SM, tiles of 128 x 256 outputs (M = 128, N = 256 MMAs) visited in
// bands of 8 N-tiles, n fastest (consecutive tiles share an A row block).  Warp roles (192 threads):
//   warp 0     TMA producer: A [128 rows][64 k] and B [256 rows][64 k] per k-step into a ring of
//              STAGES stages (128-byte swizzle; 48 KB a stage)
//   warp 1     TMEM allocator (512 columns: two 256-column accumulators) + single-thread MMA issuer
//   warps 2-5  epilogue: thread = output row = TMEM lane; drains accumulator b while the MMAs of the
//              next tile run into the other one, writing through shared memory with TMA stores
// Epilogues:
//   PLAIN   C[m][n] = bf16(acc)
//   SWIGLU  B's rows are the gate / up projections interleaved in blocks of 128 rows (block j:
//           gate rows [128 j, +128) then up rows [128 j, +128)), so one tile holds 128 gate and the
//           matching 128 up columns: C[m][128 j + c] = bf16(silu(g) * u) from the fp32 accumulators
//           ([tf]:706-708 -- the [T, 2 I] projection is never written to HBM)
// Every mbarrier wait is bounded (see sm100.cuh); a wait that runs out sets this file's device error
// word (bit 16 of fdk_poll_device_error's code), the CTA drains its copies and MMAs and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "sm100.cuh"

namespace fdk {
namespace gemm {
using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, ST_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t OUT_BOX = 32 * 128;                     // [32 rows][64 bf16] output block, 128-byte swizzle
constexpr uint32_t OFF_OUT = STAGES * ST_BYTES;              // per epilogue warp: two OUT_BOX buffers
constexpr uint32_t OFF_BAR = OFF_OUT + 4 * 2 * OUT_BOX;
constexpr int UNIT_RING = 16;  // claimed work units in flight between the producer and the consumers
enum { B_FULL = 0, B_EMPTY = STAGES, B_TFULL = 2 * STAGES, B_TEMPTY = 2 * STAGES + 2, B_DRAIN = 2 * STAGES + 4,
       B_UNIT = 2 * STAGES + 5, NBAR = 2 * STAGES + 5 + UNIT_RING };
constexpr uint32_t SMEM_BYTES = OFF_BAR + 8 * NBAR + 16 + 4 * UNIT_RING + 1024;
constexpr int THREADS = 192;
constexpr uint32_t TM_COLS = 512;
constexpr long long DRAIN_BUDGET = 2000000000LL;

enum Epi { PLAIN = 0, SWIGLU = 1, QKNORM128 = 2, QKNORM256 = 3, RESADD = 4, PARTIAL = 5 };

__device__ int g_gemm_error = 0;

struct Params {
  int m, n, k;          // C is m x (n, or n / 2 for SWIGLU)
  int m_tiles, n_tiles, k_steps;
  // QKNORM: the attention projection [q_h gate_h]... k_0.. v_0.. (head_dim columns each)
  int hq, hkv;
  const bf16* q_norm_w;  // [D] offsets of the (1 + w) RMSNorm
  const bf16* k_norm_w;
  const int32_t* positions;
  const float* rope;     // [max_pos][rot]: cos then sin of p * inv_freq
  int max_pos;
  float eps;
  int band;             // n-blocks per band of the tile order
  int k_split, kps;     // work unit = (tile, one of k_split slices of kps k-steps); RESADD only splits
  int* tickets;         // RESADD with k_split > 1: [tiles][4] slice tickets, then the claim and exit
                        // counters of the dynamic schedule (all zero between calls)
  int dynamic;          // units claimed from tickets[4 tiles] instead of the static round robin
  bf16* c;
  int64_t ldc;
};

// work unit -> (tile, first k-step, k-steps); the slices of one tile are consecutive units
__device__ __forceinline__ void unit_coords(int u, const Params& p, int& t, int& ks0, int& nks) {
  t = u / p.k_split;
  ks0 = (u - t * p.k_split) * p.kps;
  nks = min(p.kps, p.k_steps - ks0);
}

// tile index -> (m block, n block): bands of p.band n-blocks, n fastest inside a band (the ~148
// tiles in flight share a few A row blocks and the band's B blocks in L2)
__device__ __forceinline__ void tile_coords(int t, const Params& p, int& mb, int& nb) {
  const int band_tiles = p.band * p.m_tiles;
  const int band = t / band_tiles, r = t - band * band_tiles;
  const int width = min(p.band, p.n_tiles - band * p.band);
  mb = r / width;
  nb = band * p.band + (r - mb * width);
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
            const __grid_constant__ CUtensorMap tc, const __grid_constant__ CUtensorMap tq,
            const __grid_constant__ CUtensorMap tk, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + OFF_BAR;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * NBAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + 8 * NBAR + 4);
  volatile int* unit_ring = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * NBAR + 16);
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int num_units = p.m_tiles * p.n_tiles * p.k_split;
  int* claim = p.dynamic ? p.tickets + 4 * p.m_tiles * p.n_tiles : nullptr;  // then the exit counter
  // The unit of this CTA's local-th turn, -1 when there is none left.  Static: round robin.
  // Dynamic (ordered split-K): the producer claims units from an atomic counter and publishes them
  // in a ring with one mbarrier an entry; a claimed unit's earlier slices were claimed before it,
  // by CTAs that are running, so every ticket wait has a running producer.  The ring cannot be
  // overrun: the producer is at most STAGES k-steps (units) ahead of the MMAs, which are at most
  // two units ahead of the epilogue.
  auto consumer_unit = [&](int local, bool& ok) -> int {
    if (!p.dynamic) {
      const int u = blockIdx.x + local * gridDim.x;
      return u < num_units ? u : -1;
    }
    const int e = local % UNIT_RING;
    ok = mbar_wait(bar(B_UNIT + e), (local / UNIT_RING) & 1, abort_flag);
    return ok ? unit_ring[e] : -1;
  };
  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(bar(i), (i == B_TEMPTY || i == B_TEMPTY + 1) ? 128u : 1u);
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
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tb);
      int it = 0;  // k-steps issued by this CTA (ring position)
      bool ok = true;
      for (int local = 0; ok; ++local) {
        int u;
        if (p.dynamic) {
          u = atomicAdd(claim, 1);
          if (u >= num_units) u = -1;
          unit_ring[local % UNIT_RING] = u;
          mbar_arrive(bar(B_UNIT + local % UNIT_RING));
        } else {
          u = blockIdx.x + local * gridDim.x;
          if (u >= num_units) u = -1;
        }
        if (u < 0) break;
        int t, ks0, nks, mb, nb;
        unit_coords(u, p, t, ks0, nks);
        tile_coords(t, p, mb, nb);
        for (int ks = ks0; ks < ks0 + nks; ++ks, ++it) {
          const int st = it % STAGES;
          if (it >= STAGES && !mbar_wait(bar(B_EMPTY + st), ((it / STAGES) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + st * ST_BYTES;
          mbar_expect_tx(bar(B_FULL + st), ST_BYTES);
          tma_load_2d(sa, &ta, bar(B_FULL + st), ks * BK, mb * BM);
          tma_load_2d(sa + A_BYTES, &tb, bar(B_FULL + st), ks * BK, nb * BN);
        }
      }
      // every issued copy has landed before the CTA exits
      volatile int never = 0;
      for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
        mbar_wait(bar(B_FULL + j % STAGES), (j / STAGES) & 1, &never, DRAIN_BUDGET);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16(BM, BN, false, false);
      int it = 0, local = 0;
      bool ok = true;
      for (; ok; ++local) {
        const int u = consumer_unit(local, ok);
        if (u < 0) break;
        int t, ks0, nks;
        unit_coords(u, p, t, ks0, nks);
        const int acc = local & 1;
        // the epilogue has drained this accumulator (its previous use was tile local - 2)
        if (local >= 2 && !mbar_wait(bar(B_TEMPTY + acc), ((local >> 1) - 1) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)acc * BN;
        for (int ks = ks0; ks < ks0 + nks; ++ks, ++it) {
          const int st = it % STAGES;
          if (!mbar_wait(bar(B_FULL + st), (it / STAGES) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + st * ST_BYTES;
          const uint64_t da = sdesc_sw128(sa, 16, 1024), db = sdesc_sw128(sa + A_BYTES, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_ss(d, da + (uint32_t)(2 * kk), db + (uint32_t)(2 * kk), IDESC, (ks > ks0 || kk > 0) ? 1u : 0u);
          umma_commit(bar(B_EMPTY + st));
        }
        if (ok) umma_commit(bar(B_TFULL + acc));
      }
      volatile int never = 0;
      umma_commit(bar(B_DRAIN));
      mbar_wait(bar(B_DRAIN), 0, &never, DRAIN_BUDGET);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    // Thread = output row = TMEM lane.  Each 64-column piece of the warp's 32 rows is converted to
    // bf16 into a 128-byte-swizzled [32][64] shared-memory block and written by one TMA store
    // (rows past m and columns past n are clipped by the tensor map); two blocks per warp alternate.
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    const uint32_t obuf = base + OFF_OUT + (uint32_t)q4 * 2 * OUT_BOX;
    uint8_t* obuf_g = gbase + OFF_OUT + q4 * 2 * OUT_BOX;
    int local = 0, pieces = 0;
    auto put_piece = [&](const float (&f)[64], const CUtensorMap* map, int x, int y) {
      const int b = pieces & 1;
      if (lane == 0 && pieces >= 2) bulk_wait_read<1>();  // the store that used buffer b is done reading
      __syncwarp();
      uint8_t* dst = obuf_g + b * OUT_BOX + lane * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = f[j * 8 + i];
        *reinterpret_cast<uint4*>(dst + ((j ^ (lane & 7)) << 4)) = pack8(h);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(map, obuf + b * OUT_BOX, x, y);
        bulk_commit();
      }
      ++pieces;
    };
    for (;; ++local) {
      bool uok = true;
      const int u = __shfl_sync(0xffffffffu, consumer_unit(local, uok), 0);
      if (u < 0) break;
      const int acc = local & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(B_TFULL + acc), (local >> 1) & 1, abort_flag) ? 1 : 0)) break;
      tc_fence_after();
      int t, ks0, nks, mb, nb;
      unit_coords(u, p, t, ks0, nks);
      tile_coords(t, p, mb, nb);
      const int y = mb * BM + q4 * 32;
      const uint32_t tacc = tmem + lane_addr + (uint32_t)acc * BN;
      if constexpr (EPI == PLAIN) {
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t v[2][32];
          tmem_ld32(tacc + c * 64, v[0]);
          tmem_ld32(tacc + c * 64 + 32, v[1]);
          tmem_ld_wait();
          if (c == BN / 64 - 1) {  // the accumulator is free once its last columns are in registers
            tc_fence_before();
            mbar_arrive(bar(B_TEMPTY + acc));
          }
          float f[64];
#pragma unroll
          for (int i = 0; i < 64; ++i) f[i] = __uint_as_float(v[i >> 5][i & 31]);
          put_piece(f, &tc, nb * BN + c * 64, y);
        }
      } else if constexpr (EPI == RESADD) {
        // C (fp32) += acc: 32-column pieces staged as [32 rows][32 fp32] (128-byte rows, swizzled)
        // and added by TMA reduce-add stores, so the k-slices of a tile sum in place.  The slices add
        // in a fixed order (slice 0 first): this warp's rows wait on their ticket until the previous
        // slice's adds have completed, so results do not depend on scheduling.
        const int slice = u - t * p.k_split;
        int* ticket = p.k_split > 1 ? p.tickets + (int64_t)t * 4 + q4 : nullptr;
        if (ticket != nullptr && slice > 0) {
          bool ok = true;
          if (lane == 0) {
            const long long t0 = clock64();
            for (uint32_t i = 0;; ++i) {
              int v;
              asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(ticket) : "memory");
              if (v == slice) break;
              if ((i & 63) == 63 && (*abort_flag || clock64() - t0 > 4000000000LL)) {
                *abort_flag = 1;
                ok = false;
                break;
              }
              __nanosleep(32);
            }
            asm volatile("fence.proxy.async.global;\n" ::: "memory");
          }
          if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        }
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tacc + c * 32, v);
          tmem_ld_wait();
          if (c == BN / 32 - 1) {
            tc_fence_before();
            mbar_arrive(bar(B_TEMPTY + acc));
          }
          const int b = pieces & 1;
          if (lane == 0 && pieces >= 2) bulk_wait_read<1>();
          __syncwarp();
          uint8_t* dst = obuf_g + b * OUT_BOX + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(dst + ((j ^ (lane & 7)) << 4)) = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_2d(&tc, obuf + b * OUT_BOX, nb * BN + c * 32, y);
            bulk_commit();
          }
          ++pieces;
        }
        if (ticket != nullptr && lane == 0) {  // this slice's adds are done: pass the ticket on
          bulk_wait<0>();
          asm volatile("fence.proxy.async.global;\n" ::: "memory");
          __threadfence();
          const int next = slice + 1 == p.k_split ? 0 : slice + 1;  // the last slice leaves it zeroed
          asm volatile("st.release.gpu.global.b32 [%0], %1;\n" ::"l"(ticket), "r"(next) : "memory");
        }
        __syncwarp();
      } else if constexpr (EPI == PARTIAL) {
        // k-slice `slice` of the tile -> plane `slice` of C ([k_split][m][n] float32, a 3-D map with
        // [32 rows][32 fp32] boxes, 128-byte swizzle): plain TMA stores, no ordering between slices
        const int slice = u - t * p.k_split;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tacc + c * 32, v);
          tmem_ld_wait();
          if (c == BN / 32 - 1) {
            tc_fence_before();
            mbar_arrive(bar(B_TEMPTY + acc));
          }
          const int b = pieces & 1;
          if (lane == 0 && pieces >= 2) bulk_wait_read<1>();
          __syncwarp();
          uint8_t* dst = obuf_g + b * OUT_BOX + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(dst + ((j ^ (lane & 7)) << 4)) = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tc, obuf + b * OUT_BOX, nb * BN + c * 32, y, slice);
            bulk_commit();
          }
          ++pieces;
        }
      } else if constexpr (EPI == SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < BN / 128; ++c) {
          float f[64];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t g[32], u[32];
            tmem_ld32(tacc + c * 64 + h * 32, g);
            tmem_ld32(tacc + BN / 2 + c * 64 + h * 32, u);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float gv = __uint_as_float(g[i]);
              f[h * 32 + i] = gv / (1.0f + __expf(-gv)) * __uint_as_float(u[i]);
            }
          }
          if (c == BN / 128 - 1) {
            tc_fence_before();
            mbar_arrive(bar(B_TEMPTY + acc));
          }
          put_piece(f, &tc, nb * (BN / 2) + c * 64, y);
        }
      } else {
        // QKNORM: head blocks of D columns; q / k blocks get RMSNorm (1 + w) over the head and the
        // rotary embedding of their first D / 4 features ([tf]:657-668), then go to q_out / k_out
        constexpr int D = EPI == QKNORM128 ? 128 : 256, ROT = D / 4, HALF = ROT / 2;
        const int m = mb * BM + row;
        int pos = (m < p.m) ? p.positions[m] : 0;
        pos = pos < 0 ? 0 : (pos >= p.max_pos ? p.max_pos - 1 : pos);
        const float* cs = p.rope + (int64_t)pos * ROT;  // cos[0:HALF] then sin[0:HALF]
        const int qcols = 2 * p.hq * D, kcols = p.hkv * D;
#pragma unroll 1
        for (int blk = 0; blk < BN / D; ++blk) {
          const int c0 = nb * BN + blk * D;  // first column of this head block
          if (c0 >= p.n) break;
          const uint32_t tb0 = tacc + blk * D;
          const bool is_q = c0 < qcols && ((c0 / D) & 1) == 0;
          const bool is_k = c0 >= qcols && c0 < qcols + kcols;
          if (!is_q && !is_k) {  // output gate or v: stored as computed
#pragma unroll 1
            for (int c = 0; c < D / 64; ++c) {
              uint32_t v[2][32];
              tmem_ld32(tb0 + c * 64, v[0]);
              tmem_ld32(tb0 + c * 64 + 32, v[1]);
              tmem_ld_wait();
              float f[64];
#pragma unroll
              for (int i = 0; i < 64; ++i) f[i] = __uint_as_float(v[i >> 5][i & 31]);
              put_piece(f, &tc, c0 + c * 64, y);
            }
            continue;
          }
          float ss = 0.f;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(tb0 + c * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) ss = fmaf(__uint_as_float(v[i]), __uint_as_float(v[i]), ss);
          }
          const float inv = rsqrtf(ss / (float)D + p.eps);
          const bf16* wn = is_q ? p.q_norm_w : p.k_norm_w;
          const CUtensorMap* map = is_q ? &tq : &tk;
          const int head = is_q ? c0 / (2 * D) : (c0 - qcols) / D;
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t v[2][32];
            tmem_ld32(tb0 + c * 64, v[0]);
            tmem_ld32(tb0 + c * 64 + 32, v[1]);
            tmem_ld_wait();
            float f[64];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float wv[8];
              unpack8(__ldg(reinterpret_cast<const uint4*>(wn + c * 64 + j * 8)), wv);
#pragma unroll
              for (int i = 0; i < 8; ++i) f[j * 8 + i] = __uint_as_float(v[(j * 8 + i) >> 5][(j * 8 + i) & 31]) * inv * (1.0f + wv[i]);
            }
            if (c == 0) {  // rotate-half over the first ROT features (all inside the first piece)
              float r[ROT];
#pragma unroll
              for (int i = 0; i < ROT; ++i) {
                const int ii = i < HALF ? i : i - HALF;
                const float cv = __ldg(cs + ii), sv = __ldg(cs + HALF + ii);
                r[i] = i < HALF ? fmaf(f[i], cv, -f[i + HALF] * sv) : fmaf(f[i], cv, f[i - HALF] * sv);
              }
#pragma unroll
              for (int i = 0; i < ROT; ++i) f[i] = r[i];
            }
            put_piece(f, map, head * D + c * 64, y);
          }
        }
        tc_fence_before();
        mbar_arrive(bar(B_TEMPTY + acc));
      }
    }
    if (lane == 0) bulk_wait<0>();  // every store has completed before the CTA exits
    __syncwarp();
  }
  // ------------------------------------------------------------------ teardown
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
  if (tid == 0 && *abort_flag) atomicOr(&g_gemm_error, 1);
  if (tid == 0 && p.dynamic) {  // the last CTA out leaves both counters zeroed for the next call
    __threadfence();
    if (atomicAdd(claim + 1, 1) == (int)gridDim.x - 1) {
      claim[0] = 0;
      claim[1] = 0;
      __threadfence();
    }
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

// [rows][cols] bf16 (row stride ld elements), box 64 x box_rows, 128-byte swizzle; out-of-range
// rows / columns read as zero (ragged m, n and k tails)
static int kmajor_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeFn enc = encode_fn();
  if (!enc) return set_error(FDK_ERR_DEVICE, "gemm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm: tensor map encode failed (%d)", (int)r);
  return FDK_OK;
}

// [rows][cols] float32 (row stride ld elements), box 32 x box_rows, 128-byte swizzle
static int f32_map(CUtensorMap* m, void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeFn enc = encode_fn();
  if (!enc) return set_error(FDK_ERR_DEVICE, "gemm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm: tensor map encode failed (%d)", (int)r);
  return FDK_OK;
}

}  // namespace gemm

int gemm_take_device_error() {
  int h = 0;
  if (cudaMemcpyFromSymbol(&h, gemm::g_gemm_error, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (h) {
    int zero = 0;
    cudaMemcpyToSymbol(gemm::g_gemm_error, &zero, sizeof(int));
  }
  return h;
}

}  // namespace fdk

using namespace fdk;

extern "C" int fdk_gemm_bf16(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc, int64_t m,
                             int64_t n, int64_t k, int epilogue, void* stream) {
  using namespace fdk::gemm;
  if (int st = check_device()) return st;
  if (!a || !b || !c) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm: null pointer");
  if (epilogue != PLAIN && epilogue != SWIGLU)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm: unknown epilogue %d", epilogue);
  if (m < 0 || n <= 0 || k <= 0 || m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm: bad sizes m=%lld n=%lld k=%lld", (long long)m, (long long)n,
                     (long long)k);
  if (n % 8 || k % 8) return set_error(FDK_ERR_ALIGNMENT, "gemm: n and k must be multiples of 8 (16-byte rows)");
  if (epilogue == SWIGLU && n % BN)
    return set_error(FDK_ERR_UNSUPPORTED, "gemm: the SwiGLU epilogue needs n (gate + up rows) a multiple of %d", BN);
  const int64_t nout = epilogue == SWIGLU ? n / 2 : n;
  if (lda < k || ldb < k || ldc < nout) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm: row stride too small");
  if (!aligned16(a) || !aligned16(b) || !aligned16(c) || lda % 8 || ldb % 8 || ldc % 8)
    return set_error(FDK_ERR_ALIGNMENT, "gemm: pointers and row strides must be 16-byte aligned");
  if (m == 0) return FDK_OK;
  CUtensorMap ma, mb, mc;
  if (int st = kmajor_map(&ma, a, m, k, lda, BM)) return st;
  if (int st = kmajor_map(&mb, b, n, k, ldb, BN)) return st;
  if (int st = kmajor_map(&mc, c, m, nout, ldc, 32)) return st;  // output: [32 rows][64 cols] boxes
  Params p{};
  p.m = (int)m;
  p.n = (int)n;
  p.k = (int)k;
  p.m_tiles = (int)((m + BM - 1) / BM);
  p.n_tiles = (int)((n + BN - 1) / BN);
  p.k_steps = (int)((k + BK - 1) / BK);
  p.band = 8;  // measured: sweeping every n-block first (A read from HBM once) was no faster
  p.k_split = 1;
  p.kps = p.k_steps;
  p.c = static_cast<bf16*>(c);
  p.ldc = ldc;
  const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
  if (tiles > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "gemm: too many tiles");
  const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (epilogue == SWIGLU) {
    if (int st = ensure_smem_attr((const void*)gemm_kernel<SWIGLU>, (int)SMEM_BYTES, "gemm")) return st;
    gemm_kernel<SWIGLU><<<grid, THREADS, SMEM_BYTES, s>>>(ma, mb, mc, mc, mc, p);
  } else {
    if (int st = ensure_smem_attr((const void*)gemm_kernel<PLAIN>, (int)SMEM_BYTES, "gemm")) return st;
    gemm_kernel<PLAIN><<<grid, THREADS, SMEM_BYTES, s>>>(ma, mb, mc, mc, mc, p);
  }
  return check_launch("gemm");
}

extern "C" int fdk_gemm_bf16_qk_norm_rope(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                                          int64_t m, int64_t n, int64_t k, int64_t hq, int64_t hkv, int64_t head_dim,
                                          const void* q_norm_w, const void* k_norm_w, const int32_t* positions,
                                          const float* rope_table, int64_t max_pos, int rot_dim, float eps, void* q_out,
                                          void* k_out, void* stream) {
  using namespace fdk::gemm;
  if (int st = check_device()) return st;
  if (!a || !b || !c || !q_norm_w || !k_norm_w || !positions || !rope_table || !q_out || !k_out)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_qk_norm_rope: null pointer");
  if (head_dim != 128 && head_dim != 256)
    return set_error(FDK_ERR_UNSUPPORTED, "gemm_qk_norm_rope: head_dim=%lld (128 or 256)", (long long)head_dim);
  if (rot_dim != head_dim / 4)
    return set_error(FDK_ERR_UNSUPPORTED, "gemm_qk_norm_rope: rot_dim must be head_dim / 4 (partial rotary factor 0.25)");
  if (hq < 1 || hkv < 1 || hq > 4096 || hkv > 4096 || max_pos < 1 || max_pos > 0x7fffffff)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_qk_norm_rope: bad head counts or max_pos");
  if (n != (2 * hq + 2 * hkv) * head_dim)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_qk_norm_rope: n must be (2 hq + 2 hkv) x head_dim");
  if (m < 0 || k <= 0 || m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_qk_norm_rope: bad sizes");
  if (k % 8) return set_error(FDK_ERR_ALIGNMENT, "gemm_qk_norm_rope: k must be a multiple of 8");
  if (lda < k || ldb < k || ldc < n) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_qk_norm_rope: row stride too small");
  if (!aligned16(a) || !aligned16(b) || !aligned16(c) || !aligned16(q_out) || !aligned16(k_out) || !aligned16(q_norm_w) ||
      !aligned16(k_norm_w) || lda % 8 || ldb % 8 || ldc % 8)
    return set_error(FDK_ERR_ALIGNMENT, "gemm_qk_norm_rope: pointers and row strides must be 16-byte aligned");
  if (m == 0) return FDK_OK;
  CUtensorMap ma, mb, mc, mq, mk;
  if (int st = kmajor_map(&ma, a, m, k, lda, BM)) return st;
  if (int st = kmajor_map(&mb, b, n, k, ldb, BN)) return st;
  if (int st = kmajor_map(&mc, c, m, n, ldc, 32)) return st;
  if (int st = kmajor_map(&mq, q_out, m, hq * head_dim, hq * head_dim, 32)) return st;
  if (int st = kmajor_map(&mk, k_out, m, hkv * head_dim, hkv * head_dim, 32)) return st;
  Params p{};
  p.m = (int)m;
  p.n = (int)n;
  p.k = (int)k;
  p.m_tiles = (int)((m + BM - 1) / BM);
  p.n_tiles = (int)((n + BN - 1) / BN);
  p.k_steps = (int)((k + BK - 1) / BK);
  p.band = 8;
  p.k_split = 1;
  p.kps = p.k_steps;
  p.c = static_cast<bf16*>(c);
  p.ldc = ldc;
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.q_norm_w = static_cast<const bf16*>(q_norm_w);
  p.k_norm_w = static_cast<const bf16*>(k_norm_w);
  p.positions = positions;
  p.rope = rope_table;
  p.max_pos = (int)max_pos;
  p.eps = eps;
  const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
  if (tiles > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "gemm_qk_norm_rope: too many tiles");
  const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 128) {
    if (int st = ensure_smem_attr((const void*)gemm_kernel<QKNORM128>, (int)SMEM_BYTES, "gemm_qk_norm_rope")) return st;
    gemm_kernel<QKNORM128><<<grid, THREADS, SMEM_BYTES, s>>>(ma, mb, mc, mq, mk, p);
  } else {
    if (int st = ensure_smem_attr((const void*)gemm_kernel<QKNORM256>, (int)SMEM_BYTES, "gemm_qk_norm_rope")) return st;
    gemm_kernel<QKNORM256><<<grid, THREADS, SMEM_BYTES, s>>>(ma, mb, mc, mq, mk, p);
  }
  return check_launch("gemm_qk_norm_rope");
}

extern "C" int fdk_gemm_bf16_residual_add(const void* a, int64_t lda, const void* b, int64_t ldb, float* h, int64_t ldh,
                                          int64_t m, int64_t n, int64_t k, int split_k, int32_t* tickets,
                                          void* stream) {
  using namespace fdk::gemm;
  if (int st = check_device()) return st;
  if (!a || !b || !h) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_residual_add: null pointer");
  if (m < 0 || n <= 0 || k <= 0 || m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_residual_add: bad sizes");
  if (split_k < 0 || split_k > 16) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_residual_add: split_k in [0, 16]");
  if (n % 8 || k % 8) return set_error(FDK_ERR_ALIGNMENT, "gemm_residual_add: n and k must be multiples of 8");
  if (lda < k || ldb < k || ldh < n) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_residual_add: row stride too small");
  if (!aligned16(a) || !aligned16(b) || !aligned16(h) || lda % 8 || ldb % 8 || ldh % 4)
    return set_error(FDK_ERR_ALIGNMENT, "gemm_residual_add: pointers and row strides must be 16-byte aligned");
  if (m == 0) return FDK_OK;
  CUtensorMap ma, mb, mh;
  if (int st = kmajor_map(&ma, a, m, k, lda, BM)) return st;
  if (int st = kmajor_map(&mb, b, n, k, ldb, BN)) return st;
  if (int st = f32_map(&mh, h, m, n, ldh, 32)) return st;  // [32 rows][32 fp32] boxes
  Params p{};
  p.m = (int)m;
  p.n = (int)n;
  p.k = (int)k;
  p.m_tiles = (int)((m + BM - 1) / BM);
  p.n_tiles = (int)((n + BN - 1) / BN);
  p.k_steps = (int)((k + BK - 1) / BK);
  p.band = 8;
  const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
  if (tiles * 16 > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "gemm_residual_add: too many tiles");
  // 0 = no split: ordered slices serialise their epilogues, measured slower than one slice at
  // m = 1536 (config-4 forward 5.46 ms unsplit, 5.97 with 2 slices, 6.19 with 3)
  int s = split_k > 0 ? split_k : 1;
  if (s > p.k_steps) s = p.k_steps;
  if (tickets == nullptr) s = 1;  // ordered slices need the caller's ticket array
  p.kps = (p.k_steps + s - 1) / s;
  p.k_split = (p.k_steps + p.kps - 1) / p.kps;  // every slice non-empty
  p.c = nullptr;
  p.ldc = ldh;
  p.tickets = p.k_split > 1 ? tickets : nullptr;
  p.dynamic = p.k_split > 1 ? 1 : 0;
  const int64_t units = tiles * p.k_split;
  const int grid = (int)(units < sm_count() ? units : sm_count());
  if (int st = ensure_smem_attr((const void*)gemm_kernel<RESADD>, (int)SMEM_BYTES, "gemm_residual_add")) return st;
  gemm_kernel<RESADD><<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(ma, mb, mh, mh, mh, p);
  return check_launch("gemm_residual_add");
}

extern "C" int fdk_gemm_bf16_partials(const void* a, int64_t lda, const void* b, int64_t ldb, float* partials,
                                      int64_t m, int64_t n, int64_t k, int slices, void* stream) {
  using namespace fdk::gemm;
  if (int st = check_device()) return st;
  if (!a || !b || !partials) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_partials: null pointer");
  if (m < 0 || n <= 0 || k <= 0 || m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
    return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_partials: bad sizes");
  if (slices < 1 || slices > 16) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_partials: slices in [1, 16]");
  if (n % 8 || k % 8) return set_error(FDK_ERR_ALIGNMENT, "gemm_partials: n and k must be multiples of 8");
  if (lda < k || ldb < k) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_partials: row stride too small");
  if (!aligned16(a) || !aligned16(b) || !aligned16(partials) || lda % 8 || ldb % 8)
    return set_error(FDK_ERR_ALIGNMENT, "gemm_partials: pointers and row strides must be 16-byte aligned");
  if (m == 0) return FDK_OK;
  Params p{};
  p.m = (int)m;
  p.n = (int)n;
  p.k = (int)k;
  p.m_tiles = (int)((m + BM - 1) / BM);
  p.n_tiles = (int)((n + BN - 1) / BN);
  p.k_steps = (int)((k + BK - 1) / BK);
  p.band = 8;
  int s = slices > p.k_steps ? p.k_steps : slices;
  p.kps = (p.k_steps + s - 1) / s;
  p.k_split = (p.k_steps + p.kps - 1) / p.kps;  // every slice non-empty
  if (p.k_split != slices)
    return set_error(FDK_ERR_UNSUPPORTED, "gemm_partials: %d slices of %d k-steps leave one empty; use %d", slices,
                     p.k_steps, p.k_split);
  CUtensorMap ma, mb, mp;
  if (int st = kmajor_map(&ma, a, m, k, lda, BM)) return st;
  if (int st = kmajor_map(&mb, b, n, k, ldb, BN)) return st;
  {  // [slices][m][n] float32, box 32 x 32 x 1, 128-byte swizzle
    EncodeFn enc = encode_fn();
    if (!enc) return set_error(FDK_ERR_DEVICE, "gemm_partials: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)n, (cuuint64_t)m, (cuuint64_t)slices};
    cuuint64_t strides[2] = {(cuuint64_t)n * 4, (cuuint64_t)m * n * 4};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(&mp, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, partials, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(FDK_ERR_INVALID_ARGUMENT, "gemm_partials: tensor map encode failed (%d)", (int)r);
  }
  const int64_t units = (int64_t)p.m_tiles * p.n_tiles * p.k_split;
  if (units > 0x7fffffff) return set_error(FDK_ERR_UNSUPPORTED, "gemm_partials: too many tiles");
  const int grid = (int)(units < sm_count() ? units : sm_count());
  if (int st = ensure_smem_attr((const void*)gemm_kernel<PARTIAL>, (int)SMEM_BYTES, "gemm_partials")) return st;
  gemm_kernel<PARTIAL><<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(ma, mb, mp, mp, mp, p);
  return check_launch("gemm_partials");
}
