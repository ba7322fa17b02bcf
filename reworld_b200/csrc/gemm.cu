// Dense bf16 GEMM for the projections around the chunk attention, on CTA pairs
// (2-SM tcgen05.mma, cta_group::2) with TMA-fed shared-memory stages and a
// double-buffered fp32 accumulator in tensor memory:
//   C[M, N] = act(A[M, K] B[N, K]^T + bias[N])     (bf16 in / out, fp32 accumulation)
// i.e. torch.nn.functional.linear(A, B, bias) with B the Linear's [out, in] weight,
// optionally followed by the tanh-approximated GELU, or with a residual added the
// way torch adds two bf16 tensors (C = bf16(R + bf16(A B^T + bias))).  It replaces the reference's
// nn.Linear calls of the self-attention (q/k/v projections, action_model.py:
// 164-166, stacked into one [3C, C] weight; value_proj :203; o and prope_proj
// :308-318, stacked into one [C, 2C] weight over [y | P y]) and the block's FFN
// (Linear -> GELU(tanh) -> Linear, action_model.py:547-556).
//
// A pair (cluster of two CTAs, one per SM) computes a 256 x BN tile of C: each CTA
// holds 128 rows of A and half of the BN rows of B in every stage; the even CTA
// issues M = 256 MMAs that read B from both CTAs and leave each CTA's 128 rows of
// the accumulator in its own TMEM.  Pairs are persistent and walk the tiles
// pair, pair + Np, ... (M-block fastest, so the pairs busy at the same time share
// the B block); TMEM holds two accumulators of BN columns so the epilogue of one
// tile overlaps the main loop of the next.
//
// Warps (320 threads per CTA): warp 0 TMA producer (both CTAs load their own
// halves, completion counted on the even CTA's barrier), warp 1 MMA issuer (even
// CTA) and TMEM owner, warps 2-9 epilogue (two warps per TMEM lane quarter, each
// with half of the tile's columns; one accumulator row per thread: bias,
// activation, bf16 into a swizzled shared-memory box per warp, written out by a
// TMA store of 32 rows x 32 columns that clips the rows past M).  Every wait is
// bounded; on a timeout the kernel raises both CTAs' abort flags, records a status
// bit, drains its copies and MMAs and returns.
#include "common.cuh"
#include "host_util.h"

#include <atomic>

namespace rw {
namespace gemm {

constexpr int BM = 128;            // rows of C per CTA (256 per pair)
constexpr int BK = 64;             // K per stage: one 128-byte swizzle row of bf16
constexpr int NUM_THREADS = 320;
constexpr int WARP_LOAD = 0, WARP_MMA = 1;
constexpr int EPI_THREADS = 256;           // warps 2-9: two per TMEM lane quarter, half the columns each

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;                   // 16 KB
  static constexpr int B_BYTES = (BN / 2) * BK * 2;             // this CTA's half of the B tile
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NSTAGE = (200 * 1024) / STAGE_BYTES;     // 6 (BN 256) or 8 (BN 128)
  static constexpr int STAGING_BYTES = 8 * 2048;                // one 32 x 32 bf16 box per epilogue warp
  static constexpr int SMEM_BYTES = NSTAGE * STAGE_BYTES + STAGING_BYTES + 1024;
  static constexpr int TMEM_COLS = 2 * BN;                      // two accumulators
};

struct Params {
  int M, N, K;
  int mb;                  // 256-row blocks of M
  int tiles;
  int Np;                  // pairs in the grid
  int split;               // 1: the tiles after the whole rounds are shared out by k-blocks
  float* ws;               // split: 2 * Np partial slots of 128 x BN floats (column-major)
  int* flags;              // split: 2 * Np ready flags (pair, CTA rank), zero between launches
  int epi;                 // RW_GEMM_EPI_*
  const __nv_bfloat16* bias;
  const __nv_bfloat16* R;  // residual rows (RW_GEMM_EPI_BIAS_RESIDUAL), may alias C
  long long ldr;
  __nv_bfloat16* C;
  long long ldc;
  int* status;
};

template <int NSTAGE>
struct __align__(8) Bars {
  uint64_t full[NSTAGE];   // even CTA: both CTAs' parts of the stage landed
  uint64_t empty[NSTAGE];  // both: the MMAs that read the stage completed
  uint64_t acc_full[2];    // both: accumulator buffer complete
  uint64_t acc_empty[2];   // even CTA: both CTAs' epilogues drained the buffer (2 x 128 arrivals)
  uint64_t drain;          // even CTA: every MMA issued so far completed
  uint32_t tmem_base;
  int abort_flag;
};

// One item of a pair's work: k-blocks [kb0, kb1) of a tile.  kind 0: the whole tile
// (stored); 1: the first part of a tail tile (the fp32 accumulator goes to this
// pair's workspace slot); 2: the tile's last part (adds the slots of pairs q_lo ..
// pair - 1, which computed the tile's earlier k-blocks, then stores).
struct Work {
  int tile, kb0, kb1, kind, q_lo;
};

// The pairs' work: floor(T / Np) rounds of whole tiles (pair p: tiles p, p + Np, ...)
// and, with the split on, the remaining R tiles' R * KB k-blocks as one sequence
// (tile-major) of which pair p takes [U p / Np, U (p + 1) / Np), U = R * KB: at most
// one tile's end (its final part) and the next tile's start (a partial part).  A
// pair runs its partial part first, then its final part, then its whole tiles, so a
// pair waiting on earlier pairs' partials never holds up a partial that another pair
// waits for.  Without the split the tail tiles run whole in one more round.
struct WorkIter {
  int pair, Np, KB, tiles, whole, k, n_tail;
  Work tail0, tail1;  // the tail items in order (kept out of an indexed array: no local memory)
  __device__ WorkIter(const Params& p, int pair_) : pair(pair_), Np(p.Np), KB(p.K / BK), tiles(p.tiles), k(0) {
    n_tail = 0;
    if (!p.split) {
      whole = (tiles - pair + Np - 1) / Np;  // rounds with a tile for this pair
      return;
    }
    const int W = tiles / Np;
    whole = W;
    const long long R = tiles - (long long)W * Np, U = R * KB;
    const long long s = U * pair / Np, e = U * (pair + 1) / Np;
    if (s >= e) return;
    const int js = (int)(s / KB), je = (int)((e - 1) / KB);
    Work a{W * Np + js, (int)(s - (long long)js * KB), 0, 0, 0};
    if (je == js) {
      a.kb1 = (int)(e - (long long)js * KB);
      a.kind = a.kb1 == KB ? (a.kb0 == 0 ? 0 : 2) : 1;
      if (a.kind == 2) a.q_lo = pair_of((long long)js * KB, U);
      tail0 = a;
      n_tail = 1;
      return;
    }
    // the share ends inside tile je: that partial part first, then tile js's end
    Work b{W * Np + je, 0, (int)(e - (long long)je * KB), 1, 0};
    a.kb1 = KB;
    a.kind = a.kb0 == 0 ? 0 : 2;
    if (a.kind == 2) a.q_lo = pair_of((long long)js * KB, U);
    tail0 = b;
    tail1 = a;
    n_tail = 2;
  }
  // the pair whose share holds tail k-block u
  __device__ int pair_of(long long u, long long U) const {
    int q = (int)(u * Np / U);
    while (q + 1 < Np && U * (q + 1) / Np <= u) ++q;
    while (q > 0 && U * q / Np > u) --q;
    return q;
  }
  // The tail items come first: every partial is published early, the finalising
  // epilogues overlap the whole tiles' main loops, and all pairs end on a whole tile.
  __device__ bool next(Work& w) {
    if (k < n_tail) {
      w = k == 0 ? tail0 : tail1;
      ++k;
      return true;
    }
    const int j = k - n_tail;
    if (j >= whole) return false;
    w = Work{pair + j * Np, 0, KB, 0, 0};
    ++k;
    return true;
  }
};

// 0.5 x (1 + tanh(u)) with u = sqrt(2/pi) (x + 0.044715 x^3), written as
// x * sigmoid(2u) = x / (1 + e^(-2u)) (the same function: 0.5 (1 + tanh u) = 1 / (1 + e^(-2u))).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return x / (1.0f + __expf(-2.0f * u));
}

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ Params p) {
  using C = Cfg<BN>;
  constexpr int NSTAGE = C::NSTAGE;
  extern __shared__ uint8_t dsmem_raw[];
  __shared__ Bars<NSTAGE> sb;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~uintptr_t(1023));

  const uint32_t rank = cluster_ctarank();
  const bool even = rank == 0;
  const int warp = __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&sb.full[s], 1);
      mbar_init(&sb.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sb.acc_full[b], 1);
      mbar_init(&sb.acc_empty[b], 2 * EPI_THREADS);
    }
    mbar_init(&sb.drain, 1);
    sb.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc_pair(&sb.tmem_base, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  griddep_launch_dependents();  // the next kernel may be scheduled; it waits for this one
  griddep_wait();  // launched as a dependent: the previous kernel's outputs (A, the residual) are complete
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem = sb.tmem_base;
  const uint32_t peer_abort = mapa_shared(smem_u32(&sb.abort_flag), rank ^ 1u);
  auto aborted = [&]() { return *(volatile int*)&sb.abort_flag != 0; };
  // bounded wait; on expiry raises both CTAs' abort flags and records `err`
  auto gwait = [&](uint64_t* bar, uint32_t parity, int err) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
      if (mbar_try_wait(bar, parity)) return true;
      if ((it & 15u) == 0u) {
        if (aborted()) return false;
        if (globaltimer_ns() - t0 > RW_WAIT_TIMEOUT_NS) {
          sb.abort_flag = 1;
          st_shared_cluster_u32(peer_abort, 1u);
          report_status(p.status, err);
          return false;
        }
      }
    }
  };

  if (warp == WARP_LOAD) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      const uint32_t full0 = mapa_shared(smem_u32(&sb.full[0]), 0);  // the even CTA's barriers
      int it = 0;
      bool ok = true;
      WorkIter wi(p, pair);
      Work w;
      while (ok && wi.next(w)) {
        const int m0 = (w.tile % p.mb) * 2 * BM + (int)rank * BM;
        const int n0 = (w.tile / p.mb) * BN + (int)rank * (BN / 2);
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % NSTAGE;
          if (it >= NSTAGE && !(ok = gwait(&sb.empty[s], (uint32_t)(it / NSTAGE - 1) & 1u, RW_STATUS_TIMEOUT_LOAD)))
            break;
          if (even) mbar_expect_tx(&sb.full[s], 2 * C::STAGE_BYTES);
          uint8_t* st = smem + s * C::STAGE_BYTES;
          tma_load_2d_pair(st, &tm_a, full0 + 8u * (uint32_t)s, kb * BK, m0);
          tma_load_2d_pair(st + C::A_BYTES, &tm_b, full0 + 8u * (uint32_t)s, kb * BK, n0);
        }
      }
      if (!ok) {
        // copies issued without their wait may still land: give them time before leaving
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) {
        }
      }
    }
    __syncwarp();
  } else if (warp == WARP_MMA) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (even) {
      constexpr uint32_t IDESC = idesc_bf16_f32(2 * BM, BN, 0, 0);  // A and B K-major
      const uint64_t da0 = umma_desc(smem_u32(smem), 16, 1024);
      const uint64_t db0 = umma_desc(smem_u32(smem + C::A_BYTES), 16, 1024);
      constexpr uint64_t STAGE_DESC = C::STAGE_BYTES >> 4;
      int it = 0, i = 0;
      bool ok = true;
      WorkIter wi(p, pair);
      Work w;
      for (; ok && wi.next(w); ++i) {
        const int b = i & 1;
        if (i >= 2 && !(ok = __all_sync(0xffffffffu, gwait(&sb.acc_empty[b], (uint32_t)((i >> 1) - 1) & 1u,
                                                          RW_STATUS_TIMEOUT_MMA))))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % NSTAGE;
          if (!(ok = __all_sync(0xffffffffu, gwait(&sb.full[s], (uint32_t)(it / NSTAGE) & 1u, RW_STATUS_TIMEOUT_MMA))))
            break;
          tc_fence_after();
          if (elect_one()) {
            const uint64_t da = da0 + (uint64_t)s * STAGE_DESC, db = db0 + (uint64_t)s * STAGE_DESC;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              mma_ss_pair(acc, da + (uint64_t)(2 * kk), db + (uint64_t)(2 * kk), IDESC,
                          (kb != w.kb0 || kk != 0) ? 1u : 0u);
            tc_commit_pair_mc(&sb.empty[s], 0x3);
            if (kb == w.kb1 - 1) tc_commit_pair_mc(&sb.acc_full[b], 0x3);
          }
          __syncwarp();
        }
      }
      // every MMA issued by this thread completes before TMEM is released
      if (elect_one()) {
        tc_commit_pair_mc(&sb.drain, 0x1);
        mbar_wait_drain(&sb.drain, 0);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-9, both CTAs)
    const int q = warp & 3;                                   // the TMEM lane quarter this warp may read
    const int half = (warp - 2) >> 2;                         // which half of the tile's columns
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t acc_empty0 = mapa_shared(smem_u32(&sb.acc_empty[0]), 0);
    const int erow = q * 32 + lane;                           // this thread's row within the CTA's 128
    const bool leader = warp == 2 && lane == 0;
    // this warp's staging box: 32 rows x 64 bytes, 64-byte swizzle (16-byte chunk
    // c of row r at r * 64 + ((c ^ (r / 2 % 4)) * 16): a warp's 16-byte stores of one
    // chunk column spread over all banks)
    uint8_t* stg = smem + C::NSTAGE * C::STAGE_BYTES + (warp - 2) * 2048;
    if (lane == 0) tma_prefetch_desc(&tm_c);
    int i = 0;
    WorkIter wi(p, pair);
    Work w;
    // Every epilogue thread walks every work item and meets the same named barriers
    // (a failed wait only skips the item's data work), so no thread waits at a
    // barrier for threads that left the loop.
    for (; wi.next(w); ++i) {
      const int b = i & 1;
      if (w.kind == 2) {
        // the earlier parts of the tile: wait (bounded) until every contributing pair's
        // CTA of this rank has published its slot, then let all epilogue threads read
        if (leader && !aborted()) {
          bool fine = true;
          for (int qq = w.q_lo; qq < pair && fine; ++qq) {
            int* f = p.flags + 2 * qq + (int)rank;
            const uint64_t t0 = globaltimer_ns();
            int v = 0;
            while (true) {
              asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
              if (v != 0) break;
              if (aborted() || globaltimer_ns() - t0 > RW_WAIT_TIMEOUT_NS) {
                fine = false;
                break;
              }
            }
            if (fine) *f = 0;                                 // consumed: ready for the next launch
          }
          if (!fine && !aborted()) {
            sb.abort_flag = 1;
            st_shared_cluster_u32(peer_abort, 1u);
            report_status(p.status, RW_STATUS_TIMEOUT_SOFTMAX);
          }
        }
        named_bar_sync(1, EPI_THREADS);
      }
      const bool ok = !aborted() &&
                      __all_sync(0xffffffffu, gwait(&sb.acc_full[b], (uint32_t)(i >> 1) & 1u, RW_STATUS_TIMEOUT_SOFTMAX));
      if (ok) {
        tc_fence_after();
        const int row = (w.tile % p.mb) * 2 * BM + (int)rank * BM + erow;
        const int n0 = (w.tile / p.mb) * BN;
        float* slot = p.ws + (size_t)(2 * pair + (int)rank) * (BM * BN);
#pragma unroll 1
        for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + (uint32_t)(b * BN + 32 * c), r);
          tmem_wait_ld();
          reg_fence32(r);
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
          if (w.kind == 1) {
            // partial: fp32 column-major, a warp's 32 rows of a column are one 128-byte line
#pragma unroll
            for (int e = 0; e < 32; ++e) slot[(size_t)(32 * c + e) * BM + erow] = v[e];
            continue;
          }
          if (w.kind == 2) {
            for (int qq = w.q_lo; qq < pair; ++qq) {
              const float* src = p.ws + (size_t)(2 * qq + (int)rank) * (BM * BN) + (size_t)(32 * c) * BM + erow;
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] += __ldcg(src + (size_t)e * BM);
            }
          }
          if (p.epi != RW_GEMM_EPI_NONE) {
            const uint4* bp = reinterpret_cast<const uint4*>(p.bias + n0 + 32 * c);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const uint4 bb = __ldg(bp + g);
              const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                v[8 * g + 2 * h] += bf16_lo(bw[h]);
                v[8 * g + 2 * h + 1] += bf16_hi(bw[h]);
              }
            }
          }
          if (p.epi == RW_GEMM_EPI_BIAS_GELU) {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = gelu_tanh(v[e]);
          }
          if (p.epi == RW_GEMM_EPI_BIAS_RESIDUAL && row < p.M) {
            // the Linear's output is rounded to bf16 first, then added to the residual in
            // fp32 and rounded again, as torch's bf16 `r + linear(x)` does
            const uint4* rp = reinterpret_cast<const uint4*>(p.R + (long long)row * p.ldr + n0 + 32 * c);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const uint4 rr = rp[g];
              const uint32_t rw_[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const uint32_t lin = pack_bf16x2(v[8 * g + 2 * h], v[8 * g + 2 * h + 1]);
                v[8 * g + 2 * h] = bf16_lo(rw_[h]) + bf16_lo(lin);
                v[8 * g + 2 * h + 1] = bf16_hi(rw_[h]) + bf16_hi(lin);
              }
            }
          }
          // bf16 row chunk -> the warp's staging box -> one TMA store of 32 rows x 32
          // columns (rows past M are clipped); the box is reused once the previous
          // store has read it
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 o;
            o.x = pack_bf16x2(v[8 * g + 0], v[8 * g + 1]);
            o.y = pack_bf16x2(v[8 * g + 2], v[8 * g + 3]);
            o.z = pack_bf16x2(v[8 * g + 4], v[8 * g + 5]);
            o.w = pack_bf16x2(v[8 * g + 6], v[8 * g + 7]);
            *reinterpret_cast<uint4*>(stg + lane * 64 + ((g ^ ((lane >> 1) & 3)) << 4)) = o;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_c, stg, n0 + 32 * c, row - lane);
            bulk_commit_group();
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(acc_empty0 + 8u * (uint32_t)b);
      if (w.kind == 1) {
        // publish the slot: every epilogue thread's stores, then one release of the flag
        named_bar_sync(1, EPI_THREADS);
        if (leader && !aborted()) {
          __threadfence();
          asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p.flags + 2 * pair + (int)rank), "r"(1)
                       : "memory");
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();                      // the last stores are done before exit
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA of the pair leaves while the other may still touch its memory or TMEM
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

// Pairs that can be resident at once for a kernel configuration, per device.
template <int BN>
int resident_pairs() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 74;
  const int known = cached[dev].load(std::memory_order_acquire);
  if (known > 0) return known;
  int n = 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg<BN>::SMEM_BYTES;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  if (cudaFuncSetAttribute((const void*)gemm_pair_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           Cfg<BN>::SMEM_BYTES) != cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&n, (const void*)gemm_pair_kernel<BN>, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    n = sms / 2;
  }
  cached[dev].store(n, std::memory_order_release);
  return n;
}

// Work shape of one call: pairs, tiles, and whether the tail tiles are shared out
// by k-blocks.  The split pays when the last round would leave over an eighth of the
// pairs idle and every pair gets at least two k-blocks of the tail.
struct Shape {
  int mb, tiles, Np;
  bool split;
};

inline Shape shape_for(int M, int N, int K, int BN, int resident) {
  Shape sh;
  sh.mb = (M + 2 * BM - 1) / (2 * BM);
  sh.tiles = sh.mb * (N / BN);
  sh.Np = sh.tiles < resident ? sh.tiles : resident;
  const long long R = sh.tiles % sh.Np;
  sh.split = R > 0 && 8 * R <= 7LL * sh.Np && R * (K / BK) >= 2LL * sh.Np;
  return sh;
}

constexpr long long FLAGS_BYTES = 4096;  // room for 2 flags per pair of up to 512 pairs

inline long long workspace_for(const Shape& sh, int BN) {
  return sh.split ? 2LL * sh.Np * BM * BN * (long long)sizeof(float) + FLAGS_BYTES : 0;
}

template <int BN>
int launch(const void* A, long long lda, const void* B, long long ldb, const void* bias, const void* R,
           long long ldr, void* Cm, long long ldc, int M, int N, int K, int epi, void* workspace,
           long long workspace_bytes, int* status, cudaStream_t stream) {
  CUtensorMap ma, mb, mc;
  if (make_bf16_2d_map(&ma, A, M, K, lda, BM) || make_bf16_2d_map(&mb, B, N, K, ldb, BN / 2) ||
      make_bf16_2d_store_map(&mc, Cm, M, N, ldc))
    return RW_ERR_DRIVER;
  static std::atomic<unsigned long long> attr_done{0};
  if (!ensure_smem_attr((const void*)gemm_pair_kernel<BN>, Cfg<BN>::SMEM_BYTES, &attr_done)) return RW_ERR_CUDA;
  Params prm{};
  prm.M = M;
  prm.N = N;
  prm.K = K;
  const Shape sh = shape_for(M, N, K, BN, resident_pairs<BN>());
  prm.mb = sh.mb;
  prm.tiles = sh.tiles;
  prm.Np = sh.Np;
  // the split needs the caller's workspace (slots, then zeroed flags); without it the
  // tail tiles run whole
  const long long need = workspace_for(sh, BN);
  prm.split = sh.split && workspace != nullptr && workspace_bytes >= need && aligned16(workspace) ? 1 : 0;
  if (prm.split) {
    prm.ws = reinterpret_cast<float*>(workspace);
    prm.flags = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(workspace) + (need - FLAGS_BYTES));
  }
  prm.epi = epi;
  prm.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  prm.R = reinterpret_cast<const __nv_bfloat16*>(R);
  prm.ldr = ldr;
  prm.C = reinterpret_cast<__nv_bfloat16*>(Cm);
  prm.ldc = ldc;
  prm.status = status;
  return launch_dependent(gemm_pair_kernel<BN>, dim3((unsigned)(2 * prm.Np)), dim3(NUM_THREADS),
                          (size_t)Cfg<BN>::SMEM_BYTES, stream, ma, mb, mc, prm) == cudaSuccess
             ? RW_OK
             : RW_ERR_CUDA;
}

}  // namespace gemm
}  // namespace rw

using namespace rw;

extern "C" long long rw_gemm_workspace_bytes(int M, int N, int K) {
  if (M < 1 || N < 1 || K < 1 || K % gemm::BK != 0 || N % 128 != 0) return 0;
  const int BN = N % 256 == 0 ? 256 : 128;
  const int res = BN == 256 ? gemm::resident_pairs<256>() : gemm::resident_pairs<128>();
  return gemm::workspace_for(gemm::shape_for(M, N, K, BN, res), BN);
}

extern "C" int rw_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, const void* bias,
                            const void* R, long long ldr, void* C, long long ldc, int M, int N, int K, int epilogue,
                            void* workspace, long long workspace_bytes, int* status, void* stream) {
  if (!A || !B || !C) return RW_ERR_INVALID_ARG;
  if (M < 1 || N < 1 || K < 1) return RW_ERR_INVALID_ARG;
  if (epilogue < RW_GEMM_EPI_NONE || epilogue > RW_GEMM_EPI_BIAS_RESIDUAL) return RW_ERR_INVALID_ARG;
  if (epilogue != RW_GEMM_EPI_NONE && (bias == nullptr || !aligned16(bias))) return RW_ERR_INVALID_ARG;
  if (epilogue == RW_GEMM_EPI_BIAS_RESIDUAL && (R == nullptr || !aligned16(R) || ldr < N || ldr % 8))
    return RW_ERR_INVALID_ARG;
  if (K % gemm::BK != 0 || N % 128 != 0) return RW_ERR_UNSUPPORTED;
  if (!aligned16(A) || !aligned16(B) || !aligned16(C)) return RW_ERR_INVALID_ARG;
  if (lda < K || ldb < K || ldc < N || lda % 8 || ldb % 8 || ldc % 8) return RW_ERR_INVALID_ARG;
  if ((long long)M * lda >= (1ll << 40) || (long long)N * ldb >= (1ll << 40)) return RW_ERR_INVALID_ARG;
  // 256-column tiles whenever N allows: 128-column tiles need 96 bytes of A and B per
  // SM clock from L2 and starve the tensor pipe (measured at the q|k|v shape); 256-column
  // ones need 64
  const bool wide = N % 256 == 0;
  return wide ? gemm::launch<256>(A, lda, B, ldb, bias, R, ldr, C, ldc, M, N, K, epilogue, workspace,
                                  workspace_bytes, status, (cudaStream_t)stream)
              : gemm::launch<128>(A, lda, B, ldb, bias, R, ldr, C, ldc, M, N, K, epilogue, workspace,
                                  workspace_bytes, status, (cudaStream_t)stream);
}
