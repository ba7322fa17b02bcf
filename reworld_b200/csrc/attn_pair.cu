// Chunk attention forward for sm_100a on CTA pairs: o = softmax(q k^T * scale) v,
// non-causal, bf16 in/out, fp32 accumulation in tensor memory.  Same contract as
// attn_fwd.cu (the reference call it replaces: wan_5b/modules/action_model.py:302
// -> wan_5b/modules/attention.py:133-179; optional 3-D RoPE + PM-RoPE phase of q,
// causal_model.py:156-184 / action_model.py:40-51, applied in shared memory).
//
// A cluster of two CTAs (a pair, one per SM) owns 256 query rows of one
// (batch, head); each CTA holds 128 of them.  The even CTA issues 2-SM
// tcgen05.mma (cta_group::2, M = 256): A rows come from each CTA's own Q tile /
// TMEM, the B operand is split between the two CTAs (keys [0, 64) / [64, 128) of
// a K tile, head dims [0, 64) / [64, 128) of a V tile), and each CTA's TMEM
// receives its own 128 rows.  Each CTA therefore loads half of every K and V
// tile (the pair reads each tile once, like one CTA with 256 rows) and its TMEM
// only holds 128 rows, which leaves room for three S buffers:
//   TMEM columns  O [0,128)  S0 [128,256)  S1 [256,384)  S2 [384,512)
// so QK^T of key tile j+3 runs while the softmax of tile j is still working and
// the tensor pipe never waits for one softmax in a serial chain.  P_j (bf16
// pairs) overwrites the first 64 columns of its S buffer.
//
// Warps (per CTA): two softmax warpgroups (warps 4w..4w+3 handle the key tiles
// j = w mod 2; one query row per thread), warp 8 TMA producer, warp 9 MMA issuer
// (even CTA) and TMEM owner (both CTAs, 2-SM allocation), warps 10-11 idle.
// Key tile j lands in S buffer j mod 3, so the QK^T of tile j + 3 can run while
// tiles j + 1 and j + 2 are in softmax.
// MMA order (single issuing thread): QK(0), QK(1), QK(2), then for every key tile
// j: PV(j), QK(j+3).  The softmax warpgroups pass the running row maximum of
// tile j to the one handling j+1 through shared memory; when the maximum grows
// by more than 2^8 (log2 units) the warpgroup rescales O in TMEM after PV(j-1)
// completed and before publishing P(j); otherwise the stale exponent base is
// kept (exact after the final division).  Each warpgroup keeps its own partial
// row sum, rebased when the shared maximum changes; the two are merged at the end.
#include "common.cuh"
#include "host_util.h"
#include "rope.cuh"
#include "se3.cuh"
#include "sp_sync.cuh"

namespace rw {
namespace pair {

constexpr int BM = 128;                      // query rows per CTA (256 per pair)
constexpr int BN = 128;                      // keys per key tile
constexpr int HD = 128;                      // head dim
constexpr int NSBUF = 3;                     // S buffers in TMEM
constexpr int NSTAGE = 4;                    // K/V stages per CTA
constexpr int Q_BYTES = BM * HD * 2;         // 32 KB
constexpr int Q_HALF = Q_BYTES / 2;          // 128 rows x 64 dims (one TMA box)
constexpr int HALF_TILE = 16384;             // 64 keys x 128 dims (K half) or 128 keys x 64 dims (V half)
constexpr int K_BOX = 8192;                  // 64 keys x 64 dims
constexpr int PRE_BYTES = NSBUF * HALF_TILE; // K halves of key tiles 0-2 (the first QKs)
constexpr int STAGE_BYTES = 2 * HALF_TILE;   // stage j: V half of key tile j, then K half of key tile j + 3
constexpr int NWG = 2;                       // softmax warpgroups (key tiles j = w mod NWG)
constexpr int NUM_THREADS = 128 * (NWG + 1);
constexpr int SMEM_BYTES = Q_BYTES + PRE_BYTES + NSTAGE * STAGE_BYTES + 1024;
constexpr int WARP_LOAD = 4 * NWG;
constexpr int WARP_MMA = 4 * NWG + 1;
constexpr int SOFTMAX_THREADS = 128 * NWG;
// Registers: the launch gives 168 per thread (384 x 168 = 64512); the producer /
// MMA warpgroup keeps 88 and the softmax warpgroups take 208: 128 x 88 + 256 x 208.
// (At 72 / 216 the compiler spills in the softmax's one-pass branch.)
// (Three softmax warpgroups at 152 registers measured 4 % slower: the softmax
// latency rose with three warps per SMSP competing for MUFU / FMA / ALU.)
constexpr int REG_SOFTMAX = 208;
constexpr int REG_OTHER = 88;
static_assert(NWG * 128 * REG_SOFTMAX + 128 * REG_OTHER <= NUM_THREADS * 168, "register split exceeds the launch's registers");
constexpr float RESCALE_THRESHOLD = 8.0f;    // log2 units
__host__ __device__ constexpr uint32_t tcol_o() { return 0u; }
__host__ __device__ constexpr uint32_t tcol_s(int b) { return 128u + 128u * (uint32_t)b; }

// Output of a sequence-parallel layer (batch 1): query token t, local head h goes
// to rank t / Ls, row t % Ls, head h0 + h of that rank's [Ls, H, 128] bf16 buffer.
struct PeerOut {
  const unsigned long long* ptrs;  // device array: every rank's buffer base (peer pointers)
  int Ls, H, h0;
};

__device__ __forceinline__ uint8_t* peer_row(const PeerOut& po, int t, int head) {
  const int owner = t / po.Ls;
  return reinterpret_cast<uint8_t*>(po.ptrs[owner]) +
         2 * (((long long)(t - owner * po.Ls) * po.H + po.h0 + head) * 128);
}

// Work.  A unit is one (batch, head, 256-row query block) over all key tiles.
// Of the U units, the first W = floor(U / Np) * Np run whole in waves: pair p of
// the Np pairs runs units p, p + Np, ..., so the pairs working at the same time
// share heads and their K/V tiles come from L2.  The key tiles of the remaining
// units form one sequence of T = (U - W) x n_kv tiles (unit-major); pair p then
// walks the tiles [p T / Np, (p + 1) T / Np) as segments (the parts of its range
// inside one unit).  A segment covering a whole unit writes the output; any
// other one writes its unnormalised partial result (O, m, l; fp32) to scratch
// slot 2p (the pair's first tail segment) or 2p + 1 (its last), merged by
// combine_kernel (attn_fwd.cu).  With Np = U every pair runs one whole unit and
// no scratch is used.
struct Params {
  int B, Lq, Lk, H;
  int nqp;
  int U;        // units
  int Np;       // pairs in the grid
  float scale_log2;
  int rope_on;
  rw_rope_t rope;
  int* status;
  float* scratch;
  PeerOut peer;  // peer.ptrs == nullptr: output through tm_o (local); else rows go to their owner ranks
  int sync_wait;    // 1: every CTA's producer waits for the ranks' scatters before its first load
  int sync_signal;  // 1: the last CTA to finish signals the ranks (no merge kernel follows)
  rw_sp_sync_t sync;
  Se3Out se3;       // se3.mats != nullptr: whole units also store P y through tm_po (local output only)
};

struct __align__(8) Barriers {
  uint64_t pre_full;             // even CTA: both CTAs' K halves of key tiles 0-2 landed
  uint64_t stage_full[NSTAGE];   // even CTA: both CTAs' halves of the stage landed
  uint64_t stage_free[NSTAGE];   // both: PV(j) and QK(j+3) reading stage j completed
  uint64_t q_full;               // own Q tile landed
  uint64_t q_ready;              // even CTA: both Q tiles RoPE'd (2 x 256 arrivals)
  uint64_t s_full[NSBUF];        // both: S of the buffer's current key tile complete
  uint64_t p_ready[NSBUF];       // even CTA: P written in both CTAs (2 x 128 arrivals)
  uint64_t m_ready[NSBUF];       // own: running maximum of a key tile published (128 arrivals)
  uint64_t o_done;            // both: last PV complete
  uint64_t epi;               // own: output rows staged in shared memory (256 arrivals)
  uint64_t drain;             // even CTA: every MMA complete
  uint32_t tmem_base;
  int abort_flag;
};

struct Ctx {
  Barriers* sb;
  uint32_t peer_abort;  // shared::cluster address of the peer's abort flag
  int* status;
};

constexpr long long SLOT_FLOATS = 128LL * 256 + 2 * 256;

struct Seg {
  int unit, kv0, kv1, slot;  // slot -1: whole unit (output written directly)
};

// Segments of one pair, in order: its whole units of the waves, then the parts
// of its tail range.
struct SegIter {
  long long t, t0, t1;  // tail range, in tiles after the waves' units
  int n_kv, pair, Np, w, waves, base;
  __device__ __forceinline__ SegIter(const Params& p, int pair_, int n_kv_)
      : n_kv(n_kv_), pair(pair_), Np(p.Np), w(0) {
    waves = p.U / p.Np;
    base = waves * p.Np;
    const long long T = (long long)(p.U - base) * n_kv_;
    t0 = T * pair_ / p.Np;
    t1 = T * (pair_ + 1) / p.Np;
    t = t0;
  }
  __device__ __forceinline__ bool next(Seg& sg) {
    if (w < waves) {
      sg.unit = w * Np + pair;
      sg.kv0 = 0;
      sg.kv1 = n_kv;
      sg.slot = -1;
      ++w;
      return true;
    }
    if (t >= t1) return false;
    const long long u = t / n_kv;
    const long long ue = (u + 1) * n_kv;
    const long long e = t1 < ue ? t1 : ue;
    sg.unit = base + (int)u;
    sg.kv0 = (int)(t - u * n_kv);
    sg.kv1 = (int)(e - u * n_kv);
    sg.slot = (sg.kv0 == 0 && sg.kv1 == n_kv) ? -1 : (t == t0 ? 2 * pair : 2 * pair + 1);
    t = e;
    return true;
  }
};

__device__ __forceinline__ void init_barriers(Barriers& sb) {
  mbar_init(&sb.pre_full, 1);
  for (int t = 0; t < NSTAGE; ++t) {
    mbar_init(&sb.stage_full[t], 1);
    mbar_init(&sb.stage_free[t], 1);
  }
  mbar_init(&sb.q_full, 1);
  mbar_init(&sb.q_ready, 2 * 256);
  for (int b = 0; b < NSBUF; ++b) {
    mbar_init(&sb.s_full[b], 1);
    mbar_init(&sb.p_ready[b], 2 * BM);
  }
  for (int b = 0; b < NSBUF; ++b) mbar_init(&sb.m_ready[b], BM);
  mbar_init(&sb.o_done, 1);
  mbar_init(&sb.epi, 256);
  mbar_init(&sb.drain, 1);
}

// Bounded wait; on expiry raises this CTA's and the peer's abort flags and
// records `err` in the status word.
__device__ __forceinline__ bool pwait(uint64_t* bar, uint32_t parity, const Ctx& c, int err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 0u) {
      if (*(volatile int*)&c.sb->abort_flag) return false;
      if (globaltimer_ns() - t0 > RW_WAIT_TIMEOUT_NS) {
        c.sb->abort_flag = 1;
        st_shared_cluster_u32(c.peer_abort, 1u);
        report_status(c.status, err);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool pwait_warp(uint64_t* bar, uint32_t parity, const Ctx& c, int err) {
  const bool ok = pwait(bar, parity, c, err);
  return __all_sync(0xffffffffu, ok);
}

// RoPE of head dims [64 h, 64 h + 64) of one row of the 128-byte-swizzled Q tile.
__device__ __forceinline__ void rope_row_half(uint8_t* tile, int r, int h, int token, int b, const rw_rope_t& rp) {
  const RopeToken rt = rope_token(rp, token, b);
  if (!rt.on) return;
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    uint4* ptr = reinterpret_cast<uint4*>(tile + h * Q_HALF + r * 128 + ((c ^ (r & 7)) << 4));
    *ptr = rope_chunk(*ptr, 8 * h + c, rt);
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                     const __grid_constant__ CUtensorMap tm_po, const __grid_constant__ Params p) {
  extern __shared__ uint8_t dsmem_raw[];
  __shared__ Barriers sb;
  __shared__ float m_sh[NSBUF][BM];    // running maximum handed from key tile j to j + 1
  __shared__ float fin[2 * NWG][BM];   // per warpgroup: exponent base and partial row sum

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_q = smem;
  uint8_t* pre = smem + Q_BYTES;
  uint8_t* stages = pre + PRE_BYTES;

  const uint32_t rank = cluster_ctarank();
  const bool even = rank == 0;
  const int warp = __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
  const int lane = threadIdx.x & 31;
  const int n_kv_all = (p.Lk + BN - 1) / BN;
  const int kv_tail = p.Lk - (n_kv_all - 1) * BN;
  const int pair_id = blockIdx.x >> 1;

  if (threadIdx.x == WARP_LOAD * 32) {
    init_barriers(sb);
    sb.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc_pair(&sb.tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem = sb.tmem_base;
  const Ctx cx{&sb, mapa_shared(smem_u32(&sb.abort_flag), rank ^ 1u), p.status};
  // Between two segments, every thread of both CTAs: all work of the segment is
  // done (the producer drained its barriers, the MMA issuer its MMAs, the
  // epilogue its store) before either CTA starts the next one.  The barriers
  // keep running: a per-key-tile barrier is indexed by the pair's running key
  // tile count J (buffer J mod 3, stage J mod NSTAGE, phase parity from J), a
  // once-per-segment barrier by the parity of the segment index.
  auto boundary = [&]() {
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
  };
  auto aborted = [&]() { return *(volatile int*)&sb.abort_flag != 0; };
  // per-segment coordinates, same in every role
  struct SegPos {
    int kv0, n_kv, slot, head, bidx, row0;
  };
  auto seg_pos = [&](const Seg& sg) {
    SegPos q;
    q.kv0 = sg.kv0;
    q.n_kv = sg.kv1 - sg.kv0;
    q.slot = sg.slot;
    const int qp = sg.unit % p.nqp;
    q.head = (sg.unit / p.nqp) % p.H;
    q.bidx = sg.unit / (p.nqp * p.H);
    q.row0 = qp * (2 * BM) + (int)rank * BM;  // this CTA's first query row
    return q;
  };

  if (warp == WARP_LOAD) {
    // ------------------------------------------------------------ producer (both CTAs)
    setmaxnreg_dec<REG_OTHER>();
    // launched as a programmatic dependent: the previous kernel (the cache write) has
    // finished and its rows are visible before the first load; every global access of
    // this kernel follows these loads
    if (lane == 0) griddep_wait();
    __syncwarp();
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_o);
    }
    if (p.sync_wait && lane == 0 && !sp_wait_peers(p.sync, p.status, &sb.abort_flag) && !aborted()) {
      // the ranks' q / k / v did not arrive in time: stop both CTAs of the pair
      sb.abort_flag = 1;
      st_shared_cluster_u32(cx.peer_abort, 1u);
    }
    __syncwarp();
    SegIter it(p, pair_id, n_kv_all);
    Seg sg;
    int J0 = 0, segi = 0;  // key tiles and segments of this pair before the current one
    for (bool first = true; it.next(sg); first = false, J0 += sg.kv1 - sg.kv0, ++segi) {
    if (!first) boundary();
    const uint32_t sph = (uint32_t)segi & 1u;  // phase parity of the once-per-segment barriers
    const SegPos sp = seg_pos(sg);
    const int kv0 = sp.kv0, n_kv = sp.n_kv, head = sp.head, bidx = sp.bidx, row0 = sp.row0;
    if (lane == 0 && !aborted()) {
      const uint64_t pol = l2_policy_evict_last();  // K/V tiles are re-read by the other query pairs of the head
      mbar_expect_tx(&sb.q_full, Q_BYTES);
      tma_load_4d(smem_q, &tm_q, &sb.q_full, 0, head, row0, bidx);
      tma_load_4d(smem_q + Q_HALF, &tm_q, &sb.q_full, 64, head, row0, bidx);
      bool ok = true;
      const int k_off = 64 * (int)rank;  // this CTA's keys of a K tile / head dims of a V tile
      auto load_k = [&](uint8_t* dst, uint32_t bar, int kt) {
        const int key0 = (kv0 + kt) * BN + k_off;
        tma_load_4d_pair(dst, &tm_k, bar, 0, head, key0, bidx, pol);
        tma_load_4d_pair(dst + K_BOX, &tm_k, bar, 64, head, key0, bidx, pol);
      };
      const int n_pre = n_kv < NSBUF ? n_kv : NSBUF;
      if (even) mbar_expect_tx(&sb.pre_full, 2 * HALF_TILE * n_pre);
      const uint32_t pre_bar = mapa_shared(smem_u32(&sb.pre_full), 0);
      for (int kt = 0; kt < n_pre; ++kt) load_k(pre + kt * HALF_TILE, pre_bar, kt);
      for (int j = 0; j < n_kv; ++j) {
        const int J = J0 + j;
        const int t = J % NSTAGE;
        if (J >= NSTAGE && !(ok = pwait(&sb.stage_free[t], (uint32_t)(J / NSTAGE - 1) & 1u, cx, RW_STATUS_TIMEOUT_LOAD)))
          break;
        const bool has_k = j + NSBUF < n_kv;
        if (even) mbar_expect_tx(&sb.stage_full[t], 2 * HALF_TILE * (has_k ? 2 : 1));
        const uint32_t bar = mapa_shared(smem_u32(&sb.stage_full[t]), 0);
        uint8_t* st = stages + t * STAGE_BYTES;
        tma_load_4d_pair(st, &tm_v, bar, k_off, head, (kv0 + j) * BN, bidx, pol);
        if (has_k) load_k(st + HALF_TILE, bar, j + NSBUF);
      }
      // The even CTA sees every issued copy of the pair complete on its barriers
      // (already consumed by the MMA issuer on the normal path); both CTAs see the
      // last stage releases land (multicast commits nobody else waits for), so
      // no arrival is in flight when the barriers are set up for the next segment.
      const int last = n_kv > NSTAGE ? n_kv - NSTAGE : 0;
      if (even) {
        mbar_wait_drain(&sb.pre_full, sph);
        for (int J = J0 + last; J < J0 + n_kv; ++J)
          mbar_wait_drain(&sb.stage_full[J % NSTAGE], (uint32_t)(J / NSTAGE) & 1u);
      }
      if (ok)
        for (int J = J0 + last; J < J0 + n_kv; ++J)
          mbar_wait_drain(&sb.stage_free[J % NSTAGE], (uint32_t)(J / NSTAGE) & 1u);
      mbar_wait_drain(&sb.q_full, sph);
    }
    __syncwarp();
    }
  } else if (warp == WARP_MMA) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    setmaxnreg_dec<REG_OTHER>();
    SegIter it(p, pair_id, n_kv_all);
    Seg sg;
    int J0 = 0, segi = 0;  // key tiles and segments of this pair before the current one
    for (bool first = true; it.next(sg); first = false, J0 += sg.kv1 - sg.kv0, ++segi) {
    if (!first) boundary();
    const uint32_t sph = (uint32_t)segi & 1u;  // phase parity of the once-per-segment barriers
    const int n_kv = sg.kv1 - sg.kv0;
    if (even && !aborted()) {
      constexpr uint32_t IDESC_QK = idesc_bf16_f32(2 * BM, BN, 0, 0);  // Q K-major, K K-major
      constexpr uint32_t IDESC_PV = idesc_bf16_f32(2 * BM, HD, 0, 1);  // P from TMEM, V MN-major
      // Descriptor bases; a byte offset d within a buffer is added as d >> 4 (the
      // start-address field never carries: shared addresses stay below 256 KB).
      const uint64_t dq = umma_desc(smem_u32(smem_q), 16, 1024);
      const uint64_t dk_pre = umma_desc(smem_u32(pre), 16, 1024);             // K halves: 64 keys, K-major
      const uint64_t dv_st = umma_desc(smem_u32(stages), 16384, 1024);        // V halves: 64 dims, MN-major
      const uint64_t dk_st = umma_desc(smem_u32(stages + HALF_TILE), 16, 1024);
      constexpr uint64_t PRE_DESC = HALF_TILE >> 4, STAGE_DESC = STAGE_BYTES >> 4;
      auto issue_qk = [](uint32_t ts, uint64_t dqa, uint64_t dkb) {
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t oa = (uint64_t)(((kk >> 2) * Q_HALF + (kk & 3) * 32) >> 4);
          const uint64_t ob = (uint64_t)(((kk >> 2) * K_BOX + (kk & 3) * 32) >> 4);
          mma_ss_pair(ts, dqa + oa, dkb + ob, IDESC_QK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [](uint32_t to, uint32_t ts, uint64_t dvb, bool acc) {
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_ts_pair(to, ts + kk * 8, dvb + (uint64_t)((kk * 2048) >> 4), IDESC_PV, (acc || kk > 0) ? 1u : 0u);
      };
      // Per key tile the issuer waits twice (P ready, stage landed) and commits
      // twice (S of tile j + 3 ready, stage j free): waits and commits cost ~100
      // clocks each and an MMA issue ~50, so one thread keeps up with 1024
      // clocks of tensor work per key tile only with this little bookkeeping.
      bool ok = pwait_warp(&sb.q_ready, sph, cx, RW_STATUS_TIMEOUT_MMA) &&
                pwait_warp(&sb.pre_full, sph, cx, RW_STATUS_TIMEOUT_MMA);
      tc_fence_after();
      if (ok) {
        const int n_pre = n_kv < NSBUF ? n_kv : NSBUF;
        if (elect_one()) {
          for (int kt = 0; kt < n_pre; ++kt) {
            const int bk = (J0 + kt) % NSBUF;
            issue_qk(tmem + tcol_s(bk), dq, dk_pre + kt * PRE_DESC);
            tc_commit_pair_mc(&sb.s_full[bk], 0x3);
          }
        }
        __syncwarp();
      }
      int b = J0 % NSBUF, t = J0 % NSTAGE;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int J = J0 + j;
        if (!(ok = pwait_warp(&sb.p_ready[b], (uint32_t)(J / NSBUF) & 1u, cx, RW_STATUS_TIMEOUT_MMA))) break;
        if (!(ok = pwait_warp(&sb.stage_full[t], (uint32_t)(J / NSTAGE) & 1u, cx, RW_STATUS_TIMEOUT_MMA))) break;
        tc_fence_after();
        if (elect_one()) {
          issue_pv(tmem + tcol_o(), tmem + tcol_s(b), dv_st + t * STAGE_DESC, j > 0);
          if (j == n_kv - 1) tc_commit_pair_mc(&sb.o_done, 0x3);
          if (j + NSBUF < n_kv) {
            // S buffer b is free again in pipe order: PV(j) reads P(j) before QK(j+3) writes it.
            issue_qk(tmem + tcol_s(b), dq, dk_st + t * STAGE_DESC);
            tc_commit_pair_mc(&sb.s_full[b], 0x3);
          }
          tc_commit_pair_mc(&sb.stage_free[t], 0x3);
        }
        __syncwarp();
        if (++b == NSBUF) b = 0;
        if (++t == NSTAGE) t = 0;
      }
      if (elect_one()) {
        tc_commit_pair_mc(&sb.drain, 0x1);
        mbar_wait_drain(&sb.drain, sph);
      }
      __syncwarp();
    }
    }
  } else if (warp < 4 * NWG) {
    // ------------------------------------------------------------ softmax + epilogue (both CTAs)
    setmaxnreg_inc<REG_SOFTMAX>();
    const int w = warp >> 2;  // key tiles j = w mod NWG
    const int r = threadIdx.x & 127;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tO = tmem + lane_base + tcol_o();
    const float sl2 = p.scale_log2;
    const uint32_t p_ready_cl0 = mapa_shared(smem_u32(&sb.p_ready[0]), 0);
    SegIter it(p, pair_id, n_kv_all);
    Seg sg;
    int n_epi = 0;  // whole units stored through shared memory so far (completions of `epi`)
    int J0 = 0, segi = 0;  // key tiles and segments of this pair before the current one
    for (bool first = true; it.next(sg); first = false, J0 += sg.kv1 - sg.kv0, ++segi) {
    if (!first) boundary();
    const uint32_t sph = (uint32_t)segi & 1u;  // phase parity of the once-per-segment barriers
    const SegPos sp = seg_pos(sg);
    const int kv0 = sp.kv0, n_kv = sp.n_kv, slot = sp.slot, head = sp.head, bidx = sp.bidx, row0 = sp.row0;
    bool ok = !aborted() && pwait_warp(&sb.q_full, sph, cx, RW_STATUS_TIMEOUT_SOFTMAX);
    if (ok && w < 2) {
      if (p.rope_on) rope_row_half(smem_q, r, w, row0 + r, bidx, p.rope);
      fence_proxy_async_smem();
      mbar_arrive_cluster(mapa_shared(smem_u32(&sb.q_ready), 0));
    }
    float m_base = -INFINITY;  // exponent base of this warpgroup's partial row sum
    uint64_t l2 = 0ull;        // packed (even-column, odd-column) partial row sums
    for (int j = w; j < n_kv && ok; j += NWG) {
      const int J = J0 + j;
      const int b = J % NSBUF;  // S buffer of key tile j
      const uint32_t tS = tmem + lane_base + tcol_s(b);
      if (!(ok = pwait_warp(&sb.s_full[b], (uint32_t)(J / NSBUF) & 1u, cx, RW_STATUS_TIMEOUT_SOFTMAX))) break;
      tc_fence_after();
      const bool tail = kv0 + j == n_kv_all - 1 && kv_tail < BN;
      // S columns [32 q, 32 q + 32) into registers, masked past the last key
      auto load_quarter = [&](int q, uint32_t (&v)[32]) {
        tmem_ld32(tS + 32 * q, v);
        tmem_wait_ld();
        reg_fence32(v);
        if (tail) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (32 * q + e >= kv_tail) v[e] = __float_as_uint(-INFINITY);
        }
      };
      // S columns [64 h, 64 h + 64) into registers (one wait for both loads); not for the
      // last key tile, whose columns past the last key need the mask of load_quarter
      auto load_half = [&](int h, uint32_t (&v)[2][32]) {
        tmem_ld32(tS + 64 * h, v[0]);
        tmem_ld32(tS + 64 * h + 32, v[1]);
        tmem_wait_ld();
        reg_fence32(v[0]);
        reg_fence32(v[1]);
      };
      // row maximum over 32 columns: four independent 3-input max chains of depth 4,
      // then a depth-2 tree
      auto quarter_max = [](const uint32_t (&v)[32], float row_max) -> float {
        float a[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint32_t* x = &v[g * 8];
          float t = fmax3(__uint_as_float(x[0]), __uint_as_float(x[1]), __uint_as_float(x[2]));
          t = fmax3(t, __uint_as_float(x[3]), __uint_as_float(x[4]));
          t = fmax3(t, __uint_as_float(x[5]), __uint_as_float(x[6]));
          a[g] = fmaxf(t, __uint_as_float(x[7]));
        }
        return fmax3(row_max, fmax3(a[0], a[1], a[2]), a[3]);
      };
      // P = 2^(s*scale_log2 - m*scale_log2) over 32 columns as 16 bf16 pairs (pk[o, o + 16)),
      // every exponential on MUFU (ex2; with the one-pass softmax, moving a share of them to
      // the FMA pipe as a polynomial measured slower); the exponentials are added into the
      // packed (even-pair, odd-pair) sums lacc.
      auto quarter_exp = [](const uint32_t (&v)[32], uint64_t sl2x2, uint64_t nmx2, uint32_t (&pk)[32],
                            const int o, uint64_t (&lacc)[2]) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint64_t xv = ffma2(f2_pack(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])), sl2x2, nmx2);
          float x0, x1;
          f2_unpack(xv, x0, x1);
          const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          lacc[e & 1] = fadd2(lacc[e & 1], f2_pack(p0, p1));
          pk[o + e] = pack_bf16x2(p0, p1);
        }
      };
      const uint64_t sl2x2 = f2_pack(sl2, sl2);
      // Every key tile after this warpgroup's first: ONE pass over S, the exponentials taken
      // against the base this warpgroup used for key tile j - 2 while the row maximum is
      // found alongside, P held in registers.  That P stands when key tile j - 1 kept the
      // same base and tile j does not call for a new one (the test of the two-pass path
      // below, so P and the row sums are bit for bit what it computes); the running-maximum
      // hand-over is then needed only after the exponentials, not between two reads of S.
      // Otherwise (the first key tiles, a rising maximum, the masked last key tile) the
      // two-pass path re-reads S, which is still in TMEM.
      float row_max = -INFINITY;
      float m_prev = -INFINITY;
      bool fast = false;
      const bool one_pass = j >= NWG && !tail;
      if (one_pass) {
        uint32_t pk[2][32];
        uint64_t l2f = l2;  // l2 with this tile's sums, in the two-pass path's order
        const float nm0 = -m_base * sl2;
        const uint64_t nm0x2 = f2_pack(nm0, nm0);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t v[2][32];
          load_half(h, v);
          uint64_t lacc[2] = {0ull, 0ull};
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            row_max = quarter_max(v[c], row_max);
            quarter_exp(v[c], sl2x2, nm0x2, pk[h], 16 * c, lacc);
          }
          l2f = fadd2(l2f, fadd2(lacc[0], lacc[1]));
        }
        const int Jp = J - 1;
        if (!(ok = pwait_warp(&sb.m_ready[Jp % NSBUF], (uint32_t)(Jp / NSBUF) & 1u, cx, RW_STATUS_TIMEOUT_SOFTMAX)))
          break;
        m_prev = m_sh[Jp % NSBUF][r];
        const float m_new = fmaxf(m_prev, row_max);
        fast = __all_sync(0xffffffffu, m_prev == m_base && !((m_new - m_prev) * sl2 > RESCALE_THRESHOLD));
        if (fast) {
          m_sh[b][r] = m_base;
          mbar_arrive(&sb.m_ready[b]);
          l2 = l2f;
          tmem_st32(tS, pk[0]);
          tmem_st32(tS + 32, pk[1]);
        }
      }
      if (!fast) {
        if (!one_pass) {
          // pass 1: row maximum
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t v[32];
            load_quarter(q, v);
            row_max = quarter_max(v, row_max);
          }
          // running maximum after key tile j - 1, from the warpgroup that handled it
          if (j > 0) {
            const int Jp = J - 1;
            if (!(ok = pwait_warp(&sb.m_ready[Jp % NSBUF], (uint32_t)(Jp / NSBUF) & 1u, cx, RW_STATUS_TIMEOUT_SOFTMAX)))
              break;
            m_prev = m_sh[Jp % NSBUF][r];
          }
        }
        const float m_new = fmaxf(m_prev, row_max);
        const bool need = (m_new - m_prev) * sl2 > RESCALE_THRESHOLD;
        const float m_use = need ? m_new : m_prev;
        m_sh[b][r] = m_use;
        mbar_arrive(&sb.m_ready[b]);
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // O holds tiles < j relative to m_prev: rescale it once PV(j-1) has landed
          // (PV(j) is issued only after this warpgroup publishes P(j)).
          const float alpha = need ? fast_exp2((m_prev - m_use) * sl2) : 1.f;
          // stage_free of key tile j - 1 is committed after PV(j-1)
          if (!(ok = pwait_warp(&sb.stage_free[(J - 1) % NSTAGE], (uint32_t)((J - 1) / NSTAGE) & 1u, cx,
                                RW_STATUS_TIMEOUT_SOFTMAX)))
            break;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + 32 * c, o);
            tmem_wait_ld();
            reg_fence32(o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + 32 * c, o);
          }
        }
        if (m_base != m_use) {  // rebase this warpgroup's partial sum (0 while it is empty)
          float l_lo, l_hi;
          f2_unpack(l2, l_lo, l_hi);
          const float f = fast_exp2((m_base - m_use) * sl2);
          l2 = f2_pack(l_lo * f, l_hi * f);
          m_base = m_use;
        }
        // pass 2: P of columns [64 h, 64 h + 64) goes to columns [32 h, 32 h + 32) of the
        // buffer (S columns already read)
        const float nm = -m_use * sl2;
        const uint64_t nmx2 = f2_pack(nm, nm);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t pk[32];
          uint64_t lacc[2] = {0ull, 0ull};
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t v[32];
            load_quarter(2 * h + c, v);
            quarter_exp(v, sl2x2, nmx2, pk, 16 * c, lacc);
          }
          l2 = fadd2(l2, fadd2(lacc[0], lacc[1]));
          tmem_st32(tS + 32 * h, pk);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_cluster(p_ready_cl0 + 8u * (uint32_t)b);
    }
    // ---- merge the three partial row sums; epilogue (warpgroups 0 and 1)
    {
      float l_lo, l_hi;
      f2_unpack(l2, l_lo, l_hi);
      fin[2 * w][r] = m_base;
      fin[2 * w + 1][r] = l_lo + l_hi;
    }
    named_bar_sync(1, SOFTMAX_THREADS);
    float m_fin = -INFINITY;
#pragma unroll
    for (int g = 0; g < NWG; ++g) m_fin = fmaxf(m_fin, fin[2 * g][r]);
    float l_row = 0.f;
#pragma unroll
    for (int g = 0; g < NWG; ++g) {
      const float lg = fin[2 * g + 1][r];
      if (lg > 0.f) l_row += lg * fast_exp2((fin[2 * g][r] - m_fin) * sl2);
    }
    ok = __all_sync(0xffffffffu, ok) && !*(volatile int*)&sb.abort_flag;
    if (ok && w < 2) ok = pwait_warp(&sb.o_done, sph, cx, RW_STATUS_TIMEOUT_SOFTMAX);
    if (ok && w < 2 && slot >= 0) {
      // partial key range: unnormalised O columns [64 w, 64 w + 64) (column-major),
      // the exponent base and the row sum, for combine_kernel
      tc_fence_after();
      float* base = p.scratch + (size_t)slot * SLOT_FLOATS;
      const int row = (int)rank * BM + r;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + 64 * w + 32 * c, o);
        tmem_wait_ld();
        reg_fence32(o);
#pragma unroll
        for (int e = 0; e < 32; ++e) base[(size_t)(64 * w + 32 * c + e) * 256 + row] = __uint_as_float(o[e]);
      }
      if (w == 0) {
        base[128 * 256 + row] = m_fin;
        base[128 * 256 + 256 + row] = l_row;
      }
    } else if (ok && w < 2 && p.peer.ptrs != nullptr) {
      // whole unit, sequence-parallel output: O / l -> bf16 stored straight into the
      // owner rank's output row (head dims [64 w, 64 w + 64), 128 contiguous bytes)
      tc_fence_after();
      const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
      const int t = row0 + r;
      uint8_t* dst = t < p.Lq ? peer_row(p.peer, t, head) + 128 * w : nullptr;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + 64 * w + 32 * c, o);
        tmem_wait_ld();
        reg_fence32(o);
        if (dst != nullptr) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + 16 * (c * 4 + q)) = v;
          }
        }
      }
    } else if (ok && w < 2) {
      // whole unit: O / l -> bf16 -> shared memory (reusing the Q tile; every QK
      // completed before o_done) -> TMA store; warpgroup w writes box w
      tc_fence_after();
      const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
      // with P y: the row's frame matrix (rows past Lq, clipped by the store, use frame 0);
      // P y is staged in the first K/V stage, idle once every PV completed (o_done)
      // until the next segment's loads, which start after the boundary
      const bool with_po = p.se3.mats != nullptr;
      float m[16];
      if (with_po) se3_mat(p.se3.mats, p.se3.frames, bidx, row0 + r < p.Lq ? (row0 + r) / p.se3.fs : 0, m);
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + 64 * w + 32 * c, o);
        tmem_wait_ld();
        reg_fence32(o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = c * 4 + q;
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv);
          v.y = pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv);
          v.z = pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv);
          v.w = pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv);
          const int off = w * Q_HALF + r * 128 + ((chunk ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(smem_q + off) = v;
          if (with_po) *reinterpret_cast<uint4*>(stages + off) = se3_chunk(m, v);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&sb.epi);
      if (threadIdx.x == 0) {
        if (pwait(&sb.epi, (uint32_t)n_epi & 1u, cx, RW_STATUS_TIMEOUT_SOFTMAX)) {
          tma_store_4d(&tm_o, smem_q, 0, head, row0, bidx);
          tma_store_4d(&tm_o, smem_q + Q_HALF, 64, head, row0, bidx);
          if (with_po) {
            tma_store_4d(&tm_po, stages, 0, head, row0, bidx);
            tma_store_4d(&tm_po, stages + Q_HALF, 64, head, row0, bidx);
          }
          bulk_commit_group();
          bulk_wait_group_read<0>();
        }
      }
    }
    if (slot < 0 && p.peer.ptrs == nullptr) ++n_epi;
    }
  } else {
    setmaxnreg_dec<REG_OTHER>();  // idle warps of the producer / MMA warpgroup
    SegIter it(p, pair_id, n_kv_all);
    Seg sg;
    for (bool first = true; it.next(sg); first = false)
      if (!first) boundary();
  }

  if (warp == WARP_LOAD && lane == 0 && aborted()) {
    // After a timeout some copies may have been issued without the matching
    // wait (the odd CTA's copies complete on the even CTA's barriers): give them
    // time to land before either CTA leaves.
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 200000ull) {
    }
  }
  if (threadIdx.x == 0) griddep_launch_dependents();  // the merge kernel may start its prologue
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA of the pair leaves while the other may still touch its memory or TMEM
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
  if (p.sync_signal) sp_signal_done(p.sync);  // every output row is at its owner rank
}

}  // namespace pair
}  // namespace rw

namespace rw {
namespace pair {

// Pairs that can be resident at once (cluster placement may leave SMs unused).
// Cached per device; concurrent first calls from several host threads compute
// the same value and the atomic store keeps the cache well defined.
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
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  if (cudaFuncSetAttribute((const void*)attn_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&n, (const void*)attn_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    n = sms / 2;
  }
  cached[dev].store(n, std::memory_order_release);
  return n;
}

int launch(const void* q, const void* k, const void* v, void* o, int B, int Lq, int Lk, int H, long long q_sb,
           long long q_sl, long long q_sh, long long k_sb, long long k_sl, long long k_sh, long long v_sb,
           long long v_sl, long long v_sh, long long o_sb, long long o_sl, long long o_sh, float scale_log2,
           const rw_rope_t* rope, int* status, float* scratch, int nqp, int U, int Np,
           const unsigned long long* peer_ptrs, int peer_Ls, int peer_H, int peer_h0, const rw_sp_sync_t* sync,
           bool sync_signal, const Se3Out& se3, cudaStream_t stream) {
  CUtensorMap mq, mk, mv, mo, mpo;
  if (make_bf16_bl_hd_map(&mq, q, B, Lq, H, HD, q_sb, q_sl, q_sh, BM) ||
      make_bf16_bl_hd_map(&mk, k, B, Lk, H, HD, k_sb, k_sl, k_sh, BN / 2) ||
      make_bf16_bl_hd_map(&mv, v, B, Lk, H, HD, v_sb, v_sl, v_sh, BN) ||
      make_bf16_bl_hd_map(&mo, o, B, Lq, H, HD, o_sb, o_sl, o_sh, BM))
    return RW_ERR_DRIVER;
  if (se3.mats == nullptr)
    mpo = mo;  // unused
  else if (make_bf16_bl_hd_map(&mpo, se3.out, B, Lq, H, HD, se3.sb, se3.sl, se3.sh, BM))
    return RW_ERR_DRIVER;
  static std::atomic<unsigned long long> attr_done{0};
  if (!ensure_smem_attr((const void*)attn_pair_kernel, SMEM_BYTES, &attr_done)) return RW_ERR_CUDA;
  Params prm{};
  prm.B = B;
  prm.Lq = Lq;
  prm.Lk = Lk;
  prm.H = H;
  prm.nqp = nqp;
  prm.U = U;
  prm.Np = Np;
  prm.scale_log2 = scale_log2;
  prm.status = status;
  prm.scratch = scratch;
  prm.peer = PeerOut{peer_ptrs, peer_Ls, peer_H, peer_h0};
  prm.se3 = se3;
  prm.rope_on = 0;
  if (rope != nullptr) {
    prm.rope = *rope;
    prm.rope_on = 1;
  }
  prm.sync_wait = 0;
  prm.sync_signal = 0;
  if (sync != nullptr) {
    prm.sync = *sync;
    prm.sync_wait = sync->wait_epoch > 0 ? 1 : 0;
    prm.sync_signal = sync_signal && sync->signal_epoch > 0 ? 1 : 0;
  }
  if (Np < 1 || U < 1 || 2LL * Np > 0x7fffffffLL) return RW_ERR_INVALID_ARG;
  if (U % Np != 0 && (long long)(U % Np) * ((Lk + BN - 1) / BN) < Np) return RW_ERR_INVALID_ARG;  // empty tail shares
  // a programmatic dependent of the previous kernel on the stream: the pairs' setup
  // (barriers, TMEM, descriptors) overlaps that kernel's last wave; the producer waits
  // for it (and then, in a sequence-parallel layer, for the ranks' signals) before the
  // first load
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(2 * Np), 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_pair_kernel, mq, mk, mv, mo, mpo, prm) == cudaSuccess ? RW_OK : RW_ERR_CUDA;
}

}  // namespace pair
}  // namespace rw
