// Chunk attention forward for sm_100a: o = softmax(q k^T * scale) v, non-causal,
// bf16 in/out, fp32 accumulation in tensor memory.
//
// Replaces the reference's attention call for the cached chunk
// (wan_5b/modules/action_model.py:302 -> wan_5b/modules/attention.py:133-179):
// the current chunk's queries attend every key of kv_cache[:, :local_end]
// (sink + recent + retrieved landmarks + the chunk itself), no mask, default
// scale head_dim^-1/2.  Optionally the 3-D RoPE (+ PM-RoPE phase) of
// causal_model.py:156-184 / action_model.py:40-51 is applied to q in shared
// memory before the first QK^T, so raw (normed, un-roped) q can be passed.
//
// One CTA owns two 128-row query tiles of one (batch, head) and streams all key
// tiles of 128 keys through a 5-slot shared-memory ring:
//   warps 0-3  softmax + epilogue of query tile 0   (one query row per thread)
//   warps 4-7  softmax + epilogue of query tile 1
//   warp  8    TMA producer (Q tiles, then K_j, V_j into the ring)
//   warp  9    tcgen05.mma issuer + TMEM owner
//   warps 10-11 idle
// Tensor memory (512 columns x 128 lanes, fp32):
//   S0 [0,128)  S1 [128,256)  O0 [256,384)  O1 [384,512);  P_i (bf16 pairs)
//   overwrites the first 64 columns of S_i once S_i has been read.
// MMA order per key tile j (single issuing thread, executed in order):
//   PV0(j-1), QK0(j), PV1(j-1), QK1(j)
// so that P_i(j-1) is consumed before S_i(j) overwrites it, and the commit that
// publishes S_i(j) also guarantees PV_i(j-1) has landed in O_i; the softmax
// warps can therefore rescale O_i in place between S_i(j) ready and P_i(j)
// published.  Rescaling is skipped unless the running row maximum grew by more
// than 2^8 in the exponent (the exponent base stays stale otherwise, which is
// exact after the final division by the row sum).
#include "common.cuh"
#include "host_util.h"
#include "rope.cuh"

namespace rw {
namespace attn {

constexpr int BM = 128;                     // query rows per tile
constexpr int BN = 128;                     // keys per tile
constexpr int HD = 128;                     // head dim
constexpr int NSLOT = 5;                    // K/V ring slots (K_j and V_j alternate)
constexpr int NSTEPBAR = 3;                 // step_free barriers (>= 3 keeps producer waits unambiguous)
constexpr int TILE_BYTES = BM * HD * 2;     // 32 KB: every Q/K/V/O tile
constexpr int HALF_BYTES = TILE_BYTES / 2;  // 128 rows x 64 columns (one TMA box)
constexpr int NUM_THREADS = 384;
constexpr int SMEM_BYTES = (2 + NSLOT) * TILE_BYTES + 1024;  // + 1 KB to align to the swizzle atom
__host__ __device__ constexpr uint32_t tcol_s(int i) { return (uint32_t)i * 128u; }        // S_i columns
__host__ __device__ constexpr uint32_t tcol_o(int i) { return 256u + (uint32_t)i * 128u; } // O_i columns
constexpr int WARP_LOAD = 8;
constexpr int WARP_MMA = 9;
constexpr float RESCALE_THRESHOLD = 8.0f;   // log2 units

// Work split.  A unit is one (batch, head, query-tile pair) over all keys.  The
// first n_whole units run whole (one CTA each, result written directly); the
// remaining n_tail units are cut into `splits` key ranges each, ordered
// piece-major so that concurrently running CTAs share a head and a key range
// (K/V tiles then come from L2), and write unnormalised partial results to the
// workspace, merged by combine_kernel.  splits == 1 means no tail.
struct Params {
  int B, Lq, Lk, H;
  int nqp;              // query-tile pairs per (batch, head)
  int n_whole, n_tail, splits;
  float scale_log2;
  int rope_on;
  rw_rope_t rope;
  int* status;
  float* scratch;       // n_tail * splits partial slots (column-major O, then m, then l)
};

// one partial slot: O [128 columns][256 rows] fp32, m [256], l [256]
constexpr long long SLOT_FLOATS = 128LL * 256 + 2 * 256;

struct __align__(8) Barriers {
  uint64_t slot_full[NSLOT];
  uint64_t q_full[2];
  uint64_t q_ready[2];
  uint64_t s_full[2];
  uint64_t p_ready[2];
  uint64_t o_done[2];
  uint64_t epi[2];
  uint64_t drain;
  uint64_t step_free[NSTEPBAR];
  uint32_t tmem_base;
  int abort_flag;
};

// Applies RoPE (+ PM-RoPE phase) in place to one 128-wide row of a
// 128-byte-swizzled Q tile (arithmetic of rope.cuh, same as the cache-store kernel).
__device__ __forceinline__ void rope_row_inplace(uint8_t* tile, int r, int token, int b, const rw_rope_t& rp) {
  const RopeToken rt = rope_token(rp, token, b);
  if (!rt.on) return;
#pragma unroll 1
  for (int c16 = 0; c16 < 16; ++c16) {
    const int half = c16 >> 3, c = c16 & 7;
    uint4* p = reinterpret_cast<uint4*>(tile + half * HALF_BYTES + r * 128 + ((c ^ (r & 7)) << 4));
    *p = rope_chunk(*p, c16, rt);
  }
}

// Warp-uniform bounded wait.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, Barriers& sb, int* status, int err) {
  const bool ok = mbar_wait(bar, parity, &sb.abort_flag, status, err);
  return __all_sync(0xffffffffu, ok);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                    const __grid_constant__ Params p) {
  extern __shared__ uint8_t dsmem_raw[];
  __shared__ Barriers sb;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_q[2] = {smem, smem + TILE_BYTES};
  uint8_t* smem_ring = smem + 2 * TILE_BYTES;

  const int warp = __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
  const int lane = threadIdx.x & 31;
  const int n_kv_all = (p.Lk + BN - 1) / BN;
  const int kv_tail = p.Lk - (n_kv_all - 1) * BN;  // valid keys in the last key tile, 1..128
  int unit, kv0, kv1, slot = -1;
  if ((int)blockIdx.x < p.n_whole) {
    unit = blockIdx.x;
    kv0 = 0;
    kv1 = n_kv_all;
  } else {
    const int t = blockIdx.x - p.n_whole;
    const int e = t % p.n_tail, piece = t / p.n_tail;
    unit = p.n_whole + e;
    kv0 = (int)((long long)piece * n_kv_all / p.splits);
    kv1 = (int)((long long)(piece + 1) * n_kv_all / p.splits);
    slot = e * p.splits + piece;
  }
  const int qp = unit % p.nqp;
  const int head = (unit / p.nqp) % p.H;
  const int bidx = unit / (p.nqp * p.H);
  const int q_row0 = qp * (2 * BM);
  const bool has_q1 = (q_row0 + BM) < p.Lq;
  const int n_kv = kv1 - kv0;  // key tiles of this CTA

  if (threadIdx.x == WARP_LOAD * 32) {
    for (int s = 0; s < NSLOT; ++s) mbar_init(&sb.slot_full[s], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sb.q_full[i], 1);
      mbar_init(&sb.q_ready[i], BM);
      mbar_init(&sb.s_full[i], 1);
      mbar_init(&sb.p_ready[i], BM);
      mbar_init(&sb.o_done[i], 1);
      mbar_init(&sb.epi[i], BM);
    }
    mbar_init(&sb.drain, 1);
    for (int t = 0; t < NSTEPBAR; ++t) mbar_init(&sb.step_free[t], 1);
    sb.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(&sb.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sb.tmem_base;
  // Registers: the launch gives 168 per thread (384 x 168 = 64512); the producer /
  // MMA warpgroup (warps 8-11) keeps 72 and hands the rest to the two softmax
  // warpgroups (216): 128 x 72 + 256 x 216 = 64512.  Each role adjusts in its own branch.

  if (warp == WARP_LOAD) {
    // ------------------------------------------------------------ producer
    setmaxnreg_dec_72();
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_o);
      const uint64_t pol = l2_policy_evict_last();  // K/V tiles are re-read by the other query CTAs of the head
      mbar_expect_tx(&sb.q_full[0], TILE_BYTES);
      tma_load_4d(smem_q[0], &tm_q, &sb.q_full[0], 0, head, q_row0, bidx);
      tma_load_4d(smem_q[0] + HALF_BYTES, &tm_q, &sb.q_full[0], 64, head, q_row0, bidx);
      if (has_q1) {
        mbar_expect_tx(&sb.q_full[1], TILE_BYTES);
        tma_load_4d(smem_q[1], &tm_q, &sb.q_full[1], 0, head, q_row0 + BM, bidx);
        tma_load_4d(smem_q[1] + HALF_BYTES, &tm_q, &sb.q_full[1], 64, head, q_row0 + BM, bidx);
      }
      uint32_t g = 0;  // ring uses issued
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        for (int t = 0; t < 2; ++t) {
          const uint32_t s = g % NSLOT;
          if (g >= (uint32_t)NSLOT) {
            // use g refills the slot of use u = g - NSLOT, freed by key tile (u + 1) / 2
            const uint32_t step = (g - NSLOT + 1) / 2;
            if (!mbar_wait(&sb.step_free[step % NSTEPBAR], (step / NSTEPBAR) & 1, &sb.abort_flag, p.status,
                           RW_STATUS_TIMEOUT_LOAD)) {
              ok = false;
              break;
            }
          }
          uint8_t* dst = smem_ring + s * TILE_BYTES;
          const CUtensorMap* m = t == 0 ? &tm_k : &tm_v;
          mbar_expect_tx(&sb.slot_full[s], TILE_BYTES);
          tma_load_4d_hint(dst, m, &sb.slot_full[s], 0, head, (kv0 + j) * BN, bidx, pol);
          tma_load_4d_hint(dst + HALF_BYTES, m, &sb.slot_full[s], 64, head, (kv0 + j) * BN, bidx, pol);
          ++g;
        }
      }
      // Every issued copy must land before the CTA may exit (normal path: already consumed).
      const uint32_t first = g > (uint32_t)NSLOT ? g - NSLOT : 0;
      for (uint32_t u = first; u < g; ++u) mbar_wait_drain(&sb.slot_full[u % NSLOT], (u / NSLOT) & 1);
      mbar_wait_drain(&sb.q_full[0], 0);
      if (has_q1) mbar_wait_drain(&sb.q_full[1], 0);
    }
    __syncwarp();
  } else if (warp == WARP_MMA) {
    // ------------------------------------------------------------ MMA issuer
    // One thread (lane 0) issues both query tiles' MMAs in the strict alternation
    // PV0(j-1), QK0(j), PV1(j-1), QK1(j): each softmax warpgroup then has the
    // other tile's two GEMMs of time to turn its S tile into P.  Per key tile it
    // commits three times: S0 ready, S1 ready, and step_free (K_j and V_{j-1}
    // no longer read), which the producer waits on before refilling those slots.
    // The whole warp runs the loop and every wait (warp-uniform control flow), so
    // the descriptors below stay warp-uniform values; lane 0 alone issues, always
    // the same thread, because a commit tracks the MMAs of the thread issuing it.
    setmaxnreg_dec_72();
    constexpr uint32_t IDESC_QK = idesc_bf16_f32(BM, BN, 0, 0);  // Q K-major, K K-major
    constexpr uint32_t IDESC_PV = idesc_bf16_f32(BM, HD, 0, 1);  // P from TMEM, V MN-major
    // Descriptor bases.  A byte offset d within the same buffer is added as d >> 4
    // to the start-address field (bits 0-13): shared addresses stay below 256 KB,
    // so the field never carries into the next one.
    const uint64_t dq0 = umma_desc(smem_u32(smem_q[0]), 16, 1024), dq1 = umma_desc(smem_u32(smem_q[1]), 16, 1024);
    const uint64_t dk_ring = umma_desc(smem_u32(smem_ring), 16, 1024);          // K tiles, K-major
    const uint64_t dv_ring = umma_desc(smem_u32(smem_ring), HALF_BYTES, 1024);  // V tiles, MN-major
    constexpr uint64_t SLOT_DESC = TILE_BYTES >> 4;
    const bool leader = lane == 0;

    const uint32_t ts0 = tmem + tcol_s(0), ts1 = tmem + tcol_s(1), to0 = tmem + tcol_o(0), to1 = tmem + tcol_o(1);
    auto issue_qk = [](uint32_t ts, uint64_t dq, uint64_t dk) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const uint64_t off = (uint64_t)(((kk >> 2) * HALF_BYTES + (kk & 3) * 32) >> 4);
        mma_ss(ts, dq + off, dk + off, IDESC_QK, kk > 0 ? 1u : 0u);
      }
    };
    auto issue_pv = [](uint32_t to, uint32_t ts, uint64_t dv, bool acc) {
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        mma_ts(to, ts + kk * 8, dv + (uint64_t)((kk * 2048) >> 4), IDESC_PV, (acc || kk > 0) ? 1u : 0u);
    };
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return warp_wait(bar, parity, sb, p.status, RW_STATUS_TIMEOUT_MMA);
    };

    bool ok = wait(&sb.q_ready[0], 0);
    if (ok && has_q1) ok = wait(&sb.q_ready[1], 0);
    tc_fence_after();
    // ring position of K_j (use 2j) and V_j (use 2j+1), advanced incrementally
    uint32_t sK = 0, parK = 0, sV = 1, parV = 0;
    uint32_t v_prev_slot = 0, v_prev_par = 0;
    uint32_t fs = 0;  // step_free barrier of key tile j
    for (int j = 0; j < n_kv && ok; ++j) {
      const uint64_t dv_prev = dv_ring + v_prev_slot * SLOT_DESC;
      if (j > 0) {
        if (!(ok = wait(&sb.p_ready[0], (j - 1) & 1))) break;
        if (!(ok = wait(&sb.slot_full[v_prev_slot], v_prev_par))) break;
        tc_fence_after();
        if (leader) issue_pv(to0, ts0, dv_prev, j > 1);
        __syncwarp();
      }
      if (!(ok = wait(&sb.slot_full[sK], parK))) break;
      const uint64_t dk = dk_ring + sK * SLOT_DESC;
      if (leader) {
        issue_qk(ts0, dq0, dk);
        tc_commit(&sb.s_full[0]);
      }
      __syncwarp();
      if (has_q1) {
        if (j > 0) {
          if (!(ok = wait(&sb.p_ready[1], (j - 1) & 1))) break;
          tc_fence_after();
          if (leader) issue_pv(to1, ts1, dv_prev, j > 1);
          __syncwarp();
        }
        if (leader) {
          issue_qk(ts1, dq1, dk);
          tc_commit(&sb.s_full[1]);
        }
        __syncwarp();
      }
      if (leader) tc_commit(&sb.step_free[fs]);  // K_j and V_{j-1} released once everything above completes
      __syncwarp();
      if (++fs == NSTEPBAR) fs = 0;
      v_prev_slot = sV;
      v_prev_par = parV;
      sK += 2;
      if (sK >= NSLOT) { sK -= NSLOT; parK ^= 1; }
      sV += 2;
      if (sV >= NSLOT) { sV -= NSLOT; parV ^= 1; }
    }
    if (ok) {
      const uint64_t dv_prev = dv_ring + v_prev_slot * SLOT_DESC;
      ok = wait(&sb.p_ready[0], (n_kv - 1) & 1) && wait(&sb.slot_full[v_prev_slot], v_prev_par);
      if (ok) {
        tc_fence_after();
        if (leader) {
          issue_pv(to0, ts0, dv_prev, n_kv > 1);
          tc_commit(&sb.o_done[0]);
        }
        __syncwarp();
        if (has_q1) {
          ok = wait(&sb.p_ready[1], (n_kv - 1) & 1);
          if (ok) {
            tc_fence_after();
            if (leader) {
              issue_pv(to1, ts1, dv_prev, n_kv > 1);
              tc_commit(&sb.o_done[1]);
            }
            __syncwarp();
          }
        }
      }
    }
    // All MMAs issued by lane 0 complete before teardown.
    if (leader) {
      tc_commit(&sb.drain);
      mbar_wait_drain(&sb.drain, 0);
    }
    __syncwarp();
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax + epilogue
    setmaxnreg_inc_216();
    const int i = warp >> 2;  // query tile of this warpgroup
    const int r = threadIdx.x & 127;
    const bool active = (i == 0) || has_q1;
    if (active) {
      const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
      const uint32_t tS = tmem + lane_base + tcol_s(i);
      const uint32_t tO = tmem + lane_base + tcol_o(i);
      const float sl2 = p.scale_log2;
      const int row0 = q_row0 + i * BM;
      bool ok = warp_wait(&sb.q_full[i], 0, sb, p.status, RW_STATUS_TIMEOUT_SOFTMAX);
      if (ok) {
        if (p.rope_on) rope_row_inplace(smem_q[i], r, row0 + r, bidx, p.rope);
        fence_proxy_async_smem();
        mbar_arrive(&sb.q_ready[i]);
      }
      float m_used = -INFINITY;
      uint64_t l2 = 0ull;  // packed (even-column, odd-column) partial row sums
      float l_lo = 0.f, l_hi = 0.f;
      for (int j = 0; j < n_kv && ok; ++j) {
        if (!(ok = warp_wait(&sb.s_full[i], j & 1, sb, p.status, RW_STATUS_TIMEOUT_SOFTMAX))) break;
        tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, sr[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) reg_fence32(sr[c]);
        if (kv0 + j == n_kv_all - 1 && kv_tail < BN) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (32 * c + e >= kv_tail) sr[c][e] = __float_as_uint(-INFINITY);
        }
        // row maximum: 3-input max tree
        float mx[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float a = fmax3(__uint_as_float(sr[c][0]), __uint_as_float(sr[c][1]), __uint_as_float(sr[c][2]));
#pragma unroll
          for (int e = 3; e + 1 < 32; e += 2)
            a = fmax3(a, __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
          mx[c] = fmaxf(a, __uint_as_float(sr[c][31]));
        }
        const float row_max = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        const float m_new = fmaxf(m_used, row_max);
        const bool need = (m_new - m_used) * sl2 > RESCALE_THRESHOLD;
        float alpha = 1.f;
        if (need) {
          alpha = fast_exp2((m_used - m_new) * sl2);
          m_used = m_new;
          l2 = f2_pack(l_lo * alpha, l_hi * alpha);
          f2_unpack(l2, l_lo, l_hi);
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // O_i is quiescent here: PV_i(j-1) completed before S_i(j) was published.
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
        // P = 2^(s*scale_log2 - m*scale_log2): three column pairs in eight on the FMA
        // pipe (exp2_poly_pair), the rest on MUFU (ex2), which balances the two
        // pipes (one MUFU ex2 costs a warp 8 issue cycles of that pipe, a polynomial
        // pair about 16 of the FMA pipe); the exponent arguments and the row sum use
        // packed fp32x2 math.
        const float nm = -m_used * sl2;
        const uint64_t sl2x2 = f2_pack(sl2, sl2), nmx2 = f2_pack(nm, nm);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t pk[32];
          uint64_t lacc[2] = {0ull, 0ull};
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int col = 64 * h + 2 * e;
            const uint64_t sv = f2_pack(__uint_as_float(sr[col >> 5][col & 31]),
                                        __uint_as_float(sr[(col + 1) >> 5][(col + 1) & 31]));
            const uint64_t xv = ffma2(sv, sl2x2, nmx2);
            float x0, x1, p0, p1;
            f2_unpack(xv, x0, x1);
            if ((0x4A >> (e & 7)) & 1) {
              exp2_poly_pair(x0, x1, p0, p1);
            } else {
              p0 = fast_exp2(x0);
              p1 = fast_exp2(x1);
            }
            lacc[e & 1] = fadd2(lacc[e & 1], f2_pack(p0, p1));
            pk[e] = pack_bf16x2(p0, p1);
          }
          l2 = fadd2(l2, fadd2(lacc[0], lacc[1]));
          tmem_st32(tS + 32 * h, pk);
        }
        f2_unpack(l2, l_lo, l_hi);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&sb.p_ready[i]);
      }
      // ---- epilogue
      if (ok) ok = warp_wait(&sb.o_done[i], 0, sb, p.status, RW_STATUS_TIMEOUT_SOFTMAX);
      if (ok && slot >= 0) {
        // partial key range: unnormalised O (column-major, coalesced across the
        // warp's rows), the exponent base m and the row sum l, for combine_kernel
        tc_fence_after();
        float* base = p.scratch + (size_t)slot * SLOT_FLOATS;
        const int row = i * BM + r;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
          reg_fence32(o);
#pragma unroll
          for (int e = 0; e < 32; ++e) base[(size_t)(32 * c + e) * 256 + row] = __uint_as_float(o[e]);
        }
        base[128 * 256 + row] = m_used;
        base[128 * 256 + 256 + row] = l_lo + l_hi;
      } else if (ok) {
        // whole unit: O_i / l -> bf16 -> smem (reusing Q_i) -> TMA store
        tc_fence_after();
        const float l = l_lo + l_hi;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint8_t* out = smem_q[i];
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
          reg_fence32(o);
          const int half = c >> 1;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = (c & 1) * 4 + q;
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv);
            *reinterpret_cast<uint4*>(out + half * HALF_BYTES + r * 128 + ((chunk ^ (r & 7)) << 4)) = v;
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&sb.epi[i]);
        if (r == 0) {
          if (mbar_wait(&sb.epi[i], 0, &sb.abort_flag, p.status, RW_STATUS_TIMEOUT_SOFTMAX)) {
            tma_store_4d(&tm_o, out, 0, head, row0, bidx);
            tma_store_4d(&tm_o, out + HALF_BYTES, 64, head, row0, bidx);
            bulk_commit_group();
            bulk_wait_group_read<0>();
          }
        }
      }
    }
  } else {
    setmaxnreg_dec_72();  // idle warps 10-11
  }

  tc_fence_before();
  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Merges the partial key ranges of each split unit: m = max m_p,
// o = sum_p 2^((m_p - m) * scale_log2) * O_p / sum_p 2^((m_p - m) * scale_log2) * l_p.
// One thread per query row; partial O is column-major so loads coalesce.
__global__ void __launch_bounds__(128)
    combine_kernel(const float* __restrict__ scratch, uint8_t* __restrict__ out, long long o_sb, long long o_sl,
                   long long o_sh, int Lq, int H, int nqp, int n_whole, int splits, float scale_log2) {
  const int e = blockIdx.x, i = blockIdx.y, r = threadIdx.x;
  const int unit = n_whole + e;
  const int qp = unit % nqp, head = (unit / nqp) % H, b = unit / (nqp * H);
  const int row_tok = qp * 2 * BM + i * BM + r;
  if (row_tok >= Lq) return;
  const int row = i * BM + r;
  const float* slot0 = scratch + (size_t)e * splits * SLOT_FLOATS;
  float m = -INFINITY;
  for (int pc = 0; pc < splits; ++pc) m = fmaxf(m, slot0[pc * SLOT_FLOATS + 128 * 256 + row]);
  float acc[128];
#pragma unroll
  for (int c = 0; c < 128; ++c) acc[c] = 0.f;
  float L = 0.f;
  for (int pc = 0; pc < splits; ++pc) {
    const float* sp = slot0 + pc * SLOT_FLOATS;
    const float w = exp2f((sp[128 * 256 + row] - m) * scale_log2);
    L += w * sp[128 * 256 + 256 + row];
#pragma unroll
    for (int c = 0; c < 128; ++c) acc[c] += w * sp[(size_t)c * 256 + row];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint4* dst = reinterpret_cast<uint4*>(out + 2 * ((long long)b * o_sb + (long long)row_tok * o_sl + head * o_sh));
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    uint4 v;
    v.x = pack_bf16x2(acc[8 * q + 0] * inv, acc[8 * q + 1] * inv);
    v.y = pack_bf16x2(acc[8 * q + 2] * inv, acc[8 * q + 3] * inv);
    v.z = pack_bf16x2(acc[8 * q + 4] * inv, acc[8 * q + 5] * inv);
    v.w = pack_bf16x2(acc[8 * q + 6] * inv, acc[8 * q + 7] * inv);
    dst[q] = v;
  }
}

// Chooses how many units run whole and into how many key ranges the rest is
// cut: minimises (whole waves) + (waves of pieces) / splits + a per-wave cost of
// ~1 % of a unit for each wave of pieces (CTA start, Q load, pipeline ramp,
// partial store); with no workspace, everything runs whole.
struct Schedule {
  int n_whole, n_tail, splits;
};

inline Schedule plan(int units, int n_kv, int sms, bool allow_split) {
  Schedule best{units, 0, 1};
  double best_cost = (double)((units + sms - 1) / sms);
  if (!allow_split || sms <= 0) return best;
  const int full_waves = units / sms;
  for (int k = full_waves; k >= 0 && k >= full_waves - 1; --k) {
    const int tail = units - k * sms;
    if (tail <= 0) continue;
    for (int S = 2; S <= 16 && S <= n_kv; ++S) {
      const long long pieces = (long long)tail * S;
      const long long waves = (pieces + sms - 1) / sms;
      const double cost = k + (double)waves / S + 0.01 * (double)waves;
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best = Schedule{k * sms, tail, S};
      }
    }
  }
  return best;
}

inline int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return sms;
}

}  // namespace attn
}  // namespace rw

using namespace rw;

extern "C" long long rw_attn_workspace_bytes(int B, int Lq, int Lk, int H) {
  if (B < 1 || Lq < 1 || Lk < 1 || H < 1) return 0;
  const int nqp = (Lq + 2 * attn::BM - 1) / (2 * attn::BM);
  const int n_kv = (Lk + attn::BN - 1) / attn::BN;
  const attn::Schedule sc = attn::plan(B * H * nqp, n_kv, attn::sm_count(), true);
  return (long long)sc.n_tail * sc.splits * attn::SLOT_FLOATS * (long long)sizeof(float);
}

extern "C" int rw_attn_fwd(const void* q, const void* k, const void* v, void* o, int B, int Lq, int Lk, int H,
                           int D, long long q_sb, long long q_sl, long long q_sh, long long k_sb, long long k_sl,
                           long long k_sh, long long v_sb, long long v_sl, long long v_sh, long long o_sb,
                           long long o_sl, long long o_sh, float softmax_scale, const rw_rope_t* rope,
                           void* workspace, long long workspace_bytes, int* status, void* stream) {
  if (!q || !k || !v || !o) return RW_ERR_INVALID_ARG;
  if (D != attn::HD) return RW_ERR_UNSUPPORTED;
  if (B < 1 || Lq < 1 || Lk < 1 || H < 1 || B > 65535 || H > 65535) return RW_ERR_INVALID_ARG;
  if (!(softmax_scale > 0.f)) return RW_ERR_INVALID_ARG;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return RW_ERR_INVALID_ARG;
  const long long strides[12] = {q_sb, q_sl, q_sh, k_sb, k_sl, k_sh, v_sb, v_sl, v_sh, o_sb, o_sl, o_sh};
  for (int i = 0; i < 12; ++i) {
    const bool batch_stride = (i % 3) == 0;
    if (batch_stride && B == 1) continue;
    if (!stride_ok(strides[i])) return RW_ERR_INVALID_ARG;
  }
  attn::Params prm{};
  prm.B = B;
  prm.Lq = Lq;
  prm.Lk = Lk;
  prm.H = H;
  prm.scale_log2 = softmax_scale * 1.4426950408889634f;
  prm.status = status;
  prm.rope_on = 0;
  if (rope != nullptr) {
    if (!rope_args_ok(*rope, D)) return RW_ERR_INVALID_ARG;
    prm.rope = *rope;
    prm.rope_on = 1;
  }
  CUtensorMap mq, mk, mv, mo;
  if (make_bf16_bl_hd_map(&mq, q, B, Lq, H, D, q_sb, q_sl, q_sh, attn::BM) ||
      make_bf16_bl_hd_map(&mk, k, B, Lk, H, D, k_sb, k_sl, k_sh, attn::BN) ||
      make_bf16_bl_hd_map(&mv, v, B, Lk, H, D, v_sb, v_sl, v_sh, attn::BN) ||
      make_bf16_bl_hd_map(&mo, o, B, Lq, H, D, o_sb, o_sl, o_sh, attn::BM))
    return RW_ERR_DRIVER;
  static unsigned long long attr_done = 0;
  if (!ensure_smem_attr((const void*)attn::attn_fwd_kernel, attn::SMEM_BYTES, &attr_done)) return RW_ERR_CUDA;
  prm.nqp = (Lq + 2 * attn::BM - 1) / (2 * attn::BM);
  const int n_kv = (Lk + attn::BN - 1) / attn::BN;
  const int units = B * H * prm.nqp;
  attn::Schedule sc = attn::plan(units, n_kv, attn::sm_count(), workspace != nullptr);
  const long long need = (long long)sc.n_tail * sc.splits * attn::SLOT_FLOATS * (long long)sizeof(float);
  if (sc.splits > 1 && (workspace_bytes < need || !aligned16(workspace))) sc = attn::Schedule{units, 0, 1};
  prm.n_whole = sc.n_whole;
  prm.n_tail = sc.n_tail;
  prm.splits = sc.splits;
  prm.scratch = (float*)workspace;
  const long long grid = (long long)sc.n_whole + (long long)sc.n_tail * sc.splits;
  if (grid > 0x7fffffffLL) return RW_ERR_INVALID_ARG;
  attn::attn_fwd_kernel<<<(unsigned)grid, attn::NUM_THREADS, attn::SMEM_BYTES, (cudaStream_t)stream>>>(mq, mk, mv, mo,
                                                                                                     prm);
  if (cudaGetLastError() != cudaSuccess) return RW_ERR_CUDA;
  if (sc.splits > 1) {
    attn::combine_kernel<<<dim3(sc.n_tail, 2), 128, 0, (cudaStream_t)stream>>>(
        (const float*)workspace, (uint8_t*)o, o_sb, o_sl, o_sh, Lq, H, prm.nqp, sc.n_whole, sc.splits,
        prm.scale_log2);
    if (cudaGetLastError() != cudaSuccess) return RW_ERR_CUDA;
  }
  return RW_OK;
}
