// rw_attn_fwd: chunk attention forward, o = softmax(q k^T * scale) v, non-causal,
// bf16 in/out, for head dim 128 — the host entry point, the work split and the
// merge of split key ranges.  The kernel itself is attn_pair.cu (CTA pairs on
// 2-SM tcgen05.mma).
//
// Replaces the reference's attention call for the cached chunk
// (wan_5b/modules/action_model.py:302 -> wan_5b/modules/attention.py:133-179):
// the current chunk's queries attend every key of kv_cache[:, :local_end]
// (sink + recent + retrieved landmarks + the chunk itself), no mask, default
// scale head_dim^-1/2.  Optionally the 3-D RoPE (+ PM-RoPE phase) of
// causal_model.py:156-184 / action_model.py:40-51 is applied to q in shared
// memory before the first QK^T, so raw (normed, un-roped) q can be passed.
//
// Work split.  A unit is one (batch, head, 256-row query block) over all keys.
// With a workspace, the resident CTA pairs (Np of them) run floor(U / Np) waves
// of whole units (pair p: units p, p + Np, ...; the pairs busy at the same time
// share heads, so K/V come from L2), then each walks an equal share of the
// remaining units' key tiles, taken in unit-major order (a share may start and
// end inside units).  The parts of units that a pair does not cover whole write
// unnormalised partial results to two workspace slots per pair, which
// combine_kernel merges.  Every pair thus gets the same work whatever the number
// of units, and a unit is cut only where a share boundary falls.  Without a
// workspace every pair runs one whole unit.
#include "common.cuh"
#include "host_util.h"
#include "rope.cuh"
#include "se3.cuh"
#include "sp_sync.cuh"

namespace rw {
namespace attn {

constexpr int BM = 128;  // query rows per CTA of a pair
constexpr int BN = 128;  // keys per key tile
constexpr int HD = 128;  // head dim

// one partial slot: O [128 columns][256 rows] fp32 (column-major), m [256], l [256]
constexpr long long SLOT_FLOATS = 128LL * 256 + 2 * 256;

// First tile of pair p's share of the T tiles (same arithmetic as the kernel).
__host__ __device__ inline long long share_start(long long T, int Np, int p) { return T * p / Np; }

// Merges the partial results of every tail unit that no single pair covered whole:
// m = max m_s, o = sum_s 2^((m_s - m) * scale_log2) * O_s / sum_s 2^((m_s - m) * scale_log2) * l_s
// over the unit's segments s.  The segment of pair p inside unit u sits in slot
// 2p when it is p's first segment (p's share starts inside u), else in 2p + 1.
// Block (unit, row half, column quarter); one thread per query row and 32 head
// dims; partial O is column-major so the loads of a warp coalesce.  With
// peer_ptrs set (sequence-parallel layer, batch 1), row t of local head h goes to
// rank t / peer_Ls, row t % peer_Ls, head peer_h0 + h of its [Ls, peer_H, 128]
// buffer instead of `out`.
constexpr int COMBINE_COLS = 32;
// One block's share of combine_kernel (returns early for rows and units with nothing to merge).
__device__ __forceinline__ void combine_unit(const float* __restrict__ scratch, uint8_t* __restrict__ out,
                                             long long o_sb, long long o_sl, long long o_sh, int Lq, int H, int nqp,
                                             int n_kv, int U, int Np, float scale_log2,
                                             const unsigned long long* __restrict__ peer_ptrs, int peer_Ls,
                                             int peer_H, int peer_h0, const Se3Out& se3) {
  const int base = (U / Np) * Np;                  // units of the waves (written whole)
  const int unit = base + (int)blockIdx.x, i = blockIdx.y, c0 = blockIdx.z * COMBINE_COLS, r = threadIdx.x;
  const long long T = (long long)(U - base) * n_kv;
  const long long a = (long long)(unit - base) * n_kv, b = a + n_kv;  // the unit's tail tiles [a, b)
  auto pair_of = [&](long long t) {
    int q = (int)(t * Np / T);
    while (q + 1 < Np && share_start(T, Np, q + 1) <= t) ++q;
    while (q > 0 && share_start(T, Np, q) > t) --q;
    return q;
  };
  const int p_lo = pair_of(a), p_hi = pair_of(b - 1);
  if (p_lo == p_hi && share_start(T, Np, p_lo) <= a && share_start(T, Np, p_lo + 1) >= b) return;  // written whole
  const int qp = unit % nqp, head = (unit / nqp) % H, bb = unit / (nqp * H);  // global unit
  const int row_tok = qp * 2 * BM + i * BM + r;
  if (row_tok >= Lq) return;
  const int row = i * BM + r;
  auto slot_of = [&](int q) { return share_start(T, Np, q) >= a ? 2 * q : 2 * q + 1; };
  float m = -INFINITY;
  for (int q = p_lo; q <= p_hi; ++q) m = fmaxf(m, scratch[slot_of(q) * SLOT_FLOATS + 128 * 256 + row]);
  float acc[COMBINE_COLS];
#pragma unroll
  for (int c = 0; c < COMBINE_COLS; ++c) acc[c] = 0.f;
  float L = 0.f;
  for (int q = p_lo; q <= p_hi; ++q) {
    const float* sp = scratch + (size_t)slot_of(q) * SLOT_FLOATS;
    const float w = exp2f((sp[128 * 256 + row] - m) * scale_log2);
    L += w * sp[128 * 256 + 256 + row];
#pragma unroll
    for (int c = 0; c < COMBINE_COLS; ++c) acc[c] += w * sp[(size_t)(c0 + c) * 256 + row];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint8_t* row_base;
  if (peer_ptrs != nullptr) {
    const int owner = row_tok / peer_Ls;
    row_base = reinterpret_cast<uint8_t*>(peer_ptrs[owner]) +
               2 * (((long long)(row_tok - owner * peer_Ls) * peer_H + peer_h0 + head) * 128);
  } else {
    row_base = out + 2 * ((long long)bb * o_sb + (long long)row_tok * o_sl + head * o_sh);
  }
  uint4* dst = reinterpret_cast<uint4*>(row_base + 2 * c0);
  // optional P y beside y (local output only): the row's frame matrix times the
  // bf16 output values
  float pm[16];
  uint4* pdst = nullptr;
  if (se3.mats != nullptr && peer_ptrs == nullptr) {
    se3_mat(se3.mats, se3.frames, bb, row_tok / se3.fs, pm);
    pdst = reinterpret_cast<uint4*>(
        se3.out + 2 * ((long long)bb * se3.sb + (long long)row_tok * se3.sl + head * se3.sh + c0));
  }
#pragma unroll
  for (int q = 0; q < COMBINE_COLS / 8; ++q) {
    uint4 v;
    v.x = pack_bf16x2(acc[8 * q + 0] * inv, acc[8 * q + 1] * inv);
    v.y = pack_bf16x2(acc[8 * q + 2] * inv, acc[8 * q + 3] * inv);
    v.z = pack_bf16x2(acc[8 * q + 4] * inv, acc[8 * q + 5] * inv);
    v.w = pack_bf16x2(acc[8 * q + 6] * inv, acc[8 * q + 7] * inv);
    dst[q] = v;
    if (pdst != nullptr) pdst[q] = se3_chunk(pm, v);
  }
}

__global__ void __launch_bounds__(128)
    combine_kernel(const float* __restrict__ scratch, uint8_t* __restrict__ out, long long o_sb, long long o_sl,
                   long long o_sh, int Lq, int H, int nqp, int n_kv, int U, int Np, float scale_log2,
                   const unsigned long long* __restrict__ peer_ptrs, int peer_Ls, int peer_H, int peer_h0,
                   const __grid_constant__ rw_sp_sync_t sync, int sync_signal, const __grid_constant__ Se3Out se3) {
  griddep_launch_dependents();  // the next kernel may be scheduled; it waits for this one
  griddep_wait();  // launched as a programmatic dependent of the attention: its slots are complete
  combine_unit(scratch, out, o_sb, o_sl, o_sh, Lq, H, nqp, n_kv, U, Np, scale_log2, peer_ptrs, peer_Ls, peer_H,
               peer_h0, se3);
  if (sync_signal) sp_signal_done(sync);  // every merged row is at its owner rank
}


// Work shape of one call: Np pairs; `shared` when pairs share tail units
// (workspace and merge needed; tail = the units after whole waves).
struct Work {
  int Np;
  bool shared;
};

// Units of fewer key tiles than this run whole even with a workspace: for short
// key ranges the merge launch and the partial results' traffic cost more than the
// idle pairs of a partial last wave (24 heads x 2640 queries: 512 keys 43.9 us
// whole vs 54.2 split, 2640 keys 100 vs 106, 5280 keys (42 tiles) 163 vs 163).
constexpr int SPLIT_MIN_KV = 43;

inline Work work_for(int units, int n_kv, int resident, bool have_workspace) {
  if (!have_workspace || resident < 1 || n_kv < SPLIT_MIN_KV) return Work{units, false};
  int Np = resident;
  if ((long long)units * n_kv < Np) Np = units * n_kv;  // all of it is tail: one tile per pair at least
  if (units % Np == 0) return Work{units, false};        // whole waves only
  if ((long long)(units % Np) * n_kv < Np) return Work{units, false};  // tail too short to share
  return Work{Np, true};
}

inline long long workspace_bytes_for(const Work& w) {
  return w.shared ? 2LL * w.Np * SLOT_FLOATS * (long long)sizeof(float) : 0;
}

}  // namespace attn

namespace pair {  // attn_pair.cu
int resident_pairs();
int launch(const void* q, const void* k, const void* v, void* o, int B, int Lq, int Lk, int H, long long q_sb,
           long long q_sl, long long q_sh, long long k_sb, long long k_sl, long long k_sh, long long v_sb,
           long long v_sl, long long v_sh, long long o_sb, long long o_sl, long long o_sh, float scale_log2,
           const rw_rope_t* rope, int* status, float* scratch, int nqp, int U, int Np,
           const unsigned long long* peer_ptrs, int peer_Ls, int peer_H, int peer_h0, const rw_sp_sync_t* sync,
           bool sync_signal, const Se3Out& se3, cudaStream_t stream);
}  // namespace pair
}  // namespace rw

using namespace rw;

extern "C" long long rw_attn_workspace_bytes(int B, int Lq, int Lk, int H) {
  if (B < 1 || Lq < 1 || Lk < 1 || H < 1) return 0;
  const int nqp = (Lq + 2 * attn::BM - 1) / (2 * attn::BM);
  const int n_kv = (Lk + attn::BN - 1) / attn::BN;
  return attn::workspace_bytes_for(attn::work_for(B * H * nqp, n_kv, pair::resident_pairs(), true));
}

namespace {

struct PeerArgs {
  const unsigned long long* ptrs;  // nullptr: output to o
  int Ls, H, h0;
  const rw_sp_sync_t* sync;        // nullptr: the caller orders the exchanges
};

int attn_run(const void* q, const void* k, const void* v, void* o, int B, int Lq, int Lk, int H, int D, long long q_sb,
             long long q_sl, long long q_sh, long long k_sb, long long k_sl, long long k_sh, long long v_sb,
             long long v_sl, long long v_sh, long long o_sb, long long o_sl, long long o_sh, float softmax_scale,
             const rw_rope_t* rope, void* workspace, long long workspace_bytes, int* status, void* stream,
             const PeerArgs& peer, const Se3Out& se3) {
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
  if (rope != nullptr && !rope_args_ok(*rope, D)) return RW_ERR_INVALID_ARG;
  if (se3.mats != nullptr) {
    // P y beside y: local output only, whole frames, 16-byte aligned rows
    if (peer.ptrs != nullptr) return RW_ERR_UNSUPPORTED;
    if (se3.out == nullptr || se3.fs < 1 || Lq % se3.fs != 0 || se3.frames != Lq / se3.fs) return RW_ERR_INVALID_ARG;
    if (!aligned16(se3.mats) || !aligned16(se3.out)) return RW_ERR_INVALID_ARG;
    const long long ps[3] = {se3.sb, se3.sl, se3.sh};
    for (int i = 0; i < 3; ++i)
      if (!(i == 0 && B == 1) && !stride_ok(ps[i])) return RW_ERR_INVALID_ARG;
  }
  const float scale_log2 = softmax_scale * 1.4426950408889634f;
  const int nqp = (Lq + 2 * attn::BM - 1) / (2 * attn::BM);
  const int n_kv = (Lk + attn::BN - 1) / attn::BN;
  const int units = B * H * nqp;
  attn::Work wk = attn::work_for(units, n_kv, pair::resident_pairs(), workspace != nullptr);
  if (wk.shared && (workspace_bytes < attn::workspace_bytes_for(wk) || !aligned16(workspace)))
    wk = attn::work_for(units, n_kv, 0, false);
  // with a sync record the signal comes from the last kernel that writes output rows
  const int rc = pair::launch(q, k, v, o, B, Lq, Lk, H, q_sb, q_sl, q_sh, k_sb, k_sl, k_sh, v_sb, v_sl, v_sh, o_sb,
                              o_sl, o_sh, scale_log2, rope, status, wk.shared ? (float*)workspace : nullptr, nqp,
                              units, wk.Np, peer.ptrs, peer.Ls, peer.H, peer.h0, peer.sync, !wk.shared, se3,
                              (cudaStream_t)stream);
  if (rc != RW_OK) return rc;
  if (wk.shared) {
    const int tail_units = units - (units / wk.Np) * wk.Np;
    rw_sp_sync_t none{};
    const bool sig = peer.sync != nullptr && peer.sync->signal_epoch > 0;
    // a programmatic dependent of the attention (its blocks start as the pairs finish
    // and wait for the whole attention grid before reading the slots)
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(tail_units, 2, attn::HD / attn::COMBINE_COLS);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const rw_sp_sync_t sy = sig ? *peer.sync : none;
    if (cudaLaunchKernelEx(&cfg, attn::combine_kernel, (const float*)workspace, (uint8_t*)o, o_sb, o_sl, o_sh, Lq, H,
                           nqp, n_kv, units, wk.Np, scale_log2, peer.ptrs, peer.Ls, peer.H, peer.h0, sy,
                           sig ? 1 : 0, se3) != cudaSuccess)
      return RW_ERR_CUDA;
  }
  return RW_OK;
}

}  // namespace

extern "C" int rw_attn_fwd(const void* q, const void* k, const void* v, void* o, int B, int Lq, int Lk, int H,
                           int D, long long q_sb, long long q_sl, long long q_sh, long long k_sb, long long k_sl,
                           long long k_sh, long long v_sb, long long v_sl, long long v_sh, long long o_sb,
                           long long o_sl, long long o_sh, float softmax_scale, const rw_rope_t* rope,
                           void* workspace, long long workspace_bytes, int* status, void* stream) {
  return attn_run(q, k, v, o, B, Lq, Lk, H, D, q_sb, q_sl, q_sh, k_sb, k_sl, k_sh, v_sb, v_sl, v_sh, o_sb, o_sl,
                  o_sh, softmax_scale, rope, workspace, workspace_bytes, status, stream,
                  PeerArgs{nullptr, 0, 0, 0, nullptr}, Se3Out{});
}

extern "C" int rw_attn_fwd_prope(const void* q, const void* k, const void* v, void* o, void* po, const float* mats,
                                 int frame_seqlen, int B, int Lq, int Lk, int H, int D, long long q_sb, long long q_sl,
                                 long long q_sh, long long k_sb, long long k_sl, long long k_sh, long long v_sb,
                                 long long v_sl, long long v_sh, long long o_sb, long long o_sl, long long o_sh,
                                 long long po_sb, long long po_sl, long long po_sh, float softmax_scale,
                                 const rw_rope_t* rope, void* workspace, long long workspace_bytes, int* status,
                                 void* stream) {
  if (mats == nullptr || po == nullptr || frame_seqlen < 1) return RW_ERR_INVALID_ARG;
  const Se3Out se3{mats, (uint8_t*)po, B == 1 ? 0 : po_sb, po_sl, po_sh, frame_seqlen, Lq / frame_seqlen};
  return attn_run(q, k, v, o, B, Lq, Lk, H, D, q_sb, q_sl, q_sh, k_sb, k_sl, k_sh, v_sb, v_sl, v_sh, o_sb, o_sl,
                  o_sh, softmax_scale, rope, workspace, workspace_bytes, status, stream,
                  PeerArgs{nullptr, 0, 0, 0, nullptr}, se3);
}

extern "C" int rw_sp_attn_fwd(const void* q, const void* k, const void* v, int Lq, int Lk, int Hp, int D,
                              long long q_sl, long long q_sh, long long k_sl, long long k_sh, long long v_sl,
                              long long v_sh, const unsigned long long* out_ptrs, int P, int rank, int H,
                              float softmax_scale, const rw_rope_t* rope, void* workspace,
                              long long workspace_bytes, const rw_sp_sync_t* sync, int* status, void* stream) {
  if (out_ptrs == nullptr || !q) return RW_ERR_INVALID_ARG;
  if (P < 1 || rank < 0 || rank >= P || H < 1 || Hp < 1 || H != Hp * P || Lq < 1 || (Lq % P) != 0)
    return RW_ERR_INVALID_ARG;
  if (sync != nullptr && (!sp_sync_ok(*sync) || sync->P != P || sync->rank != rank)) return RW_ERR_INVALID_ARG;
  // o is never written in this mode; q's layout stands in for it in the unused output map
  return attn_run(q, k, v, const_cast<void*>(q), 1, Lq, Lk, Hp, D, 0, q_sl, q_sh, 0, k_sl, k_sh, 0, v_sl, v_sh, 0,
                  q_sl, q_sh, softmax_scale, rope, workspace, workspace_bytes, status, stream,
                  PeerArgs{out_ptrs, Lq / P, H, rank * Hp, sync}, Se3Out{});
}
