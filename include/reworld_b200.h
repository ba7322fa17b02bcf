/*
 * reworld_b200 — C ABI of the B200 (sm_100a) kernels for ReWorld's per-chunk
 * causal self-attention hot path (Wan2.2-TI2V-5B DiT, KV cache + landmark bank).
 *
 * All entry points take plain device pointers, sizes and element strides, run
 * on the CUDA stream passed as `stream` (a cudaStream_t; NULL = legacy default
 * stream), never allocate device memory and return RW_OK (0) or a negative
 * RW_ERR_* code.  Asynchronous failures inside a kernel (a bounded wait that
 * ran out of time) are reported through the optional device `status` word as
 * RW_STATUS_* bits; kernels never trap.
 *
 * bf16 tensors use the reference's [B, L, H, D] layout with a contiguous head
 * dimension; the other three strides are given in elements.
 */
#ifndef REWORLD_B200_H
#define REWORLD_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes --------------------------------------------------------- */
#define RW_OK 0
#define RW_ERR_INVALID_ARG (-1)  /* null pointer, bad size, misaligned pointer/stride */
#define RW_ERR_UNSUPPORTED (-2)  /* e.g. head_dim != 128 */
#define RW_ERR_CUDA (-3)         /* a CUDA runtime call failed (launch error) */
#define RW_ERR_DRIVER (-4)       /* TMA descriptor encoding failed */
#define RW_ERR_CAPACITY (-5)     /* request exceeds a fixed capacity */

/* ---- device status word bits (atomicOr'ed into *status) -------------------- */
#define RW_STATUS_TIMEOUT_LOAD 0x01     /* TMA producer wait ran out of time */
#define RW_STATUS_TIMEOUT_MMA 0x02      /* MMA issuer wait ran out of time */
#define RW_STATUS_TIMEOUT_SOFTMAX 0x04  /* softmax/epilogue wait ran out of time */
#define RW_STATUS_TIMEOUT_COPY 0x08     /* bulk-copy wait ran out of time */
#define RW_STATUS_BAD_SLOT 0x10         /* a descriptor/slot index was out of range */
#define RW_STATUS_TIMEOUT_PEER 0x20     /* a cross-rank barrier wait ran out of time */

/* 3-D RoPE parameters (the reference's causal_rope_apply + pm_rope_delta_apply).
 * freqs: the model's complex128 table [max_pos][64] stored as (real, imag)
 * double pairs (wan_5b/modules/causal_model.py:790-807, model.py:29-39).
 * Token t of the chunk (t < grid_f*grid_h*grid_w) rotates complex pair j by
 * freqs[start_frame + t/(h*w)][j] for j < c_t, freqs[(t/w)%h][j] for
 * c_t <= j < c_t+c_h and freqs[t%w][j] otherwise; tokens past f*h*w are left
 * unchanged (causal_model.py:156-184).  The rotation is done in fp64 and rounded
 * to bf16 through fp32 as the reference's .type_as() does.  delta_cs, when not
 * NULL, holds the PM-RoPE phase as fp32 (cos, sin) pairs [B][grid_f][64] and is
 * applied after that rounding, in fp32, then rounded to bf16 again
 * (wan_5b/modules/action_model.py:40-51). */
typedef struct rw_rope {
  const double* freqs;
  int max_pos;
  int start_frame;
  int grid_f, grid_h, grid_w;
  int c_t, c_h, c_w;
  const float* delta_cs;
} rw_rope_t;

/* Chunk attention forward: o = softmax(q k^T * softmax_scale) v per (batch, head),
 * non-causal, bf16 in/out, fp32 accumulation (tcgen05/TMEM, TMA-fed).
 * workspace (device memory, 16-byte aligned, rw_attn_workspace_bytes() bytes)
 * lets the last partial wave of work be split along the keys and merged by a
 * second kernel; with workspace == NULL (or too small) every (head, query-tile
 * pair) runs whole in one CTA — same results, fewer CTAs in the last wave.
 * Replaces wan_5b/modules/attention.py:133-179 `attention(q, k, v)` (and the
 * flash_attn_varlen_func call at :111-127) as called from
 * wan_5b/modules/action_model.py:302 with k/v = kv_cache[:, :local_end].
 * q,o: [B, Lq, H, 128]; k,v: [B, Lk, H, 128].  If rope != NULL the 3-D RoPE
 * (+ PM-RoPE phase) is applied to q inside the kernel before QK^T (the
 * reference applies it at action_model.py:265-275 before the call).
 * Requirements: head_dim 128, all pointers 16-byte aligned, strides multiples
 * of 8 elements, Lq >= 1, Lk >= 1, softmax_scale > 0. */
int rw_attn_fwd(const void* q, const void* k, const void* v, void* o, int B, int Lq, int Lk, int H, int D,
                long long q_sb, long long q_sl, long long q_sh, long long k_sb, long long k_sl, long long k_sh,
                long long v_sb, long long v_sl, long long v_sh, long long o_sb, long long o_sl, long long o_sh,
                float softmax_scale, const rw_rope_t* rope, void* workspace, long long workspace_bytes,
                int* status, void* stream);

/* rw_attn_fwd that also writes P y, the PRoPE O-side transform of its output,
 * for the cached self-attention's [y | P y] output projection: po[b, t, h, 4g + i]
 * = sum_k mats[b, t / frame_seqlen][i][k] * y[b, t, h, 4g + k] from the bf16
 * output values y, bit for bit what rw_se3_block_apply(y, po, mats, ...) writes,
 * without reading y back (the attention's epilogue and merge write both).
 * Replaces action_model.py:302 followed by _se3_block_apply(x, ..., "P") at
 * :307-312 (wan_5b/modules/action_model.py:84-114).  mats: [B, Lq /
 * frame_seqlen, 4, 4] fp32 (16-byte aligned); po: [B, Lq, H, 128] bf16 with
 * strides po_*; Lq a multiple of frame_seqlen.  Other arguments as rw_attn_fwd. */
int rw_attn_fwd_prope(const void* q, const void* k, const void* v, void* o, void* po, const float* mats,
                      int frame_seqlen, int B, int Lq, int Lk, int H, int D, long long q_sb, long long q_sl,
                      long long q_sh, long long k_sb, long long k_sl, long long k_sh, long long v_sb,
                      long long v_sl, long long v_sh, long long o_sb, long long o_sl, long long o_sh,
                      long long po_sb, long long po_sl, long long po_sh, float softmax_scale,
                      const rw_rope_t* rope, void* workspace, long long workspace_bytes, int* status,
                      void* stream);

/* Workspace bytes rw_attn_fwd uses for this shape on the current device (0 when
 * the work fills whole waves). */
long long rw_attn_workspace_bytes(int B, int Lq, int Lk, int H);

/* rw_attn_fwd for callers that cannot allocate device memory: a host runtime that
 * owns all device memory and gives this library no allocator, or a real-time
 * streaming loop where a cudaMalloc (which can synchronise the whole device)
 * would stall frame delivery.  Same arguments as rw_attn_fwd without the
 * workspace: the key-split scratch is a fixed array inside the library, of
 * RW_ATTN_NOALLOC_SCRATCH_BYTES (80 MiB) of device memory that each GPU loading
 * it keeps until the process exits.  A call needs 0 bytes or 2 x 133,120 bytes
 * per resident pair, whatever the shape: 19.7 MB with the 74 pairs of a B200
 * (the 704x1280 chunk included), so only a device with more than 315 resident
 * pairs could exceed the array; shapes whose scratch (rw_attn_workspace_bytes)
 * exceeds it return RW_ERR_CAPACITY.  `stream` must belong to the current
 * device (RW_ERR_INVALID_ARG otherwise).  The first call on a device looks the
 * array's device address up (once per device); make that first call before any
 * stream capture.  All
 * calls share the array, so calls that overlap on the GPU race; nothing in it
 * needs clearing between calls.  No counterpart in the reference: it is an
 * allocation-free form of this library's own entry point. */
#define RW_ATTN_NOALLOC_SCRATCH_BYTES (80LL * 1024 * 1024)
int rw_attn_fwd_noalloc(const void* q, const void* k, const void* v, void* o, int B, int Lq, int Lk, int H, int D,
                        long long q_sb, long long q_sl, long long q_sh, long long k_sb, long long k_sl,
                        long long k_sh, long long v_sb, long long v_sl, long long v_sh, long long o_sb,
                        long long o_sl, long long o_sh, float softmax_scale, const rw_rope_t* rope, int* status,
                        void* stream);

/* RoPE(+PM-RoPE) on the new chunk's K and the cache write of K and V:
 * cache_k[b, dst_start + t] = rope(k[b, t]), cache_v[b, dst_start + t] = v[b, t]
 * for t < L; optionally q_out[b, t] = rope(q_in[b, t]) when q_in != NULL.
 * Replaces wan_5b/modules/action_model.py:265-292 (causal_rope_apply on q/k,
 * pm_rope_delta_apply, and the kv_cache["k"/"v"][:, a:b] = ... writes).
 * rope may be NULL (plain copy).  Element strides as in rw_attn_fwd. */
int rw_rope_kv_store(const void* k, const void* v, const void* q_in, void* q_out, void* cache_k, void* cache_v,
                     int B, int L, int H, int D, int dst_start, long long k_sb, long long k_sl, long long k_sh,
                     long long v_sb, long long v_sl, long long v_sh, long long q_sb, long long q_sl,
                     long long q_sh, long long qo_sb, long long qo_sl, long long qo_sh, long long ck_sb,
                     long long ck_sl, long long ck_sh, long long cv_sb, long long cv_sl, long long cv_sh,
                     const rw_rope_t* rope, void* stream);

/* RMSNorm of the new chunk's q and k projections over all heads, RoPE(+PM-RoPE)
 * of k, and the cache write of k and v, in one launch:
 *   q_out[b, t]               = rmsnorm(q_in[b, t]) * w_q
 *   cache_k[b, dst_start + t] = rope(rmsnorm(k_in[b, t]) * w_k)
 *   cache_v[b, dst_start + t] = v_in[b, t]
 * Replaces wan_5b/modules/action_model.py:164-166 (norm_q / norm_k, WanRMSNorm of
 * wan_5b/modules/model.py:73-89) with the k half of :265-292.  q_in, k_in, v_in
 * are bf16 [B, L, H*D] rows (element strides *_sb, *_sl; channels contiguous),
 * w_q / w_k bf16 [H*D]; q_out [B, L, H, D] and the caches [B, cap, H, D] take
 * strides as in rw_attn_fwd.  q is returned without RoPE (the attention applies
 * it).  eps_q / eps_k are the two norms' epsilons.  rope may be NULL.  D must be
 * 128 and H <= 288 (one token's three rows, 6*H*D bytes, fit a 216 KB stage).
 * The rows are staged through shared memory by bulk copies whose waits are
 * bounded: a wait that runs out of time sets RW_STATUS_TIMEOUT_COPY in *status
 * (optional). */
int rw_qkv_norm_rope_store(const void* q_in, const void* k_in, const void* v_in, const void* w_q, const void* w_k,
                           void* q_out, void* cache_k, void* cache_v, int B, int L, int H, int D, int dst_start,
                           float eps_q, float eps_k, long long qi_sb, long long qi_sl, long long ki_sb,
                           long long ki_sl, long long vi_sb, long long vi_sl, long long qo_sb, long long qo_sl,
                           long long qo_sh, long long ck_sb, long long ck_sl, long long ck_sh, long long cv_sb,
                           long long cv_sl, long long cv_sh, const rw_rope_t* rope, int* status, void* stream);

/* PRoPE SE3 transform: out[b, t, h, 4g+i] = sum_k M[b, t / frame_seqlen][i][k] * x[b, t, h, 4g+k]
 * for every group of 4 head-dim channels.  Replaces _se3_block_apply
 * (wan_5b/modules/action_model.py:84-114) as used for the V-side P^-1 residual
 * (:194-203) and the O-side P residual (:307-318).  mats: fp32 [B, L/frame_seqlen,
 * 4, 4] in device memory holding the frames' matrices in the activation dtype's
 * values (P, or P^-1 inverted as the reference inverts it), 16-byte aligned.
 * x, out: bf16 [B, L, H, D] with element strides; L a multiple of frame_seqlen;
 * D must be 128.  fp32 accumulation, one rounding to bf16 per output. */
int rw_se3_block_apply(const void* x, void* out, const float* mats, int B, int L, int H, int D, int frame_seqlen,
                       long long x_sb, long long x_sl, long long x_sh, long long o_sb, long long o_sl,
                       long long o_sh, void* stream);

/* Row normalisations of the DiT block on bf16 rows [rows, C] (row strides in
 * elements, multiples of 8; C a multiple of 8):
 *   RW_NORM_RMS    WanRMSNorm (wan_5b/modules/model.py:73-89): y = bf16(bf16(x * r) * w),
 *                  r = 1 / sqrt(mean(x^2) + eps); w (bf16 [C]) required, b must be NULL.
 *                  The cross-attention's norm_q (model.py:175, causal_model.py:218).
 *   RW_NORM_LAYER  WanLayerNorm (model.py:92-102): y = bf16((x - mean) * rstd * w + b) with
 *                  w, b optional (elementwise_affine off: both NULL).  norm2 / norm3 of
 *                  the block (action_model.py:399-403, 547-553).
 * fp32 statistics; C <= 8192; HBM-bound, one 128-thread CTA per row. */
#define RW_NORM_RMS 0
#define RW_NORM_LAYER 1
int rw_row_norm(const void* x, void* out, const void* w, const void* b, long long rows, int C, long long x_row_stride,
                long long out_row_stride, float eps, int mode, void* stream);

/* One byte-copy job of the landmark/cache assembly: nbytes from src to dst,
 * both 16-byte aligned, nbytes a multiple of 16. */
typedef struct rw_copy_desc {
  const void* src;
  void* dst;
  long long nbytes;
} rw_copy_desc_t;

/* Executes n copy jobs (descriptor array in DEVICE memory) with one launch of a
 * TMA bulk-copy (cp.async.bulk) kernel: the landmark gather of
 * longctx/inference/landmark_cache_v2.py:618-682 (write_into_cache, direct-write
 * path) and :362-397 (read_pair_into), for all layers at once.  Jobs must not
 * overlap each other's destinations.  Bit-exact byte copies. */
int rw_copy_chunks(const rw_copy_desc_t* descs, int n, int* status, void* stream);

/* A camera pose as the landmark bank scores it (8 doubles).  The host fills it
 * from the 4x4 pose the reference passes around:
 *   t        = pose[:3, 3]
 *   yaw_r    = math.degrees(math.atan2(pose[0,2], pose[2,2]))      (retrieval,
 *              longctx/inference/landmark_cache.py:27-28)
 *   yaw_e    = np.degrees(np.arctan2(pose[0,2], pose[2,2])) in fp64  (eviction,
 *              longctx/inference/landmark_cache_v2.py:93-94; numpy's arctan2 and
 *              Python's atan2 differ in the last bit for some inputs)
 *   is_f32   = 1.0 when the pose array is float32 (the pipeline's chunk poses,
 *              pipeline/causal_diffusion_inference_compressed.py:374-377): then
 *              retrieval forms the translation difference and its norm in fp32
 *              as numpy does for float32 arrays, else in fp64. */
typedef struct rw_pose {
  double tx, ty, tz, yaw_r, yaw_e, is_f32, pad0, pad1;
} rw_pose_t;

/* Landmark-bank decision state in device memory (written only by rw_bank_step;
 * zero-initialise before the first call).  Capacity RW_BANK_MAX members. */
#define RW_BANK_MAX 1024
typedef struct rw_bank_state {
  int n;          /* members in the bank (list order = admission order minus evictions) */
  int admitted;   /* members ever admitted (drives protect-earliest-n) */
  int pad[2];
  rw_pose_t pose[RW_BANK_MAX];
  int born[RW_BANK_MAX];
  int slot[RW_BANK_MAX];  /* caller's storage slot of the member */
  int prot[RW_BANK_MAX];  /* 1 = protected from eviction */
} rw_bank_state_t;

/* Result of one rw_bank_step (device memory). */
typedef struct rw_bank_result {
  int n_evicted;
  int evicted_born[4];
  int evicted_slot[4];
  int n_bank;          /* bank size after the step */
  int nR;              /* number of retrieved members */
  int pad;
  int R[RW_BANK_MAX];  /* retrieved bank-list indices, ascending */
  int R_slot[RW_BANK_MAX];
} rw_bank_result_t;

/* One bank decision, one launch of a single-CTA kernel, fp64:
 *  (1) when admit != 0: while the bank holds >= K members, evict the member
 *      chosen by landmark_cache_v2.py:465-479 (_evict_index: the first
 *      protect_n admitted are exempt, otherwise the smallest nearest-neighbour
 *      pose distance of _bank_D :90-98, ties evict the later-born), then append
 *      {admit_pose, admit_born, admit_slot} (:481-495 _bank_insert, always-admit);
 *  (2) retrieval (:538-592 _retrieve, plain top-k by pose_dist of
 *      landmark_cache.py:24-31) with warp-level top-k selection: mode 1 ('b') =
 *      the retrieve_k members nearest to *target (exact distance ties: lower
 *      bank index first), returned as ascending bank indices; mode 0 ('a') =
 *      all members.  target may be NULL in mode 0.
 * Poses, state and result live in DEVICE memory. */
int rw_bank_step(rw_bank_state_t* state, int K, int protect_n, int admit, const rw_pose_t* admit_pose,
                 int admit_born, int admit_slot, const rw_pose_t* target, int retrieve_k, int mode,
                 rw_bank_result_t* result, void* stream);

/* Ulysses layout transforms around the all-to-all (wan_5b/distributed/util.py:52-64
 * all_to_all with scatter_dim=2/gather_dim=1 and the inverse; ulysses.py:17-55).
 * pack:   src [B, Ls, H, D] (this rank's sequence shard, all heads) ->
 *         dst [P][B][Ls][H/P][D] (contiguous block per destination rank).
 * unpack: src [P][B][Ls][H/P][D] (block from each source rank = its head group)
 *         -> dst [B, Ls, H, D].
 * bf16 elements, contiguous src/dst. */
int rw_a2a_pack(const void* src, void* dst, int B, int Ls, int H, int D, int P, void* stream);
int rw_a2a_unpack(const void* src, void* dst, int B, int Ls, int H, int D, int P, void* stream);

/* Cross-rank ordering carried by a sequence-parallel kernel itself, in place of a
 * separate barrier launch on each side of an exchange.  sig_ptrs: DEVICE array of
 * P pointers to each rank's int32 signal array (symmetric memory, zeroed before
 * first use).  wait_epoch > 0: before touching data other ranks write, the kernel
 * waits (bounded: RW_STATUS_TIMEOUT_PEER in *status after timeout_ms) until this
 * rank's entries wait_slot .. wait_slot + P - 1 hold at least wait_epoch.
 * signal_epoch > 0: once every CTA of the call has finished, its stores (peer
 * memory included) visible system-wide, the last CTA writes signal_epoch into
 * entry signal_slot + rank of every rank's array; counter is this rank's int32
 * completion counter for the call (DEVICE, zero before its first use; every
 * completed call leaves it at zero again).  Epochs increase from call to call,
 * the same sequence on every rank. */
typedef struct rw_sp_sync {
  const unsigned long long* sig_ptrs;
  int* counter;
  int P, rank;
  int wait_slot, wait_epoch;
  int signal_slot, signal_epoch;
  int timeout_ms, pad;
} rw_sp_sync_t;

/* Ulysses exchanges over peer memory (one sequence, B = 1), the layout
 * transform fused in; q_dst / ck_dst / cv_dst / out_dst are DEVICE arrays of P
 * pointers (this rank's entry is its own buffer, the others are peer-mapped).
 * rw_sp_scatter_qkv: this rank (rank r of P) holds q, k, v [Ls, H, 128] of tokens
 * [r*Ls, (r+1)*Ls); for head h (owner p = h / (H/P), local head hl) and chunk
 * token t = r*Ls + s it writes q to q_dst[p] ([P*Ls, H/P, 128]) row t, RoPE(t)(k)
 * (+ PM-RoPE when given) and v to the caches ck_dst[p] / cv_dst[p]
 * ([cap, H/P, 128]) row dst_start + t.  Replaces the seq->head all_to_all of
 * wan_5b/distributed/ulysses.py:40-42 (util.py:52-64) together with the RoPE and
 * cache write of wan_5b/modules/action_model.py:265-292 on the receiving side.
 * rw_sp_scatter_out: o [P*Ls, H/P, 128] (this rank's heads, whole chunk) ->
 * out_dst[p] ([Ls, H, 128]) rows of rank p, heads [r*H/P, (r+1)*H/P); replaces
 * the head->seq all_to_all of ulysses.py:54.  Cross-rank completion: `sync`
 * (optional, NULL = the caller's barrier) waits before the first store and
 * signals once the call's stores are visible to every rank. */
int rw_sp_scatter_qkv(const void* q, const void* k, const void* v, long long q_sl, long long q_sh, long long k_sl,
                      long long k_sh, long long v_sl, long long v_sh, const unsigned long long* q_dst,
                      const unsigned long long* ck_dst, const unsigned long long* cv_dst, int Ls, int H, int D,
                      int P, int rank, int dst_start, int cap, const rw_rope_t* rope, const rw_sp_sync_t* sync,
                      int* status, void* stream);
int rw_sp_scatter_out(const void* o, const unsigned long long* out_dst, int L, int H, int D, int P, int rank,
                      void* stream);


/* rw_sp_wait: a kernel that only waits (the wait half of *sync), for a stream
 * that must see other ranks' signalled work before it continues, e.g. the
 * consumer of a layer's exchanged output. */
int rw_sp_wait(const rw_sp_sync_t* sync, int* status, void* stream);

/* rw_sp_barrier: stream-ordered barrier of the P ranks of a sequence-parallel
 * group over peer memory.  sig_ptrs: DEVICE array of P pointers to each rank's
 * int32 signal array (symmetric, zero-initialised, at least slot_base + P
 * entries).  Every rank calls it with the same slot_base and a strictly
 * increasing epoch (> 0): rank r writes epoch into entry slot_base + r of every
 * rank's array, after all its earlier work on the stream is visible to the
 * peers, then waits (bounded: RW_STATUS_TIMEOUT_PEER in *status after
 * timeout_ms) until its own entries slot_base .. slot_base + P - 1 hold epoch.
 * Takes the place of the process-group barriers around the exchanges of
 * wan_5b/distributed/ulysses.py:40-54. */
int rw_sp_barrier(const unsigned long long* sig_ptrs, int slot_base, int P, int rank, int epoch, int timeout_ms,
                  int* status, void* stream);

/* rw_sp_attn_fwd: the attention of a sequence-parallel layer on this rank's heads
 * with the head->seq exchange fused into its output: q [Lq, Hp, 128] (the whole
 * chunk, this rank's Hp = H/P heads), k, v [Lk, Hp, 128] (this rank's cache
 * view), element strides per token (sl) and head (sh).  Output row t, local head
 * hl is written straight to out_ptrs[t / (Lq/P)] ([Lq/P, H, 128] bf16 per rank),
 * row t % (Lq/P), head rank*Hp + hl, through peer pointers (DEVICE array of P
 * pointers).  Same attention as rw_attn_fwd (workspace, rope, status alike);
 * replaces the attention call of ulysses.py:44-52 together with the head->seq
 * all_to_all of ulysses.py:54.  Cross-rank completion: `sync` (optional, NULL =
 * the caller's barriers) makes every CTA wait, before its first load, for the
 * ranks' scatters into q / k / v, and signals once every output row (of the
 * merge kernel too, when the key split needs one) has reached its owner. */
int rw_sp_attn_fwd(const void* q, const void* k, const void* v, int Lq, int Lk, int Hp, int D, long long q_sl,
                   long long q_sh, long long k_sl, long long k_sh, long long v_sl, long long v_sh,
                   const unsigned long long* out_ptrs, int P, int rank, int H, float softmax_scale,
                   const rw_rope_t* rope, void* workspace, long long workspace_bytes, const rw_sp_sync_t* sync,
                   int* status, void* stream);

/* Dense bf16 GEMM on CTA pairs (2-SM tcgen05.mma, TMA-fed stages, fp32
 * accumulation in tensor memory):
 *   C[M, N] = A[M, K] B[N, K]^T                       RW_GEMM_EPI_NONE
 *           = A B^T + bias[N]                          RW_GEMM_EPI_BIAS
 *           = gelu_tanh(A B^T + bias)                  RW_GEMM_EPI_BIAS_GELU
 *           = R[M, N] + bf16(A B^T + bias)             RW_GEMM_EPI_BIAS_RESIDUAL
 * i.e. torch.nn.functional.linear(A, B, bias) with B an nn.Linear weight [out,
 * in] (one rounding to bf16; the residual form rounds twice, as torch's bf16
 * `r + linear(x)`; R may alias C).  Replaces the reference's nn.Linear calls
 * around the chunk attention: the q/k/v projections
 * (wan_5b/modules/action_model.py:164-166, as one GEMM over the stacked [3C, C]
 * weight), value_proj with its residual (:203), o + prope_proj (:308-318, one
 * GEMM over [y | P y] and the stacked [C, 2C] weight) and the block's FFN
 * Linear -> GELU(tanh) -> Linear (:547-556).
 * Requirements: bf16 row-major operands with 16-byte aligned bases, row strides
 * (elements) multiples of 8 with lda, ldb >= K, ldc, ldr >= N; K a multiple of
 * 64 and N of 128 (RW_ERR_UNSUPPORTED otherwise); bias (when used) 16-byte
 * aligned.  workspace (device memory, 16-byte aligned, rw_gemm_workspace_bytes()
 * bytes, ZEROED before its first use; each call leaves it ready for the next)
 * lets the tiles of a last, partial round be shared among all CTA pairs by
 * k-blocks, their partial sums meeting in the workspace; with workspace == NULL
 * (or too small) those tiles run whole, same results up to fp32 summation order.
 * Calls that share a workspace must not overlap on the GPU. */
#define RW_GEMM_EPI_NONE 0
#define RW_GEMM_EPI_BIAS 1
#define RW_GEMM_EPI_BIAS_GELU 2
#define RW_GEMM_EPI_BIAS_RESIDUAL 3
int rw_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, const void* bias, const void* R,
                 long long ldr, void* C, long long ldc, int M, int N, int K, int epilogue, void* workspace,
                 long long workspace_bytes, int* status, void* stream);

/* Workspace bytes rw_gemm_bf16 uses for this shape on the current device (0 when
 * the tiles fill whole rounds). */
long long rw_gemm_workspace_bytes(int M, int N, int K);

/* Human-readable text of an RW_ERR_* code. */
const char* rw_error_string(int code);

/* ABI version of this library (incremented on signature changes). */
int rw_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* REWORLD_B200_H */
