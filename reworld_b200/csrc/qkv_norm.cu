// rw_qkv_norm_rope_store: the step of the cached self-attention between the q/k/v
// projections and the attention, in one kernel.  From the projected rows q, k, v
// ([B, L, C] each, C = H * D) of one chunk, for every token t:
//   q_out[t]               = RMSNorm_q(q[t])                 (q's RoPE is applied
//                                                             inside the attention)
//   cache_k[dst_start + t] = RoPE(t)(RMSNorm_k(k[t]))        (+ PM-RoPE phase if given)
//   cache_v[dst_start + t] = v[t]
// Replaces wan_5b/modules/action_model.py:164-166 (norm_q / norm_k over all heads,
// WanRMSNorm of wan_5b/modules/model.py:73-89) together with the RoPE of k and the
// cache writes of :265-292.  RMSNorm follows the reference's rounding steps: the
// mean of squares in fp32, r = 1 / sqrt(mean + eps), x * r rounded to bf16
// (type_as), then times the bf16 weight and rounded to bf16.  Only the order of
// the fp32 sum (and torch's rsqrt, which is not correctly rounded on the GPU)
// differ from the reference: x * r can land one bf16 unit away, which the weight
// multiply and its rounding can widen to two, in a small fraction of elements.
//
// Work split: a pair of warps per token.  A CTA of 2S warps owns S shared-memory
// stages (6 C bytes each: the token's q, k and v rows); warp pair w processes the
// CTA's tokens w, w + S, w + 2S, ... and owns stage w: its first warp streams each
// token's three rows into the stage with the TMA bulk-copy engine (cp.async.bulk,
// completion on the stage's mbarrier).  Each warp of the pair takes half of the
// row's 16-byte chunks: a first pass over the staged q and k rows gives its part
// of the two sums of squares (warp shuffles), a 64-thread named barrier exchanges
// the parts, a second pass normalises, rotates and stores; after a second pair
// barrier the stage is refilled with the pair's next token.  No block-wide
// barrier, and the per-token work (reduction, 1 / sqrt, RoPE position) is done
// by two warps only.  HBM-bound: 6 C bytes read and 6 C bytes written per token.
#include "common.cuh"
#include "host_util.h"
#include "rope.cuh"

namespace rw {
namespace qkvn {

constexpr int MAX_SLOTS = 10;         // token slots per CTA: 2 warps each, named barriers 1..10
constexpr int STAGE_BUDGET = 221184;  // most bytes of stages per CTA (C = 3072: 10 slots, 180 KB)

struct Params {
  const uint8_t* qi;
  const uint8_t* ki;
  const uint8_t* vi;
  long long qi_sb, qi_sl, ki_sb, ki_sl, vi_sb, vi_sl;  // element strides of [B, L, C] inputs
  const uint8_t* wq;
  const uint8_t* wk;
  float eps_q, eps_k;
  int B, L, C;
  uint8_t* qo;
  long long qo_sb, qo_sl, qo_sh;
  uint8_t* ck;
  long long ck_sb, ck_sl, ck_sh;
  uint8_t* cv;
  long long cv_sb, cv_sl, cv_sh;
  int dst_start;
  int rope_on;
  rw_rope_t rope;
  unsigned long long m_hw, m_w;  // division magics of grid_h * grid_w and grid_w (0: divisor 1)
  int* status;
};

// rope_token with the two divisions by multiply-high.
__device__ __forceinline__ RopeToken rope_token_magic(const Params& p, int token, int b) {
  return rope_token_fast(p.rope, (uint32_t)token, (uint32_t)b, p.m_hw, p.m_w);
}

// A packed bf16 pair widened to an fp32 pair (exact).
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t v) { return f2_pack(bf16_lo(v), bf16_hi(v)); }

// Both halves of a * b rounded once to fp32: a fused multiply-add with a -0
// addend is the plain rounded product (signs of zero included).
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  return ffma2(a, b, f2_pack(-0.f, -0.f));
}

__device__ __forceinline__ uint32_t f2_to_bf16x2(uint64_t v) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  return pack_bf16x2(lo, hi);
}

// y = bf16(bf16(x * r) * w) for the 8 channels of one chunk: x * r in fp32
// rounded to bf16 (type_as), times the bf16 weight as an exact fp32 product
// rounded to bf16 (torch's bf16 multiply).
__device__ __forceinline__ uint4 rmsnorm_chunk(uint4 x, uint4 w, float r) {
  const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  const uint64_t r2 = f2_pack(r, r);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t n = f2_to_bf16x2(fmul2(bf16x2_to_f2(xs[i]), r2));
    o[i] = f2_to_bf16x2(fmul2(bf16x2_to_f2(n), bf16x2_to_f2(ws[i])));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Adds the squares of the 8 channels of one chunk to the fp32 pair acc.
__device__ __forceinline__ uint64_t sumsq_chunk(uint4 x, uint64_t acc) {
  const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t v = bf16x2_to_f2(xs[i]);
    acc = ffma2(v, v, acc);
  }
  return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;  // every lane holds the same bits: each step adds the same two values
}

// Issues the bulk copies of token (b, t)'s q, k and v rows into `stage`.
__device__ __forceinline__ void fetch_token(const Params& p, int b, int t, uint8_t* stage, uint64_t* bar) {
  const uint32_t row = (uint32_t)p.C * 2u;
  mbar_expect_tx(bar, 3u * row);
  bulk_load(stage, p.qi + 2 * ((long long)b * p.qi_sb + (long long)t * p.qi_sl), row, bar);
  bulk_load(stage + row, p.ki + 2 * ((long long)b * p.ki_sb + (long long)t * p.ki_sl), row, bar);
  bulk_load(stage + 2 * row, p.vi + 2 * ((long long)b * p.vi_sb + (long long)t * p.vi_sl), row, bar);
}

// bar.sync on a 64-thread named barrier that also returns whether any
// participating thread passed pred = true.
__device__ __forceinline__ bool pair_bar_or(int id, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 64, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(MAX_SLOTS * 64, 1) qkv_norm_kernel(const __grid_constant__ Params p) {
  griddep_launch_dependents();  // the attention that reads q and these rows may start its prologue now
  griddep_wait();               // launched as a dependent: the previous kernel (the projection) is done
  extern __shared__ __align__(128) uint8_t stage_mem[];
  __shared__ __align__(8) uint64_t full[MAX_SLOTS];
  __shared__ float2 red[MAX_SLOTS][2];  // [slot][half]: (sum q^2, sum k^2) of each warp
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = warp >> 1, half = warp & 1;
  const int S = blockDim.x >> 6;  // token slots = stages
  const int bar_id = 1 + slot;    // named barrier of the pair (0 is __syncthreads)
  const int nch = p.C / 8;        // 16-byte chunks per row
  const long long total = (long long)p.B * p.L;
  const long long mine = (total - blockIdx.x + gridDim.x - 1) / gridDim.x;  // grid <= total: mine >= 1
  uint8_t* stage = stage_mem + (size_t)slot * 6u * (uint32_t)p.C;
  const uint4* st = reinterpret_cast<const uint4*>(stage);
  uint64_t* bar = &full[slot];
  const bool issuer = half == 0 && lane == 0;

  if (half == 0 && lane == 0) mbar_init(bar, 1);
  if (threadIdx.x == 0) abort_flag = 0;
  fence_mbar_init();
  __syncthreads();

  // this pair's tokens: i = slot, slot + S, ...; global token blockIdx.x + i * gridDim.x
  long long i = slot;
  int b = 0, t = 0;
  int fetched = 0;  // bulk-copy rounds issued into this stage (issuer only)
  if (i < mine) {
    const long long idx = blockIdx.x + i * gridDim.x;
    b = (int)(idx / p.L);
    t = (int)(idx - (long long)b * p.L);
    if (issuer) {
      fetch_token(p, b, t, stage, bar);
      fetched = 1;
    }
  }
  const long long step = (long long)S * gridDim.x;  // tokens between this pair's tokens
  const int step_b = (int)(step / p.L), step_t = (int)(step % p.L);
  const uint4* wq = reinterpret_cast<const uint4*>(p.wq);
  const uint4* wk = reinterpret_cast<const uint4*>(p.wk);
  const int ch0 = 32 * half + lane;  // this thread's chunks: ch0, ch0 + 64, ...
  bool aborted = false;
  const int c16 = ch0 & 15;  // every chunk of this thread sits at the same place in its head
  for (int n = 0; i < mine; i += S, ++n) {
    // the 4 RoPE pairs of this thread's chunks (same for all of them), requested
    // before the wait for the rows
    double2 cs[4];
    const float2* dlp = nullptr;  // PM-RoPE factors of the same pairs (read after the exchange)
    bool rot = false;
    if (p.rope_on) {
      const RopeToken rt = rope_token_magic(p, t, b);
      rot = rt.on;
      dlp = rt.dl != nullptr ? rt.dl + 4 * c16 : nullptr;
#pragma unroll
      for (int j = 0; j < 4; ++j) cs[j] = rope_freq(4 * c16 + j, rt);
    }
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar, (uint32_t)(n & 1), &abort_flag, p.status,
                                                      RW_STATUS_TIMEOUT_COPY));
    // pass 1: this warp's part of the sums of squares of the q and k rows
    uint64_t aq = f2_pack(0.f, 0.f), ak = aq;
    if (ok) {
#pragma unroll 3
      for (int ch = ch0; ch < nch; ch += 64) {
        aq = sumsq_chunk(st[ch], aq);
        ak = sumsq_chunk(st[nch + ch], ak);
      }
    }
    float q0, q1, k0, k1;
    f2_unpack(aq, q0, q1);
    f2_unpack(ak, k0, k1);
    const float pq = warp_sum(q0 + q1), pk = warp_sum(k0 + k1);
    if (lane == 0) red[slot][half] = make_float2(pq, pk);
    if (pair_bar_or(bar_id, !ok)) {  // both warps of the pair leave together
      aborted = true;
      break;
    }
    const bool has_d = dlp != nullptr;
    float2 dl[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) dl[j] = has_d ? dlp[j] : make_float2(0.f, 0.f);
    const float2 r0 = red[slot][0], r1 = red[slot][1];  // same order in both warps
    const float rq = 1.0f / sqrtf((r0.x + r1.x) / (float)p.C + p.eps_q);
    const float rk = 1.0f / sqrtf((r0.y + r1.y) / (float)p.C + p.eps_k);
    // pass 2: normalise, rotate k, store q, the cache rows of k and v
    const long long qo_row = (long long)b * p.qo_sb + (long long)t * p.qo_sl;
    const long long ck_row = (long long)b * p.ck_sb + ((long long)p.dst_start + t) * p.ck_sl;
    const long long cv_row = (long long)b * p.cv_sb + ((long long)p.dst_start + t) * p.cv_sl;
#pragma unroll 2
    for (int ch = ch0; ch < nch; ch += 64) {
      const int h = ch >> 4;  // head
      const long long e = (long long)c16 * 8;
      const uint4 qn = rmsnorm_chunk(st[ch], __ldg(wq + ch), rq);
      uint4 kn = rmsnorm_chunk(st[nch + ch], __ldg(wk + ch), rk);
      if (rot) {
        kn.x = rope_rotate(kn.x, cs[0], has_d, dl[0]);
        kn.y = rope_rotate(kn.y, cs[1], has_d, dl[1]);
        kn.z = rope_rotate(kn.z, cs[2], has_d, dl[2]);
        kn.w = rope_rotate(kn.w, cs[3], has_d, dl[3]);
      }
      *reinterpret_cast<uint4*>(p.qo + 2 * (qo_row + h * p.qo_sh + e)) = qn;
      *reinterpret_cast<uint4*>(p.ck + 2 * (ck_row + h * p.ck_sh + e)) = kn;
      *reinterpret_cast<uint4*>(p.cv + 2 * (cv_row + h * p.cv_sh + e)) = st[2 * nch + ch];
    }
    // the pair's next token, fetched into the stage both warps have finished reading
    t += step_t;
    b += step_b;
    if (t >= p.L) {
      t -= p.L;
      ++b;
    }
    named_bar_sync(bar_id, 64);
    if (i + S < mine && issuer) {
      fence_proxy_async_smem();
      fetch_token(p, b, t, stage, bar);
      ++fetched;
    }
  }
  if (aborted && issuer && fetched > 0) {
    // the last round issued into this stage may still be landing: wait for it
    // (bounded) before the CTA's shared memory can be released
    mbar_wait_drain(bar, (uint32_t)((fetched - 1) & 1));
  }
}

}  // namespace qkvn
}  // namespace rw

using namespace rw;

extern "C" int rw_qkv_norm_rope_store(const void* q_in, const void* k_in, const void* v_in, const void* w_q,
                                      const void* w_k, void* q_out, void* cache_k, void* cache_v, int B, int L,
                                      int H, int D, int dst_start, float eps_q, float eps_k, long long qi_sb,
                                      long long qi_sl, long long ki_sb, long long ki_sl, long long vi_sb,
                                      long long vi_sl, long long qo_sb, long long qo_sl, long long qo_sh,
                                      long long ck_sb, long long ck_sl, long long ck_sh, long long cv_sb,
                                      long long cv_sl, long long cv_sh, const rw_rope_t* rope, int* status,
                                      void* stream) {
  if (!q_in || !k_in || !v_in || !w_q || !w_k || !q_out || !cache_k || !cache_v) return RW_ERR_INVALID_ARG;
  if (D != 128) return RW_ERR_UNSUPPORTED;
  if (B < 1 || B > 65535 || L < 0 || H < 1 || dst_start < 0 || !(eps_q >= 0.f) || !(eps_k >= 0.f))
    return RW_ERR_INVALID_ARG;
  if ((long long)H * D * 6 > qkvn::STAGE_BUDGET) return RW_ERR_UNSUPPORTED;  // one stage: C <= 36864
  const int C = H * D;
  if (L == 0) return RW_OK;
  const void* ptrs[8] = {q_in, k_in, v_in, w_q, w_k, q_out, cache_k, cache_v};
  for (int i = 0; i < 8; ++i)
    if (!aligned16(ptrs[i])) return RW_ERR_INVALID_ARG;
  // every stride in elements, a multiple of 8 (16 bytes); batch strides are unused when B == 1
  const long long st[15] = {qi_sb, qi_sl, ki_sb, ki_sl, vi_sb, vi_sl, qo_sb, qo_sl,
                            qo_sh, ck_sb, ck_sl, ck_sh, cv_sb, cv_sl, cv_sh};
  const bool is_batch[15] = {1, 0, 1, 0, 1, 0, 1, 0, 0, 1, 0, 0, 1, 0, 0};
  for (int i = 0; i < 15; ++i) {
    if (is_batch[i] && B == 1) continue;
    if (st[i] < 0 || (st[i] % 8) != 0) return RW_ERR_INVALID_ARG;
  }
  qkvn::Params p{};
  p.qi = (const uint8_t*)q_in;
  p.ki = (const uint8_t*)k_in;
  p.vi = (const uint8_t*)v_in;
  p.qi_sb = B == 1 ? 0 : qi_sb;
  p.ki_sb = B == 1 ? 0 : ki_sb;
  p.vi_sb = B == 1 ? 0 : vi_sb;
  p.qi_sl = qi_sl;
  p.ki_sl = ki_sl;
  p.vi_sl = vi_sl;
  p.wq = (const uint8_t*)w_q;
  p.wk = (const uint8_t*)w_k;
  p.eps_q = eps_q;
  p.eps_k = eps_k;
  p.B = B;
  p.L = L;
  p.C = C;
  p.qo = (uint8_t*)q_out;
  p.qo_sb = B == 1 ? 0 : qo_sb;
  p.qo_sl = qo_sl;
  p.qo_sh = qo_sh;
  p.ck = (uint8_t*)cache_k;
  p.ck_sb = B == 1 ? 0 : ck_sb;
  p.ck_sl = ck_sl;
  p.ck_sh = ck_sh;
  p.cv = (uint8_t*)cache_v;
  p.cv_sb = B == 1 ? 0 : cv_sb;
  p.cv_sl = cv_sl;
  p.cv_sh = cv_sh;
  p.dst_start = dst_start;
  p.status = status;
  if (rope != nullptr) {
    if (!rope_args_ok(*rope, D)) return RW_ERR_INVALID_ARG;
    p.rope = *rope;
    p.rope_on = 1;
  }
  if (rope != nullptr) {
    p.m_hw = div_magic_of((unsigned long long)rope->grid_h * rope->grid_w);
    p.m_w = div_magic_of((unsigned long long)rope->grid_w);
  }
  const int stage_bytes = 6 * C;
  int slots = qkvn::STAGE_BUDGET / stage_bytes;  // one stage per token slot (warp pair)
  if (slots > qkvn::MAX_SLOTS) slots = qkvn::MAX_SLOTS;
  const int smem = slots * stage_bytes;
  static std::atomic<unsigned long long> attr_done{0};
  if (!ensure_smem_attr((const void*)qkvn::qkv_norm_kernel, qkvn::STAGE_BUDGET, &attr_done)) return RW_ERR_CUDA;
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qkvn::qkv_norm_kernel, slots * 64, smem) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const long long total = (long long)B * L;
  const long long grid = total < (long long)sms * per_sm ? total : (long long)sms * per_sm;
  return launch_dependent(qkvn::qkv_norm_kernel, dim3((unsigned)grid), dim3(slots * 64), (size_t)smem,
                          (cudaStream_t)stream, p) == cudaSuccess
             ? RW_OK
             : RW_ERR_CUDA;
}
