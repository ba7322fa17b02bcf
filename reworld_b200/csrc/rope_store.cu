// RoPE (+ PM-RoPE phase) on the new chunk's K and the KV-cache write of K and V.
//
// Replaces wan_5b/modules/action_model.py:265-292: q_f, k_f = apply_rope(q, k,
// delta_tok, start_f=g_start_f, ...) followed by
// kv_cache["k"][:, local_start:local_end] = k_f and kv_cache["v"][...] = v.
// CTAs walk the tokens; a thread moves 16-byte chunks (8 bf16 = 4 complex
// pairs) of the token's head rows; V is a plain 16-byte copy.  HBM-bound: reads
// k, v (and q), writes the cache rows (and roped q).
#include "common.cuh"
#include "host_util.h"
#include "rope.cuh"

namespace rw {
namespace store {

struct Params {
  const uint8_t* k;
  const uint8_t* v;
  const uint8_t* q_in;
  uint8_t* q_out;
  uint8_t* ck;
  uint8_t* cv;
  int B, L, H, dst_start;
  // strides in bytes
  long long k_sb, k_sl, k_sh, v_sb, v_sl, v_sh, q_sb, q_sl, q_sh, qo_sb, qo_sl, qo_sh;
  long long ck_sb, ck_sl, ck_sh, cv_sb, cv_sl, cv_sh;
  int rope_on;
  rw_rope_t rope;
  unsigned long long m_L, m_hw, m_w;  // division magics of L, grid_h * grid_w and grid_w
};

__device__ __forceinline__ uint4 ldg16(const uint8_t* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void stg16(uint8_t* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

constexpr int THREADS = 128;         // a multiple of 16: a thread's chunks all sit at one place in their head
constexpr int HSTEP = THREADS / 16;  // heads between two chunks of a thread
constexpr int NB = 3;                // chunks per thread and batch (24 heads: one batch)

// The 4 RoPE pairs of chunk position c16 of the token (same for every head).
struct RopeRegs {
  double2 cs[4];
  float2 dl[4];
  bool rot, has_d;
};

__device__ __forceinline__ void rope_regs(const Params& p, uint32_t t, uint32_t b, int c16, RopeRegs& r) {
  const RopeToken rt = rope_token_fast(p.rope, t, b, p.m_hw, p.m_w);
  r.rot = rt.on;
  r.has_d = rt.dl != nullptr;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    r.cs[j] = rope_freq(4 * c16 + j, rt);
    r.dl[j] = r.has_d ? rt.dl[4 * c16 + j] : make_float2(0.f, 0.f);
  }
}

__device__ __forceinline__ uint4 rotate(uint4 v, const RopeRegs& r) {
  v.x = rope_rotate(v.x, r.cs[0], r.has_d, r.dl[0]);
  v.y = rope_rotate(v.y, r.cs[1], r.has_d, r.dl[1]);
  v.z = rope_rotate(v.z, r.cs[2], r.has_d, r.dl[2]);
  v.w = rope_rotate(v.w, r.cs[3], r.has_d, r.dl[3]);
  return v;
}

// CTAs walk the tokens (b, t); thread x handles the 16-byte chunk c16 = x mod 16
// of heads x / 16, x / 16 + 8, ..., so the token's position and the thread's 4
// RoPE table entries are looked up once per token, and its row addresses once per
// token (then one add per head).  The loads of a batch of NB heads are all issued
// before the batch's first store, so one round trip to memory covers them.
__global__ void __launch_bounds__(THREADS, 4) rope_kv_store_kernel(const __grid_constant__ Params p) {
  griddep_launch_dependents();  // the attention that reads these rows may start its prologue now
  griddep_wait();               // launched as a dependent: the previous kernel is done
  const uint32_t tokens = (uint32_t)p.B * (uint32_t)p.L;  // < 2^31 (host check)
  const int c16 = threadIdx.x & 15;
  const int h0 = threadIdx.x >> 4;
  const long long e = 16LL * c16;  // byte offset of the chunk within the head row
  const bool with_q = p.q_in != nullptr;
  for (uint32_t tok = blockIdx.x; tok < tokens; tok += gridDim.x) {
    const uint32_t b = div_magic(tok, p.m_L);
    const uint32_t t = tok - b * (uint32_t)p.L;
    const uint32_t td = (uint32_t)p.dst_start + t;
    const uint8_t* kp = p.k + b * p.k_sb + t * p.k_sl + e;
    const uint8_t* vp = p.v + b * p.v_sb + t * p.v_sl + e;
    uint8_t* ckp = p.ck + b * p.ck_sb + td * p.ck_sl + e;
    uint8_t* cvp = p.cv + b * p.cv_sb + td * p.cv_sl + e;
    const uint8_t* qp = with_q ? p.q_in + b * p.q_sb + t * p.q_sl + e : nullptr;
    uint8_t* qop = with_q ? p.q_out + b * p.qo_sb + t * p.qo_sl + e : nullptr;
    for (int hb = h0; hb < p.H; hb += HSTEP * NB) {
      uint4 kv[NB], vv[NB], qv[NB];
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const long long h = hb + j * HSTEP;
        if (h < p.H) {
          vv[j] = ldg16(vp + h * p.v_sh);
          kv[j] = ldg16(kp + h * p.k_sh);
          if (with_q) qv[j] = ldg16(qp + h * p.q_sh);
        }
      }
      RopeRegs r;
      r.rot = false;
      if (p.rope_on) rope_regs(p, t, b, c16, r);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const long long h = hb + j * HSTEP;
        if (h < p.H) {
          // V: plain copy into the cache slot; K: rotated into the cache slot
          stg16(cvp + h * p.cv_sh, vv[j]);
          stg16(ckp + h * p.ck_sh, r.rot ? rotate(kv[j], r) : kv[j]);
          // Q: optional rotated copy
          if (with_q) stg16(qop + h * p.qo_sh, r.rot ? rotate(qv[j], r) : qv[j]);
        }
      }
    }
  }
}

}  // namespace store
}  // namespace rw

using namespace rw;

extern "C" int rw_rope_kv_store(const void* k, const void* v, const void* q_in, void* q_out, void* cache_k,
                                void* cache_v, int B, int L, int H, int D, int dst_start, long long k_sb,
                                long long k_sl, long long k_sh, long long v_sb, long long v_sl, long long v_sh,
                                long long q_sb, long long q_sl, long long q_sh, long long qo_sb, long long qo_sl,
                                long long qo_sh, long long ck_sb, long long ck_sl, long long ck_sh,
                                long long cv_sb, long long cv_sl, long long cv_sh, const rw_rope_t* rope,
                                void* stream) {
  if (!k || !v || !cache_k || !cache_v) return RW_ERR_INVALID_ARG;
  if ((q_in == nullptr) != (q_out == nullptr)) return RW_ERR_INVALID_ARG;
  if (D != 128) return RW_ERR_UNSUPPORTED;
  if (B < 1 || B > 65535 || L < 0 || H < 1 || dst_start < 0) return RW_ERR_INVALID_ARG;
  if (L == 0) return RW_OK;
  const void* ptrs[6] = {k, v, q_in, q_out, cache_k, cache_v};
  for (int i = 0; i < 6; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return RW_ERR_INVALID_ARG;
  const long long st[18] = {k_sb, k_sl, k_sh, v_sb, v_sl, v_sh, q_sb, q_sl, q_sh,
                            qo_sb, qo_sl, qo_sh, ck_sb, ck_sl, ck_sh, cv_sb, cv_sl, cv_sh};
  for (int i = 0; i < 18; ++i) {
    if (i >= 6 && i < 12 && q_in == nullptr) continue;
    if ((i % 3) == 0 && B == 1) continue;
    if (st[i] < 0 || (st[i] % 8) != 0) return RW_ERR_INVALID_ARG;
  }
  if ((long long)B * L >= (1LL << 31)) return RW_ERR_UNSUPPORTED;
  store::Params p{};
  p.k = (const uint8_t*)k;
  p.v = (const uint8_t*)v;
  p.q_in = (const uint8_t*)q_in;
  p.q_out = (uint8_t*)q_out;
  p.ck = (uint8_t*)cache_k;
  p.cv = (uint8_t*)cache_v;
  p.L = L;
  p.H = H;
  p.dst_start = dst_start;
  // element strides -> byte strides (batch strides unused when B == 1)
  const auto bs = [B](long long s) { return B == 1 ? 0LL : 2 * s; };
  p.k_sb = bs(k_sb); p.k_sl = 2 * k_sl; p.k_sh = 2 * k_sh;
  p.v_sb = bs(v_sb); p.v_sl = 2 * v_sl; p.v_sh = 2 * v_sh;
  p.q_sb = bs(q_sb); p.q_sl = 2 * q_sl; p.q_sh = 2 * q_sh;
  p.qo_sb = bs(qo_sb); p.qo_sl = 2 * qo_sl; p.qo_sh = 2 * qo_sh;
  p.ck_sb = bs(ck_sb); p.ck_sl = 2 * ck_sl; p.ck_sh = 2 * ck_sh;
  p.cv_sb = bs(cv_sb); p.cv_sl = 2 * cv_sl; p.cv_sh = 2 * cv_sh;
  p.rope_on = 0;
  if (rope != nullptr) {
    if (!rope_args_ok(*rope, D)) return RW_ERR_INVALID_ARG;
    p.rope = *rope;
    p.rope_on = 1;
    p.m_hw = div_magic_of((unsigned long long)rope->grid_h * rope->grid_w);
    p.m_w = div_magic_of((unsigned long long)rope->grid_w);
  }
  p.B = B;
  p.m_L = div_magic_of((unsigned long long)L);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tokens = (long long)B * L;
  const long long cap = (long long)sms * 16;  // resident 128-thread CTAs, tokens strided over them
  const long long grid = tokens < cap ? tokens : cap;
  return launch_dependent(store::rope_kv_store_kernel, dim3((unsigned)grid), dim3(store::THREADS), 0,
                          (cudaStream_t)stream, p) == cudaSuccess
             ? RW_OK
             : RW_ERR_CUDA;
}
