// 3-D RoPE (+ PM-RoPE phase) arithmetic shared by the attention prologue and
// the cache-store kernel.
//
// Reference: causal_rope_apply (wan_5b/modules/causal_model.py:156-184) rotates
// complex pair j of token t by freqs[start_frame + f][j] (j < c_t),
// freqs[h][j] (c_t <= j < c_t + c_h) or freqs[w][j] (otherwise), with
// (f, h, w) the token's grid position, as a complex128 product, then casts to
// bf16 (.type_as); pm_rope_delta_apply (action_model.py:40-51) then multiplies
// by e^{i delta} in complex64 and casts to bf16 again.  The complex products
// use separately rounded multiplies and adds (no fused multiply-add), the
// double -> bf16 cast rounds through fp32, as the reference's CPU kernels do.
#pragma once

#include "common.cuh"

namespace rw {

struct RopeToken {
  const double2* ft;  // freqs row of the temporal position
  const double2* fh;  // freqs row of the height position
  const double2* fw;  // freqs row of the width position
  const float2* dl;   // PM-RoPE (cos, sin) row of the frame, or null
  int e_t, e_h;       // pair index where the h and w sections start
  bool on;            // false: token is past f*h*w and stays unchanged
};

__device__ __forceinline__ RopeToken rope_token(const rw_rope_t& rp, int token, int b) {
  RopeToken rt;
  const int hw = rp.grid_h * rp.grid_w;
  rt.on = token < rp.grid_f * hw;
  const int tok = rt.on ? token : 0;
  const int f = tok / hw;
  const int rem = tok - f * hw;
  const int hh = rem / rp.grid_w;
  const int ww = rem - hh * rp.grid_w;
  const double2* tab = reinterpret_cast<const double2*>(rp.freqs);
  rt.ft = tab + (size_t)(rp.start_frame + f) * 64;
  rt.fh = tab + (size_t)hh * 64;
  rt.fw = tab + (size_t)ww * 64;
  rt.dl = rp.delta_cs ? reinterpret_cast<const float2*>(rp.delta_cs) + ((size_t)b * rp.grid_f + f) * 64 : nullptr;
  rt.e_t = rp.c_t;
  rt.e_h = rp.c_t + rp.c_h;
  return rt;
}

// floor(n / d) from m = floor((2^64 - 1) / d) + 1 (d >= 2): n * m / 2^64 exceeds
// n / d by less than n / 2^64 < 1 / d, so the floor is exact for every 32-bit n.
// m == 0 stands for d == 1.
__device__ __forceinline__ uint32_t div_magic(uint32_t n, unsigned long long m) {
  return m == 0 ? n : (uint32_t)__umul64hi((unsigned long long)n, m);
}
inline unsigned long long div_magic_of(unsigned long long d) { return d >= 2 ? ~0ull / d + 1 : 0; }

// rope_token with the two divisions by multiply-high: m_hw = div_magic_of(grid_h *
// grid_w), m_w = div_magic_of(grid_w).
__device__ __forceinline__ RopeToken rope_token_fast(const rw_rope_t& rp, uint32_t token, uint32_t b,
                                                     unsigned long long m_hw, unsigned long long m_w) {
  RopeToken rt;
  const uint32_t hw = (uint32_t)(rp.grid_h * rp.grid_w);
  rt.on = token < (uint32_t)rp.grid_f * hw;
  const uint32_t tok = rt.on ? token : 0u;
  const uint32_t f = div_magic(tok, m_hw);
  const uint32_t rem = tok - f * hw;
  const uint32_t hh = div_magic(rem, m_w);
  const uint32_t ww = rem - hh * (uint32_t)rp.grid_w;
  const double2* tab = reinterpret_cast<const double2*>(rp.freqs);
  rt.ft = tab + (size_t)(rp.start_frame + f) * 64;
  rt.fh = tab + (size_t)hh * 64;
  rt.fw = tab + (size_t)ww * 64;
  rt.dl = rp.delta_cs ? reinterpret_cast<const float2*>(rp.delta_cs) + ((size_t)b * rp.grid_f + f) * 64 : nullptr;
  rt.e_t = rp.c_t;
  rt.e_h = rp.c_t + rp.c_h;
  return rt;
}

// The freqs entry of complex pair j of the token.
__device__ __forceinline__ double2 rope_freq(int j, const RopeToken& rt) {
  return (j < rt.e_t) ? rt.ft[j] : ((j < rt.e_h) ? rt.fh[j] : rt.fw[j]);
}

// Rotates one packed bf16 pair (low half = real, high half = imaginary) by the
// freqs entry cs, then, when has_d, by the PM-RoPE factor d = (cos, sin).
__device__ __forceinline__ uint32_t rope_rotate(uint32_t w, double2 cs, bool has_d, float2 d) {
  const double xr = (double)bf16_lo(w);
  const double xi = (double)bf16_hi(w);
  const double yr = __dsub_rn(__dmul_rn(xr, cs.x), __dmul_rn(xi, cs.y));
  const double yi = __dadd_rn(__dmul_rn(xr, cs.y), __dmul_rn(xi, cs.x));
  uint32_t o = pack_bf16x2(__double2float_rn(yr), __double2float_rn(yi));
  if (has_d) {
    const float ar = bf16_lo(o), ai = bf16_hi(o);
    const float zr = __fsub_rn(__fmul_rn(ar, d.x), __fmul_rn(ai, d.y));
    const float zi = __fadd_rn(__fmul_rn(ar, d.y), __fmul_rn(ai, d.x));
    o = pack_bf16x2(zr, zi);
  }
  return o;
}

// Rotates one packed bf16 pair that is complex pair j of the token.
__device__ __forceinline__ uint32_t rope_pair(uint32_t w, int j, const RopeToken& rt) {
  const bool has_d = rt.dl != nullptr;
  return rope_rotate(w, rope_freq(j, rt), has_d, has_d ? rt.dl[j] : make_float2(0.f, 0.f));
}

// Rotates 4 consecutive pairs (one 16-byte chunk: elements 8*c16 .. 8*c16+7).
__device__ __forceinline__ uint4 rope_chunk(uint4 v, int c16, const RopeToken& rt) {
  if (!rt.on) return v;
  v.x = rope_pair(v.x, 4 * c16 + 0, rt);
  v.y = rope_pair(v.y, 4 * c16 + 1, rt);
  v.z = rope_pair(v.z, 4 * c16 + 2, rt);
  v.w = rope_pair(v.w, 4 * c16 + 3, rt);
  return v;
}

// Host-side validation of a rope descriptor for head_dim D.
inline bool rope_args_ok(const rw_rope_t& r, int D) {
  return r.freqs != nullptr && r.c_t >= 0 && r.c_h >= 0 && r.c_w >= 0 && r.c_t + r.c_h + r.c_w == D / 2 &&
         r.grid_f >= 1 && r.grid_h >= 1 && r.grid_w >= 1 && r.start_frame >= 0 &&
         r.start_frame + r.grid_f <= r.max_pos && r.grid_h <= r.max_pos && r.grid_w <= r.max_pos &&
         (reinterpret_cast<uintptr_t>(r.freqs) & 15u) == 0 && (reinterpret_cast<uintptr_t>(r.delta_cs) & 7u) == 0;
}

}  // namespace rw
