// The PRoPE SE3 transform of one token's activations, shared by rw_se3_block_apply
// (se3.cu) and the attention output paths (attn_pair.cu epilogue, combine_kernel),
// which can write P y next to y.
//
// Reference: _se3_block_apply (wan_5b/modules/action_model.py:84-114): every group
// of 4 consecutive head-dim channels of token t is multiplied by the 4x4 matrix of
// t's frame, out[b, t, h, 4g + i] = sum_k M[b, t / fs][i][k] * x[b, t, h, 4g + k].
// The matrices arrive in the activation dtype's values, as fp32.  Each output is
// an fp32 sum of the 4 exact bf16 x bf16 products (fused multiply-adds in k order
// from +0) rounded once to bf16, as a bf16 matmul with fp32 accumulation rounds it.
#pragma once

#include "common.cuh"

namespace rw {

// An optional second output of the attention: P y written beside y.
struct Se3Out {
  const float* mats;  // [B, frames, 4, 4] fp32, or null: no second output
  uint8_t* out;       // P y rows, bf16 [B, Lq, H, 128] with the element strides below
  long long sb, sl, sh;
  int fs, frames;     // tokens per frame, frames (Lq = fs * frames)
};

// The 4x4 matrix of frame f of batch element b.
__device__ __forceinline__ void se3_mat(const float* mats, int frames, int b, int f, float (&m)[16]) {
  const float4* mp = reinterpret_cast<const float4*>(mats + ((long long)b * frames + f) * 16);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 r = __ldg(mp + j);
    m[4 * j] = r.x;
    m[4 * j + 1] = r.y;
    m[4 * j + 2] = r.z;
    m[4 * j + 3] = r.w;
  }
}

// One group of 4 channels (two packed bf16 pairs a, b) times m.
__device__ __forceinline__ void se3_group(const float (&m)[16], uint32_t a, uint32_t b, uint32_t& ya,
                                          uint32_t& yb) {
  const float x[4] = {bf16_lo(a), bf16_hi(a), bf16_lo(b), bf16_hi(b)};
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float acc = __fmaf_rn(m[4 * i], x[0], 0.f);  // from +0, like a BLAS accumulator
    acc = __fmaf_rn(m[4 * i + 1], x[1], acc);
    acc = __fmaf_rn(m[4 * i + 2], x[2], acc);
    acc = __fmaf_rn(m[4 * i + 3], x[3], acc);
    y[i] = acc;
  }
  ya = pack_bf16x2(y[0], y[1]);
  yb = pack_bf16x2(y[2], y[3]);
}

// One 16-byte chunk (two groups of 4 channels) times m.
__device__ __forceinline__ uint4 se3_chunk(const float (&m)[16], uint4 v) {
  uint4 o;
  se3_group(m, v.x, v.y, o.x, o.y);
  se3_group(m, v.z, v.w, o.z, o.w);
  return o;
}

}  // namespace rw
