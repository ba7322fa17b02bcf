// rw_row_norm: the DiT block's row normalisations on bf16 rows of C channels.
//   mode RW_NORM_RMS   y = bf16(bf16(x * r) * w),  r = 1 / sqrt(mean(x^2) + eps)
//                      (WanRMSNorm, wan_5b/modules/model.py:73-89: fp32 statistics,
//                       type_as, bf16 weight product), used for the cross-attention's
//                       norm_q (model.py:175, causal_model.py:218)
//   mode RW_NORM_LAYER y = bf16((x - mean) * rstd [* w + b]),  rstd = 1 / sqrt(var + eps)
//                      (WanLayerNorm, model.py:92-102: torch layer_norm, statistics and
//                       affine in fp32, one rounding), used for norm2 / norm3 of the block
//                       (action_model.py:399-403, 547-553); w, b optional (affine off).
// One 128-thread CTA per row: each thread keeps its chunks of the row in
// registers, so the row is read once; block reductions give the statistics.
// The fp32 sums run in another order than torch's, so an output can differ from
// it by a bf16 unit (two where a unit before the weight product, or before an
// affine that cancels, widens after it).  HBM-bound: 2 C bytes read and
// 2 C bytes written per row.
#include "common.cuh"
#include "host_util.h"

namespace rw {
namespace rown {

struct Params {
  const uint8_t* x;
  uint8_t* out;
  const uint8_t* w;  // bf16 [C] or null
  const uint8_t* b;  // bf16 [C] or null (layer mode)
  long long rows, x_rs, o_rs;  // element strides between rows
  int C, mode;
  float eps;
};

constexpr int THREADS = 128;    // one CTA per row
constexpr int MAX_PER = 8;      // 16-byte chunks per thread: C <= 8 * 8 * 128 = 8192 (PER = 3: C <= 3072)

// Sum over the CTA; every thread gets the same bits (one fixed order of the
// per-warp partials).
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5;
  __syncthreads();  // the previous use of red is finished
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  return (red[0] + red[1]) + (red[2] + red[3]);
}

template <int PER>
__global__ void __launch_bounds__(THREADS) row_norm_kernel(const __grid_constant__ Params p) {
  griddep_launch_dependents();
  griddep_wait();  // launched as a dependent: the previous kernel is done
  __shared__ float red[THREADS / 32];
  const int nch = p.C / 8;
  const uint4* wv = reinterpret_cast<const uint4*>(p.w);
  const uint4* bv = reinterpret_cast<const uint4*>(p.b);
  for (long long row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(p.x + 2 * row * p.x_rs);
    uint4* orow = reinterpret_cast<uint4*>(p.out + 2 * row * p.o_rs);
    // the row is read once: this thread's chunks c = threadIdx.x + 128 k stay in registers
    uint4 v[PER];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int c = threadIdx.x + THREADS * k;
      v[k] = c < nch ? __ldg(xr + c) : make_uint4(0, 0, 0, 0);
      const uint32_t xs[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = bf16_lo(xs[i]), b = bf16_hi(xs[i]);
        if (p.mode == RW_NORM_RMS) {
          s = __fmaf_rn(a, a, s);
          s = __fmaf_rn(b, b, s);
        } else {
          s += a;
          s += b;
        }
      }
    }
    s = block_sum(s, red);
    float scale, shift = 0.f;  // y = x * scale + shift (before the affine / weight)
    if (p.mode == RW_NORM_RMS) {
      scale = 1.0f / sqrtf(s / (float)p.C + p.eps);
    } else {
      const float mean = s / (float)p.C;
      // variance about the mean (two-pass, population variance as layer_norm)
      float q = 0.f;
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        if (threadIdx.x + THREADS * k >= nch) continue;
        const uint32_t xs[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float a = bf16_lo(xs[i]) - mean, b = bf16_hi(xs[i]) - mean;
          q = __fmaf_rn(a, a, q);
          q = __fmaf_rn(b, b, q);
        }
      }
      q = block_sum(q, red);
      scale = 1.0f / sqrtf(q / (float)p.C + p.eps);
      shift = -mean * scale;
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int c = threadIdx.x + THREADS * k;
      if (c >= nch) continue;
      const uint32_t xs[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
      uint32_t ws[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};  // bf16 1.0 pairs
      uint32_t bs[4] = {0u, 0u, 0u, 0u};
      if (wv != nullptr) {
        const uint4 t = __ldg(wv + c);
        ws[0] = t.x, ws[1] = t.y, ws[2] = t.z, ws[3] = t.w;
      }
      if (bv != nullptr) {
        const uint4 t = __ldg(bv + c);
        bs[0] = t.x, bs[1] = t.y, bs[2] = t.z, bs[3] = t.w;
      }
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float y0, y1;
        if (p.mode == RW_NORM_RMS) {
          // bf16(bf16(x * r) * w)
          const uint32_t n = pack_bf16x2(__fmul_rn(bf16_lo(xs[i]), scale), __fmul_rn(bf16_hi(xs[i]), scale));
          y0 = __fmul_rn(bf16_lo(n), bf16_lo(ws[i]));
          y1 = __fmul_rn(bf16_hi(n), bf16_hi(ws[i]));
        } else {
          // (x - mean) * rstd, then the affine, in fp32
          y0 = __fmaf_rn(bf16_lo(xs[i]), scale, shift);
          y1 = __fmaf_rn(bf16_hi(xs[i]), scale, shift);
          if (wv != nullptr) {
            y0 = __fmaf_rn(y0, bf16_lo(ws[i]), bf16_lo(bs[i]));
            y1 = __fmaf_rn(y1, bf16_hi(ws[i]), bf16_hi(bs[i]));
          }
        }
        o[i] = pack_bf16x2(y0, y1);
      }
      orow[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

}  // namespace rown
}  // namespace rw

using namespace rw;

extern "C" int rw_row_norm(const void* x, void* out, const void* w, const void* b, long long rows, int C,
                           long long x_row_stride, long long out_row_stride, float eps, int mode, void* stream) {
  if (!x || !out) return RW_ERR_INVALID_ARG;
  if (mode != RW_NORM_RMS && mode != RW_NORM_LAYER) return RW_ERR_INVALID_ARG;
  if (mode == RW_NORM_RMS && w == nullptr) return RW_ERR_INVALID_ARG;
  if (b != nullptr && w == nullptr) return RW_ERR_INVALID_ARG;
  if (rows < 0 || C < 8 || C % 8 != 0 || !(eps >= 0.f)) return RW_ERR_INVALID_ARG;
  if (C > 8 * rown::MAX_PER * rown::THREADS) return RW_ERR_UNSUPPORTED;
  if (rows == 0) return RW_OK;
  if (!aligned16(x) || !aligned16(out) || (w && !aligned16(w)) || (b && !aligned16(b))) return RW_ERR_INVALID_ARG;
  if (x_row_stride < C || out_row_stride < C || x_row_stride % 8 != 0 || out_row_stride % 8 != 0)
    return RW_ERR_INVALID_ARG;
  rown::Params p{};
  p.x = (const uint8_t*)x;
  p.out = (uint8_t*)out;
  p.w = (const uint8_t*)w;
  p.b = (const uint8_t*)b;
  p.rows = rows;
  p.x_rs = x_row_stride;
  p.o_rs = out_row_stride;
  p.C = C;
  p.mode = mode;
  p.eps = eps;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long cap = (long long)sms * 16;  // 16 resident CTAs per SM, rows strided over them
  const long long grid = rows < cap ? rows : cap;
  const cudaError_t e =
      C <= 8 * 3 * rown::THREADS
          ? launch_dependent(rown::row_norm_kernel<3>, dim3((unsigned)grid), dim3(rown::THREADS), 0,
                             (cudaStream_t)stream, p)
          : launch_dependent(rown::row_norm_kernel<rown::MAX_PER>, dim3((unsigned)grid), dim3(rown::THREADS), 0,
                             (cudaStream_t)stream, p);
  return e == cudaSuccess ? RW_OK : RW_ERR_CUDA;
}
