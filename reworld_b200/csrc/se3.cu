// rw_se3_block_apply: the PRoPE SE3 transform of a chunk's activations — every
// group of 4 consecutive head-dim channels of token t is multiplied by the 4x4
// matrix of t's frame:  out[b, t, h, 4g + i] = sum_k M[b, t / fs][i][k] * x[b, t, h, 4g + k].
// Replaces _se3_block_apply (wan_5b/modules/action_model.py:84-114: permute, view
// into [B, H, frames, fs, D/4, 4], broadcast 4x4 matmul, permute back), used for
// the V-side P^-1 residual (:194-203) and the O-side P residual (:307-318).  The
// matrices come from the host already in the activation dtype's values (the
// reference casts the context to bf16 and, for P^-1, inverts it in bf16) and
// are passed as fp32; the arithmetic is se3.cuh's (only the order of the 4-term
// sum can differ from the library's).
//
// CTAs of 64 threads walk the tokens (the token's frame matrix is loaded once);
// a thread transforms 16-byte chunks (two groups of 4), their loads issued
// together.  HBM-bound: 2 bytes read
// and 2 bytes written per element.
#include "common.cuh"
#include "host_util.h"
#include "se3.cuh"

namespace rw {
namespace se3 {

struct Params {
  const uint8_t* x;
  uint8_t* out;
  const float* mats;  // [B, frames, 4, 4]
  long long x_sb, x_sl, x_sh, o_sb, o_sl, o_sh;
  int B, L, H, fs, frames;
};

constexpr int THREADS = 64;  // small CTAs, one per token; a thread's 6 chunks (24 heads) unrolled

__global__ void __launch_bounds__(THREADS) se3_kernel(const __grid_constant__ Params p) {
  griddep_launch_dependents();
  griddep_wait();  // launched as a dependent: the previous kernel is done
  const long long tokens = (long long)p.B * p.L;
  const int nch = p.H * 16;  // 16-byte chunks per token
  for (long long tok = blockIdx.x; tok < tokens; tok += gridDim.x) {
    const int b = (int)(tok / p.L);
    const int t = (int)(tok - (long long)b * p.L);
    const int f = t / p.fs;
    float m[16];
    se3_mat(p.mats, p.frames, b, f, m);
    const uint8_t* xr = p.x + 2 * ((long long)b * p.x_sb + (long long)t * p.x_sl);
    uint8_t* orow = p.out + 2 * ((long long)b * p.o_sb + (long long)t * p.o_sl);
#pragma unroll 6
    for (int c = threadIdx.x; c < nch; c += THREADS) {
      const long long h = c >> 4, e = (long long)(c & 15) * 8;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr + 2 * (h * p.x_sh + e)));
      *reinterpret_cast<uint4*>(orow + 2 * (h * p.o_sh + e)) = se3_chunk(m, v);
    }
  }
}

}  // namespace se3
}  // namespace rw

using namespace rw;

extern "C" int rw_se3_block_apply(const void* x, void* out, const float* mats, int B, int L, int H, int D,
                                  int frame_seqlen, long long x_sb, long long x_sl, long long x_sh, long long o_sb,
                                  long long o_sl, long long o_sh, void* stream) {
  if (!x || !out || !mats) return RW_ERR_INVALID_ARG;
  if (D != 128) return RW_ERR_UNSUPPORTED;
  if (B < 1 || L < 0 || H < 1 || frame_seqlen < 1 || L % frame_seqlen != 0) return RW_ERR_INVALID_ARG;
  if (L == 0) return RW_OK;
  if (!aligned16(x) || !aligned16(out) || !aligned16(mats)) return RW_ERR_INVALID_ARG;
  const long long st[6] = {x_sb, x_sl, x_sh, o_sb, o_sl, o_sh};
  for (int i = 0; i < 6; ++i) {
    if ((i == 0 || i == 3) && B == 1) continue;
    if (st[i] < 0 || (st[i] % 8) != 0) return RW_ERR_INVALID_ARG;
  }
  se3::Params p{};
  p.x = (const uint8_t*)x;
  p.out = (uint8_t*)out;
  p.mats = mats;
  p.x_sb = B == 1 ? 0 : x_sb;
  p.x_sl = x_sl;
  p.x_sh = x_sh;
  p.o_sb = B == 1 ? 0 : o_sb;
  p.o_sl = o_sl;
  p.o_sh = o_sh;
  p.B = B;
  p.L = L;
  p.H = H;
  p.fs = frame_seqlen;
  p.frames = L / frame_seqlen;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tokens = (long long)B * L;
  const long long cap = (long long)sms * 20;  // tokens strided over at most 20 CTAs per SM
  const long long grid = tokens < cap ? tokens : cap;
  return launch_dependent(se3::se3_kernel, dim3((unsigned)grid), dim3(se3::THREADS), 0, (cudaStream_t)stream, p) ==
                 cudaSuccess
             ? RW_OK
             : RW_ERR_CUDA;
}
