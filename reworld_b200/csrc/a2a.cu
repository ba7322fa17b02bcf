// Ulysses sequence-parallel layout transforms around the all-to-all.
//
// Reference: wan_5b/distributed/util.py:52-64 all_to_all(x, scatter_dim,
// gather_dim) chunks x along the head dim (scatter_dim=2), makes each chunk
// contiguous, exchanges them with dist.all_to_all and concatenates the
// received chunks along the sequence (gather_dim=1); the inverse after the
// attention scatters the sequence and gathers heads (ulysses.py:40-54).
//
// Here the exchange itself is one all_to_all_single over a contiguous buffer:
//   pack   [B, Ls, H, D] -> [P][B][Ls][H/P][D]   (block p goes to rank p)
//   unpack [P][B][Ls][H/P][D] -> [B, Ls, H, D]   (block p came from rank p)
// With B = 1 the received buffer of the seq->head exchange, [P][Ls][H/P][D], is
// already the gathered [L, H/P, D] layout, and the send buffer of the
// head->seq exchange needs no packing, so only one transform runs per side.
// 16-byte vectorised, HBM-bound.
#include "common.cuh"

namespace rw {
namespace a2a {

// index math on 16-byte chunks (8 bf16); D multiple of 8
__global__ void __launch_bounds__(256)
    pack_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int B, int Ls, int H, int Dc, int P,
                long long n, int unpack) {
  const int Hp = H / P;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    // idx enumerates the [B, Ls, H, Dc] layout
    long long r = idx;
    const int dc = (int)(r % Dc);
    r /= Dc;
    const int h = (int)(r % H);
    r /= H;
    const int t = (int)(r % Ls);
    const int b = (int)(r / Ls);
    const int p = h / Hp, hl = h - p * Hp;
    const long long blk = ((((long long)p * B + b) * Ls + t) * Hp + hl) * Dc + dc;
    if (unpack)
      dst[idx] = src[blk];
    else
      dst[blk] = src[idx];
  }
}

int launch(const void* src, void* dst, int B, int Ls, int H, int D, int P, void* stream, int unpack) {
  if (!src || !dst) return RW_ERR_INVALID_ARG;
  if (B < 1 || Ls < 0 || H < 1 || P < 1 || D < 8 || (D % 8) != 0 || (H % P) != 0) return RW_ERR_INVALID_ARG;
  if (((uintptr_t)src & 15) || ((uintptr_t)dst & 15)) return RW_ERR_INVALID_ARG;
  const long long n = (long long)B * Ls * H * (D / 8);
  if (n == 0) return RW_OK;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  pack_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>((const uint4*)src, (uint4*)dst, B, Ls, H, D / 8,
                                                                  P, n, unpack);
  return cudaGetLastError() == cudaSuccess ? RW_OK : RW_ERR_CUDA;
}

}  // namespace a2a
}  // namespace rw

extern "C" int rw_a2a_pack(const void* src, void* dst, int B, int Ls, int H, int D, int P, void* stream) {
  return rw::a2a::launch(src, dst, B, Ls, H, D, P, stream, 0);
}

extern "C" int rw_a2a_unpack(const void* src, void* dst, int B, int Ls, int H, int D, int P, void* stream) {
  return rw::a2a::launch(src, dst, B, Ls, H, D, P, stream, 1);
}
