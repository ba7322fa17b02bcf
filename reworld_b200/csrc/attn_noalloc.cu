// rw_attn_fwd_noalloc: the chunk attention for callers that cannot allocate
// device memory.
//
// rw_attn_fwd needs a scratch workspace from its caller for the key-split last
// wave of work.  Some callers have no way to provide one: a host runtime that
// owns all device memory through its own allocator and gives this library none,
// or a real-time streaming loop in which a cudaMalloc (which can synchronise the
// whole device) would stall frame delivery.  This entry point takes the same
// inputs and outputs as rw_attn_fwd but keeps the scratch in a fixed array
// compiled into the library, so it allocates nothing.
//
// The array is RW_ATTN_NOALLOC_SCRATCH_BYTES (80 MiB) of device memory that every
// GPU loading this part of the library holds until the process exits.  The split
// needs 2 partial-result slots of 133,120 bytes per resident pair, whatever the
// shape: 19.7 MB with the 74 pairs of a B200, so the array is exceeded only on a
// device with more than 315 resident pairs; such shapes are refused with
// RW_ERR_CAPACITY.  The stream must belong to the current device (the array's
// address is per device); another device's stream is refused.  All calls share
// the one array: calls that overlap on the GPU (other streams, other host
// threads) race on it.  Nothing in it has to start at zero: every partial slot
// the merge step reads is written earlier in the same call.
#include <mutex>

#include "../../include/reworld_b200.h"
#include <cuda_runtime.h>

namespace {

static __device__ __align__(256) unsigned char g_attn_scratch[RW_ATTN_NOALLOC_SCRATCH_BYTES];

// Device address of g_attn_scratch, resolved once per device.  In host code the
// array's name is only a host-side stand-in, never a device address.
constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RW_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return RW_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_scratch) != cudaSuccess || p == nullptr) return RW_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return RW_OK;
}

}  // namespace

extern "C" int rw_attn_fwd_noalloc(const void* q, const void* k, const void* v, void* o, int B, int Lq, int Lk, int H,
                                   int D, long long q_sb, long long q_sl, long long q_sh, long long k_sb,
                                   long long k_sl, long long k_sh, long long v_sb, long long v_sl, long long v_sh,
                                   long long o_sb, long long o_sl, long long o_sh, float softmax_scale,
                                   const rw_rope_t* rope, int* status, void* stream) {
  if (stream != nullptr) {
    int cur = -1, sdev = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cudaStreamGetDevice((cudaStream_t)stream, &sdev) != cudaSuccess)
      return RW_ERR_CUDA;
    if (sdev != cur) return RW_ERR_INVALID_ARG;
  }
  const long long need = rw_attn_workspace_bytes(B, Lq, Lk, H);
  if (need > RW_ATTN_NOALLOC_SCRATCH_BYTES) return RW_ERR_CAPACITY;
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = scratch_address(&scratch);
    if (rc != RW_OK) return rc;
  }
  return rw_attn_fwd(q, k, v, o, B, Lq, Lk, H, D, q_sb, q_sl, q_sh, k_sb, k_sl, k_sh, v_sb, v_sl, v_sh, o_sb, o_sl,
                     o_sh, softmax_scale, rope, scratch, need > 0 ? RW_ATTN_NOALLOC_SCRATCH_BYTES : 0, status, stream);
}
