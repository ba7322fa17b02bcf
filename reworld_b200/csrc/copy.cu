// Landmark / KV-cache assembly: many byte-copy jobs in one launch, moved by the
// TMA bulk-copy engine (cp.async.bulk global -> shared -> global) in 16 KB
// pieces with a 6-stage shared-memory pipeline per CTA.
//
// Replaces the per-member copies of longctx/inference/landmark_cache_v2.py:
// write_into_cache direct-write path (:633-682: sink/recent window copies and
// read_pair_into per retrieved member, :362-397) and the member packing of
// add_chunk (:507-510), for every layer at once.  Pure byte copies, so the
// result is bit-identical to the reference's copy_ calls.
//
// Work split: the pieces of all jobs, in job order, form one sequence; CTA c
// copies the contiguous range [c*P/G, (c+1)*P/G) of it.  One elected thread per
// CTA drives the pipeline (the copy engine moves the data); waits are bounded.
#include "common.cuh"
#include "host_util.h"

namespace rw {
namespace copy {

constexpr int PIECE = 16384;
constexpr int STAGES = 6;
constexpr int SMEM_BYTES = PIECE * STAGES;
constexpr int CTAS_PER_SM = 2;

struct Piece {
  const uint8_t* src;
  uint8_t* dst;
  uint32_t bytes;
};

__device__ __forceinline__ bool desc_ok(const rw_copy_desc_t& d) {
  return d.nbytes > 0 && (d.nbytes & 15) == 0 && ((uintptr_t)d.src & 15) == 0 && ((uintptr_t)d.dst & 15) == 0;
}

__global__ void __launch_bounds__(32, CTAS_PER_SM)
    copy_chunks_kernel(const rw_copy_desc_t* __restrict__ descs, int n, int* status) {
  extern __shared__ __align__(128) uint8_t stage_mem[];
  __shared__ __align__(8) uint64_t full[STAGES];
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;

  // total pieces and this CTA's range
  long long total = 0;
  for (int i = 0; i < n; ++i) {
    const rw_copy_desc_t d = descs[i];
    if (desc_ok(d)) total += (d.nbytes + PIECE - 1) / PIECE;
  }
  const long long g0 = total * blockIdx.x / gridDim.x;
  const long long g1 = total * (blockIdx.x + 1) / gridDim.x;
  if (blockIdx.x == 0) {
    for (int i = 0; i < n; ++i)
      if (!desc_ok(descs[i])) report_status(status, RW_STATUS_BAD_SLOT);
  }
  if (g0 >= g1) return;

  for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
  abort_flag = 0;
  fence_mbar_init();

  // iterator positioned at global piece g0
  int di = 0;
  long long off = 0, g = 0;
  for (; di < n; ++di) {
    const rw_copy_desc_t d = descs[di];
    if (!desc_ok(d)) continue;
    const long long np = (d.nbytes + PIECE - 1) / PIECE;
    if (g + np > g0) {
      off = (g0 - g) * PIECE;
      break;
    }
    g += np;
  }
  if (di >= n) {  // cannot happen when the piece count is consistent; never read past the array
    report_status(status, RW_STATUS_BAD_SLOT);
    return;
  }
  const long long count = g1 - g0;
  Piece ring[STAGES];
  rw_copy_desc_t cur = descs[di];
  auto next_piece = [&]() -> Piece {
    while (off >= cur.nbytes || !desc_ok(cur)) {
      if (di + 1 >= n) {
        Piece none{nullptr, nullptr, 0};
        return none;
      }
      ++di;
      off = 0;
      cur = descs[di];
    }
    Piece pc;
    const long long left = cur.nbytes - off;
    pc.bytes = (uint32_t)(left < PIECE ? left : PIECE);
    pc.src = (const uint8_t*)cur.src + off;
    pc.dst = (uint8_t*)cur.dst + off;
    off += pc.bytes;
    return pc;
  };

  bool ok = true;
  long long issued = 0;
  for (long long k = 0; k < count + STAGES - 1; ++k) {
    if (k < count) {
      const int s = (int)(k % STAGES);
      if (k >= STAGES) bulk_wait_group_read<0>();  // stores that read stage s have finished reading it
      ring[s] = next_piece();
      if (ring[s].bytes == 0) {
        report_status(status, RW_STATUS_BAD_SLOT);
        ok = false;
        break;
      }
      mbar_expect_tx(&full[s], ring[s].bytes);
      bulk_load(stage_mem + s * PIECE, ring[s].src, ring[s].bytes, &full[s]);
      ++issued;
    }
    const long long kk = k - (STAGES - 1);
    if (kk >= 0) {
      const int s = (int)(kk % STAGES);
      if (!mbar_wait(&full[s], (uint32_t)((kk / STAGES) & 1), &abort_flag, status, RW_STATUS_TIMEOUT_COPY)) {
        ok = false;
        break;
      }
      bulk_store(ring[s].dst, stage_mem + s * PIECE, ring[s].bytes);
      bulk_commit_group();
    }
  }
  if (!ok) {
    // let every issued load land before the CTA's shared memory is released
    const long long first = issued > STAGES ? issued - STAGES : 0;
    for (long long u = first; u < issued; ++u) mbar_wait_drain(&full[u % STAGES], (uint32_t)((u / STAGES) & 1));
  }
  bulk_wait_group<0>();
}

}  // namespace copy
}  // namespace rw

using namespace rw;

extern "C" int rw_copy_chunks(const rw_copy_desc_t* descs, int n, int* status, void* stream) {
  if (n < 0) return RW_ERR_INVALID_ARG;
  if (n == 0) return RW_OK;
  if (!descs) return RW_ERR_INVALID_ARG;
  static std::atomic<unsigned long long> attr_done{0};
  if (!ensure_smem_attr((const void*)copy::copy_chunks_kernel, copy::SMEM_BYTES, &attr_done)) return RW_ERR_CUDA;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = sms * copy::CTAS_PER_SM;
  copy::copy_chunks_kernel<<<grid, 32, copy::SMEM_BYTES, (cudaStream_t)stream>>>(descs, n, status);
  return cudaGetLastError() == cudaSuccess ? RW_OK : RW_ERR_CUDA;
}
