// Host-side helpers shared by the launchers: driver entry point for TMA
// descriptor encoding (fetched through the runtime, so the library does not
// link libcuda directly) and argument checks.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

namespace rw {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// bf16 tensor [B, L, H, D=128] with element strides (sb, sl, sh) and unit dim stride,
// described to TMA as dims (D, H, L, B) (byte strides increase for the usual
// contiguous layout) and tiled in boxes of 64 (dim) x 1 (head) x box_rows
// (tokens) with 128-byte swizzle: one box fills box_rows rows of 128 bytes.
// Kernel coordinates are therefore (dim, head, token, batch).
inline int make_bf16_bl_hd_map(CUtensorMap* m, const void* ptr, int B, int L, int H, int D, long long sb,
                               long long sl, long long sh, int box_rows) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return -4;
  // Strides of size-1 dimensions are never used for addressing; give them a
  // valid (16-byte multiple) value.
  if (B == 1) sb = (long long)L * sl > 0 ? (long long)L * sl : 8;
  if (H == 1) sh = D;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)L, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)sl * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -4;
}

// Row-major bf16 matrix [rows, cols] (row stride ld elements) described to TMA as
// dims (cols, rows), tiled in boxes of 64 columns x box_rows rows with 128-byte
// swizzle (one box row = 128 bytes); rows past the end read as zero.
inline int make_bf16_2d_map(CUtensorMap* m, const void* ptr, long long rows, long long cols, long long ld,
                            int box_rows) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return -4;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -4;
}

// Row-major bf16 matrix [rows, cols] (row stride ld) for TMA stores of 32 x 32 boxes
// (64-byte rows, 64-byte swizzle); writes outside the matrix are clipped.
inline int make_bf16_2d_store_map(CUtensorMap* m, const void* ptr, long long rows, long long cols, long long ld) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return -4;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -4;
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device).
// Host threads may race here: the attribute call is idempotent and the mask is
// atomic, so a second thread at worst repeats the call.
inline bool ensure_smem_attr(const void* func, int bytes, std::atomic<unsigned long long>* done_mask) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  const unsigned long long bit = 1ull << dev;
  if (done_mask->load(std::memory_order_acquire) & bit) return true;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  done_mask->fetch_or(bit, std::memory_order_release);
  return true;
}

inline bool stride_ok(long long s) { return s > 0 && (s % 8) == 0 && s < (1ll << 38); }

}  // namespace rw

// Launches `kernel` as a programmatic dependent of the previous kernel on `stream`:
// it may start while that kernel's last blocks run, and must call griddep_wait()
// before it touches global memory (common.cuh).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                    Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
