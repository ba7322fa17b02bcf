// Cross-rank ordering carried by the sequence-parallel kernels themselves (the
// rw_sp_sync_t of include/reworld_b200.h): a bounded wait, at the start of a
// kernel, for the epochs other ranks wrote into this rank's signal array, and a
// signal, at the end of a kernel, from the last CTA to finish to every rank.
// This replaces a separate barrier launch on each side of the exchange
// (the process-group synchronisation around wan_5b/distributed/ulysses.py:40-54).
#pragma once

#include "common.cuh"

namespace rw {

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits (bounded) until this rank's entries wait_slot .. wait_slot + P - 1 hold at
// least wait_epoch.  Returns false on a timeout (RW_STATUS_TIMEOUT_PEER recorded) or
// when `abort` (optional) is raised meanwhile.  One thread calls it.
__device__ inline bool sp_wait_peers(const rw_sp_sync_t& s, int* status, const volatile int* abort) {
  const int* mine = reinterpret_cast<const int*>(s.sig_ptrs[s.rank]) + s.wait_slot;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t lim = (uint64_t)s.timeout_ms * 1000000ull;
  for (int q = 0; q < s.P; ++q) {
    for (uint32_t it = 0; ld_acquire_sys(mine + q) - s.wait_epoch < 0; ++it) {
      if ((it & 15u) == 15u) {
        if (abort != nullptr && *abort) return false;
        if (globaltimer_ns() - t0 > lim) {
          report_status(status, RW_STATUS_TIMEOUT_PEER);
          return false;
        }
      }
    }
  }
  return true;
}

// Called by every thread of every CTA at the very end of a kernel: each CTA makes
// its stores (peer memory included) visible system-wide and counts itself; the CTA
// that completes the count resets it for the next launch and writes signal_epoch
// into entry signal_slot + rank of every rank's array.
__device__ inline void sp_signal_done(const rw_sp_sync_t& s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int n = atomicAdd(s.counter, 1);
    const int total = (int)(gridDim.x * gridDim.y * gridDim.z);
    if (n == total - 1) {
      *s.counter = 0;
      __threadfence_system();
      for (int q = 0; q < s.P; ++q)
        st_release_sys(reinterpret_cast<int*>(s.sig_ptrs[q]) + s.signal_slot + s.rank, s.signal_epoch);
    }
  }
}

// Host-side checks of a sync record.
inline bool sp_sync_ok(const rw_sp_sync_t& s) {
  if (s.sig_ptrs == nullptr || s.P < 1 || s.P > 64 || s.rank < 0 || s.rank >= s.P || s.timeout_ms <= 0) return false;
  if (s.wait_epoch < 0 || s.signal_epoch < 0 || s.wait_slot < 0 || s.signal_slot < 0) return false;
  if (s.signal_epoch > 0 && s.counter == nullptr) return false;
  return true;
}

}  // namespace rw
