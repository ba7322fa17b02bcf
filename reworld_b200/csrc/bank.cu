// Landmark-bank decisions on the device: always-admit insertion with
// protect-earliest-n + most-redundant eviction, and pose top-k retrieval.
//
// Reference: longctx/inference/landmark_cache_v2.py
//   _bank_D        :90-98    pairwise distance used by eviction (numpy, fp64)
//   _evict_index   :465-479  protect first protect_n, argmin (nn-dist, -born)
//   _bank_insert   :481-495  evict while full, append, protected = admitted < protect_n
//   _retrieve      :538-592  plain top-k by pose_dist, sorted indices
// and pose_dist of longctx/inference/landmark_cache.py:24-31.
//
// The arithmetic follows the reference operation by operation so that the
// retrieved index sets and eviction victims are identical:
//  * pose_dist: |t_a - t_b| is formed like numpy/OpenBLAS does for a 3-vector
//    (fp32 arrays: fp32 difference, fp32 squares summed in fp64, rounded to
//    fp32, fp32 sqrt; fp64 arrays: fused multiply-add chain, fp64 sqrt), the
//    yaw term with Python float semantics (fmod, min, /60), then
//    sqrt(dxyz*dxyz + dyaw*dyaw) without contraction.
//  * _bank_D: fp64 difference, squares added left to right, sqrt; yaw term
//    with numpy remainder/minimum; sqrt(dt*dt + dy*dy).
// The yaw angles themselves come from the host (rw_pose_t), computed with the
// same library calls as the reference.
//
// One CTA of 128 threads: the O(n^2) nearest-neighbour distances are spread
// over all threads, argmin / top-k selection is done by warp 0 with shuffles.
#include "common.cuh"

namespace rw {
namespace bank {

constexpr int THREADS = 128;

__device__ __forceinline__ double yaw_term(double ya, double yb) {
  const double d = fmod(fabs(__dsub_rn(ya, yb)), 360.0);
  const double e = __dsub_rn(360.0, d);
  return __ddiv_rn(d <= e ? d : e, 60.0);
}

// pose_dist(target, member), landmark_cache.py:24-31
__device__ __forceinline__ double dist_retrieve(const rw_pose_t& a, const rw_pose_t& b) {
  double dxyz;
  if (a.is_f32 != 0.0 && b.is_f32 != 0.0) {
    const float fx = __fsub_rn((float)a.tx, (float)b.tx);
    const float fy = __fsub_rn((float)a.ty, (float)b.ty);
    const float fz = __fsub_rn((float)a.tz, (float)b.tz);
    const double s = __dadd_rn(__dadd_rn((double)__fmul_rn(fx, fx), (double)__fmul_rn(fy, fy)),
                               (double)__fmul_rn(fz, fz));
    dxyz = (double)__fsqrt_rn(__double2float_rn(s));
  } else {
    const double dx = __dsub_rn(a.tx, b.tx), dy = __dsub_rn(a.ty, b.ty), dz = __dsub_rn(a.tz, b.tz);
    dxyz = __dsqrt_rn(__fma_rn(dz, dz, __fma_rn(dy, dy, __dmul_rn(dx, dx))));
  }
  const double dyaw = yaw_term(a.yaw_r, b.yaw_r);
  return __dsqrt_rn(__dadd_rn(__dmul_rn(dxyz, dxyz), __dmul_rn(dyaw, dyaw)));
}

// _bank_D entry (i, j), landmark_cache_v2.py:90-98
__device__ __forceinline__ double dist_evict(const rw_pose_t& a, const rw_pose_t& b) {
  const double dx = __dsub_rn(a.tx, b.tx), dy = __dsub_rn(a.ty, b.ty), dz = __dsub_rn(a.tz, b.tz);
  const double dt = __dsqrt_rn(__dadd_rn(__dadd_rn(__dmul_rn(dx, dx), __dmul_rn(dy, dy)), __dmul_rn(dz, dz)));
  const double dyaw = yaw_term(a.yaw_e, b.yaw_e);
  return __dsqrt_rn(__dadd_rn(__dmul_rn(dt, dt), __dmul_rn(dyaw, dyaw)));
}

// key (d, tiebreak) smaller-is-better; returns true when (d1,t1) < (d2,t2)
__device__ __forceinline__ bool key_less(double d1, int t1, double d2, int t2) {
  return d1 < d2 || (d1 == d2 && t1 < t2);
}

// Warp-wide argmin of (d, t) pairs held one per lane; result broadcast.
__device__ __forceinline__ void warp_argmin(double& d, int& t, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double d2 = __shfl_xor_sync(0xffffffffu, d, o);
    const int t2 = __shfl_xor_sync(0xffffffffu, t, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    if (key_less(d2, t2, d, t)) {
      d = d2;
      t = t2;
      idx = i2;
    }
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    bank_step_kernel(rw_bank_state_t* __restrict__ st, int K, int protect_n, int admit,
                     const rw_pose_t* __restrict__ admit_pose, int admit_born, int admit_slot,
                     const rw_pose_t* __restrict__ target, int rk, int mode, rw_bank_result_t* __restrict__ res) {
  __shared__ double val[RW_BANK_MAX];
  __shared__ unsigned char taken[RW_BANK_MAX];
  __shared__ int s_victim;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  int n = st->n;
  int n_ev = 0;

  if (admit) {
    while (n >= K && n > 0) {
      int victim = 0;
      if (n > 1) {
        // nearest-neighbour distance of every member
        for (int i = tid; i < n; i += THREADS) {
          const rw_pose_t pi = st->pose[i];
          double m = INFINITY;
          for (int j = 0; j < n; ++j) {
            if (j == i) continue;
            const double d = dist_evict(pi, st->pose[j]);
            m = d < m ? d : m;
          }
          val[i] = m;
        }
        __syncthreads();
        if (warp == 0) {
          int any_unprot = 0;
          for (int i = lane; i < n; i += 32) any_unprot |= (st->prot[i] == 0);
          any_unprot = __any_sync(0xffffffffu, any_unprot);
          double bd = INFINITY;
          int bt = 0x7fffffff, bi = -1;
          for (int i = lane; i < n; i += 32) {
            if (any_unprot && st->prot[i]) continue;
            const int t = -st->born[i];  // ties evict the later-born
            if (bi < 0 || key_less(val[i], t, bd, bt)) {
              bd = val[i];
              bt = t;
              bi = i;
            }
          }
          if (bi < 0) bt = 0x7fffffff;
          warp_argmin(bd, bt, bi);
          if (lane == 0) s_victim = bi;
        }
        __syncthreads();
        victim = s_victim;
      }
      if (tid == 0 && n_ev < 4) {
        res->evicted_born[n_ev] = st->born[victim];
        res->evicted_slot[n_ev] = st->slot[victim];
      }
      ++n_ev;
      __syncthreads();
      // remove entry `victim`, keeping list order (single thread: n <= 1024 small records)
      if (tid == 0) {
        for (int i = victim; i + 1 < n; ++i) {
          st->pose[i] = st->pose[i + 1];
          st->born[i] = st->born[i + 1];
          st->slot[i] = st->slot[i + 1];
          st->prot[i] = st->prot[i + 1];
        }
      }
      --n;
      __syncthreads();
    }
    if (tid == 0) {
      st->pose[n] = *admit_pose;
      st->born[n] = admit_born;
      st->slot[n] = admit_slot;
      st->prot[n] = st->admitted < protect_n ? 1 : 0;
      st->admitted += 1;
    }
    ++n;
    __syncthreads();
  }

  // ---------------------------------------------------------------- retrieval
  int nR = 0;
  if (n > 0 && mode == 0) {
    nR = n;
    for (int i = tid; i < n; i += THREADS) {
      res->R[i] = i;
      res->R_slot[i] = st->slot[i];
    }
  } else if (n > 0) {
    const rw_pose_t tp = *target;
    for (int i = tid; i < n; i += THREADS) {
      val[i] = dist_retrieve(tp, st->pose[i]);
      taken[i] = 0;
    }
    __syncthreads();
    const int k = rk < n ? rk : n;
    if (warp == 0) {
      // k rounds of warp argmin over the members not taken yet
      for (int r = 0; r < k; ++r) {
        double bd = INFINITY;
        int bt = 0x7fffffff, bi = -1;
        for (int i = lane; i < n; i += 32) {
          if (taken[i]) continue;
          if (bi < 0 || key_less(val[i], i, bd, bt)) {
            bd = val[i];
            bt = i;
            bi = i;
          }
        }
        warp_argmin(bd, bt, bi);
        if (lane == 0 && bi >= 0) taken[bi] = 1;
        __syncwarp();
      }
      // emit the taken indices in ascending order (ballot prefix scan)
      int base = 0;
      for (int c = 0; c < n; c += 32) {
        const int i = c + lane;
        const bool f = i < n && taken[i];
        const unsigned m = __ballot_sync(0xffffffffu, f);
        if (f) {
          const int pos = base + __popc(m & ((1u << lane) - 1u));
          res->R[pos] = i;
          res->R_slot[pos] = st->slot[i];
        }
        base += __popc(m);
      }
    }
    nR = k;
  }
  if (tid == 0) {
    st->n = n;
    res->n_evicted = n_ev;
    res->n_bank = n;
    res->nR = nR;
  }
}

}  // namespace bank
}  // namespace rw

using namespace rw;

extern "C" int rw_bank_step(rw_bank_state_t* state, int K, int protect_n, int admit, const rw_pose_t* admit_pose,
                            int admit_born, int admit_slot, const rw_pose_t* target, int retrieve_k, int mode,
                            rw_bank_result_t* result, void* stream) {
  if (!state || !result) return RW_ERR_INVALID_ARG;
  if (K < 1 || K > RW_BANK_MAX || protect_n < 0 || retrieve_k < 0) return RW_ERR_INVALID_ARG;
  if (mode != 0 && mode != 1) return RW_ERR_INVALID_ARG;
  if (admit && !admit_pose) return RW_ERR_INVALID_ARG;
  if (mode == 1 && !target) return RW_ERR_INVALID_ARG;
  bank::bank_step_kernel<<<1, bank::THREADS, 0, (cudaStream_t)stream>>>(
      state, K, protect_n, admit, admit_pose, admit_born, admit_slot, target, retrieve_k, mode, result);
  return cudaGetLastError() == cudaSuccess ? RW_OK : RW_ERR_CUDA;
}
