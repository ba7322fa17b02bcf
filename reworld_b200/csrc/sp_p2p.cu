// Ulysses exchanges over peer memory (NVLink), fused with the layout transform
// and, on the way in, with the RoPE of k and the KV-cache write.
//
// Reference pattern: wan_5b/distributed/ulysses.py:17-55 (all_to_all of q, k, v
// seq -> head, attention, all_to_all of the output head -> seq) and
// wan_5b/distributed/util.py:52-64; the cache write and RoPE it replaces on the
// receiving side are wan_5b/modules/action_model.py:265-292.
//
// Rank r holds q, k, v of tokens [r*Ls, (r+1)*Ls) of the chunk for all H heads
// ([Ls, H, D], one sequence) and owns heads [r*Hp, (r+1)*Hp) of every cache.
// rw_sp_scatter_qkv writes, for each (token s, head h) with p = h / Hp,
// hl = h % Hp and t = r*Ls + s:
//     q_dst[p][t][hl]               = q[s][h]          (RoPE of q is applied later,
//                                                       inside the attention kernel)
//     ck_dst[p][dst_start + t][hl]  = rope_t(k[s][h])
//     cv_dst[p][dst_start + t][hl]  = v[s][h]
// straight into the owning rank's buffers (plain 16-byte stores through peer
// pointers; no multicast), so no packed staging buffer, no collective library
// call and no separate cache-write kernel are needed.  rw_sp_scatter_out sends
// the attention output o[t][hl] (t in [0, P*Ls)) back to rank p = t / Ls as
// out_dst[p][t % Ls][r*Hp + hl].  Completion across ranks: either the caller's
// stream-ordered barrier after each scatter, or the scatter's own sync record
// (sp_sync.cuh: a bounded wait before its first store, a signal from its last CTA).
#include "common.cuh"
#include "host_util.h"
#include "rope.cuh"
#include "sp_sync.cuh"

namespace rw {
namespace sp {

struct ScatterQKV {
  const uint8_t* q;
  const uint8_t* k;
  const uint8_t* v;
  long long q_sl, q_sh, k_sl, k_sh, v_sl, v_sh;
  const unsigned long long* q_dst;
  const unsigned long long* ck_dst;
  const unsigned long long* cv_dst;
  int Ls, H, Hp, P, rank, dst_start;
  int rope_on;
  rw_rope_t rope;
  int sync_on;
  rw_sp_sync_t sync;
  int* status;
};

constexpr int SCATTER_THREADS = 128;  // a multiple of 16 (see scatter_qkv_kernel)
constexpr int SCATTER_HSTEP = SCATTER_THREADS / 16;  // heads between two chunks of a thread
constexpr int SCATTER_NB = 3;                         // chunks per thread and batch (24 heads: one batch)

// CTAs walk this rank's tokens s; thread x handles chunk c16 = x mod 16 of heads
// x / 16, x / 16 + 8, ..., so its 4 RoPE table entries are looked up once per
// token, and the loads of a batch of heads are issued before its first store.
__global__ void __launch_bounds__(SCATTER_THREADS) scatter_qkv_kernel(const __grid_constant__ ScatterQKV p) {
  __shared__ int go;
  griddep_launch_dependents();  // the attention may be scheduled; its producer waits for this kernel
  griddep_wait();               // launched as a dependent: the previous kernel is done
  if (p.sync_on && p.sync.wait_epoch > 0) {
    // the ranks' earlier reads of the buffers this scatter overwrites are done
    if (threadIdx.x == 0) go = sp_wait_peers(p.sync, p.status, nullptr) ? 1 : 0;
    __syncthreads();
    if (!go) {
      if (p.sync.signal_epoch > 0) sp_signal_done(p.sync);
      return;
    }
  }
  const int c16 = threadIdx.x & 15;
  const int h0 = threadIdx.x >> 4;
  const long long eoff = (long long)c16 * 8;
  for (int s = blockIdx.x; s < p.Ls; s += gridDim.x) {
    const int t = p.rank * p.Ls + s;
    const uint8_t* qrow = p.q + 2 * (s * p.q_sl + eoff);
    const uint8_t* krow = p.k + 2 * (s * p.k_sl + eoff);
    const uint8_t* vrow = p.v + 2 * (s * p.v_sl + eoff);
    for (int hb = h0; hb < p.H; hb += SCATTER_HSTEP * SCATTER_NB) {
      uint4 qv[SCATTER_NB], kv[SCATTER_NB], vv[SCATTER_NB];
#pragma unroll
      for (int j = 0; j < SCATTER_NB; ++j) {
        const long long h = hb + j * SCATTER_HSTEP;
        if (h < p.H) {
          qv[j] = __ldg(reinterpret_cast<const uint4*>(qrow + 2 * h * p.q_sh));
          kv[j] = __ldg(reinterpret_cast<const uint4*>(krow + 2 * h * p.k_sh));
          vv[j] = __ldg(reinterpret_cast<const uint4*>(vrow + 2 * h * p.v_sh));
        }
      }
      double2 cs[4];
      float2 dl[4];
      bool rot = false, has_d = false;
      if (p.rope_on) {
        const RopeToken rt = rope_token(p.rope, t, 0);
        rot = rt.on;
        has_d = rt.dl != nullptr;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          cs[j] = rope_freq(4 * c16 + j, rt);
          dl[j] = has_d ? rt.dl[4 * c16 + j] : make_float2(0.f, 0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < SCATTER_NB; ++j) {
        const int h = hb + j * SCATTER_HSTEP;
        if (h < p.H) {
          const int owner = h / p.Hp, hl = h - owner * p.Hp;
          uint4 kr = kv[j];
          if (rot) {
            kr.x = rope_rotate(kr.x, cs[0], has_d, dl[0]);
            kr.y = rope_rotate(kr.y, cs[1], has_d, dl[1]);
            kr.z = rope_rotate(kr.z, cs[2], has_d, dl[2]);
            kr.w = rope_rotate(kr.w, cs[3], has_d, dl[3]);
          }
          const long long qoff = 2 * (((long long)t * p.Hp + hl) * 128 + eoff);
          const long long coff = 2 * (((long long)(p.dst_start + t) * p.Hp + hl) * 128 + eoff);
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.q_dst[owner]) + qoff) = qv[j];
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.ck_dst[owner]) + coff) = kr;
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.cv_dst[owner]) + coff) = vv[j];
        }
      }
    }
  }
  if (p.sync_on && p.sync.signal_epoch > 0) sp_signal_done(p.sync);
}

__global__ void __launch_bounds__(32) wait_kernel(const __grid_constant__ rw_sp_sync_t s, int* status) {
  if (threadIdx.x == 0) sp_wait_peers(s, status, nullptr);
}

__global__ void __launch_bounds__(256)
    scatter_out_kernel(const uint8_t* __restrict__ o, const unsigned long long* __restrict__ out_dst, int L, int H,
                       int Hp, int P, int rank) {
  const int Ls = L / P;
  const long long n = (long long)L * Hp * 16;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c16 = (int)(idx & 15);
    const long long th = idx >> 4;
    const int hl = (int)(th % Hp);
    const int t = (int)(th / Hp);
    const int owner = t / Ls, s = t - owner * Ls;
    const uint4 val = __ldg(reinterpret_cast<const uint4*>(o + 2 * (((long long)t * Hp + hl) * 128 + c16 * 8)));
    const long long doff = 2 * (((long long)s * H + rank * Hp + hl) * 128 + c16 * 8);
    *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(out_dst[owner]) + doff) = val;
  }
}

// Cross-rank barrier: thread p signals rank p and waits for rank p's signal.

__global__ void __launch_bounds__(32) barrier_kernel(const unsigned long long* __restrict__ sig_ptrs, int slot_base,
                                                     int P, int rank, int epoch, unsigned long long timeout_ns,
                                                     int* status) {
  const int p = threadIdx.x;
  if (p < P) {
    __threadfence_system();  // this rank's earlier stores (peer memory included) before the signal
    st_release_sys(reinterpret_cast<int*>(sig_ptrs[p]) + slot_base + rank, epoch);
    const int* mine = reinterpret_cast<const int*>(sig_ptrs[rank]) + slot_base + p;
    if (ld_acquire_sys(mine) - epoch < 0) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(mine) - epoch < 0) {
        if (globaltimer_ns() - t0 > timeout_ns) {
          report_status(status, RW_STATUS_TIMEOUT_PEER);
          break;
        }
      }
    }
  }
  __syncwarp();
}

inline unsigned grid_for(long long n) {
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  return (unsigned)(blocks < 1 ? 1 : blocks);
}

}  // namespace sp
}  // namespace rw

using namespace rw;

extern "C" int rw_sp_scatter_qkv(const void* q, const void* k, const void* v, long long q_sl, long long q_sh,
                                 long long k_sl, long long k_sh, long long v_sl, long long v_sh,
                                 const unsigned long long* q_dst, const unsigned long long* ck_dst,
                                 const unsigned long long* cv_dst, int Ls, int H, int D, int P, int rank,
                                 int dst_start, int cap, const rw_rope_t* rope, const rw_sp_sync_t* sync,
                                 int* status, void* stream) {
  if (!q || !k || !v || !q_dst || !ck_dst || !cv_dst) return RW_ERR_INVALID_ARG;
  if (D != 128) return RW_ERR_UNSUPPORTED;
  if (Ls < 1 || H < 1 || P < 1 || (H % P) != 0 || rank < 0 || rank >= P || dst_start < 0) return RW_ERR_INVALID_ARG;
  if ((long long)dst_start + (long long)P * Ls > cap) return RW_ERR_CAPACITY;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v)) return RW_ERR_INVALID_ARG;
  const long long st[6] = {q_sl, q_sh, k_sl, k_sh, v_sl, v_sh};
  for (int i = 0; i < 6; ++i)
    if (st[i] < 0 || (st[i] % 8) != 0) return RW_ERR_INVALID_ARG;
  sp::ScatterQKV p{};
  p.q = (const uint8_t*)q;
  p.k = (const uint8_t*)k;
  p.v = (const uint8_t*)v;
  p.q_sl = q_sl; p.q_sh = q_sh; p.k_sl = k_sl; p.k_sh = k_sh; p.v_sl = v_sl; p.v_sh = v_sh;
  p.q_dst = q_dst;
  p.ck_dst = ck_dst;
  p.cv_dst = cv_dst;
  p.Ls = Ls;
  p.H = H;
  p.Hp = H / P;
  p.P = P;
  p.rank = rank;
  p.dst_start = dst_start;
  p.rope_on = 0;
  if (rope != nullptr) {
    if (!rope_args_ok(*rope, D)) return RW_ERR_INVALID_ARG;
    p.rope = *rope;
    p.rope_on = 1;
  }
  p.sync_on = 0;
  p.status = status;
  if (sync != nullptr) {
    if (!sp_sync_ok(*sync) || sync->P != P || sync->rank != rank) return RW_ERR_INVALID_ARG;
    p.sync = *sync;
    p.sync_on = 1;
  }
  {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // with a signal every CTA ends with a system-scope fence: a few CTAs per SM, each
    // walking several tokens, keep that cost small; without one, a CTA per token
    const int cap_ctas = p.sync_on && p.sync.signal_epoch > 0 ? sms * 2 : sms * 16;
    const int grid = Ls < cap_ctas ? Ls : cap_ctas;
    if (launch_dependent(sp::scatter_qkv_kernel, dim3(grid), dim3(sp::SCATTER_THREADS), 0, (cudaStream_t)stream, p) !=
        cudaSuccess)
      return RW_ERR_CUDA;
  }
  return RW_OK;
}

extern "C" int rw_sp_scatter_out(const void* o, const unsigned long long* out_dst, int L, int H, int D, int P,
                                 int rank, void* stream) {
  if (!o || !out_dst) return RW_ERR_INVALID_ARG;
  if (D != 128) return RW_ERR_UNSUPPORTED;
  if (L < 1 || H < 1 || P < 1 || (H % P) != 0 || (L % P) != 0 || rank < 0 || rank >= P) return RW_ERR_INVALID_ARG;
  if (!aligned16(o)) return RW_ERR_INVALID_ARG;
  sp::scatter_out_kernel<<<sp::grid_for((long long)L * (H / P) * 16), 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)o, out_dst, L, H, H / P, P, rank);
  return cudaGetLastError() == cudaSuccess ? RW_OK : RW_ERR_CUDA;
}

extern "C" int rw_sp_barrier(const unsigned long long* sig_ptrs, int slot_base, int P, int rank, int epoch,
                             int timeout_ms, int* status, void* stream) {
  if (!sig_ptrs) return RW_ERR_INVALID_ARG;
  if (P < 1 || P > 32 || rank < 0 || rank >= P || slot_base < 0 || epoch <= 0 || timeout_ms <= 0)
    return RW_ERR_INVALID_ARG;
  sp::barrier_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(sig_ptrs, slot_base, P, rank, epoch,
                                                         (unsigned long long)timeout_ms * 1000000ull, status);
  return cudaGetLastError() == cudaSuccess ? RW_OK : RW_ERR_CUDA;
}

extern "C" int rw_sp_wait(const rw_sp_sync_t* sync, int* status, void* stream) {
  if (sync == nullptr || !sp_sync_ok(*sync) || sync->wait_epoch <= 0) return RW_ERR_INVALID_ARG;
  sp::wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(*sync, status);
  return cudaGetLastError() == cudaSuccess ? RW_OK : RW_ERR_CUDA;
}
