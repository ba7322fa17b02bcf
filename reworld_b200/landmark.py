"""Landmark bank on the device: pose decisions by rw_bank_step, K/V moves by
rw_copy_chunks (TMA bulk copies), storage in one preallocated HBM pool.

Reference: longctx/inference/landmark_cache_v2.py (LandmarkCacheV2 :413-722)
and the way the compressed pipeline drives it
(pipeline/causal_diffusion_inference_compressed.py:809-852, one bank per layer
whose decisions are identical across layers).

* `LandmarkCacheV2` — per-layer drop-in with the reference's constructor and
  methods (add_chunk -> retrieved bank indices, write_into_cache -> local end
  index, active_layout, get_active_kv, stats, events).
* `LandmarkBankStack` — the same bank for all layers of the model at once: one
  decision per chunk and ONE gather launch that assembles
  sink | recent | bank[R] into every layer's cache.

Storage: chunk K/V live in a device pool of slots [n_slots, n_layers, 2, ct, H,
D] (bf16); sink, recent and bank members each own a slot, recycled through a
free list (the reference keeps bank members in a host pool and copies them in
over PCIe each chunk; here every member stays resident in HBM).
"""
import ctypes
import math
import os

import numpy as np
import torch

from . import _native
from ._native import c_vp

BANK_MAX = 1024


class RwPose(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in ("tx", "ty", "tz", "yaw_r", "yaw_e", "is_f32", "pad0", "pad1")]


class RwBankState(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int), ("admitted", ctypes.c_int), ("pad", ctypes.c_int * 2),
                ("pose", RwPose * BANK_MAX), ("born", ctypes.c_int * BANK_MAX), ("slot", ctypes.c_int * BANK_MAX),
                ("prot", ctypes.c_int * BANK_MAX)]


class RwBankResult(ctypes.Structure):
    _fields_ = [("n_evicted", ctypes.c_int), ("evicted_born", ctypes.c_int * 4), ("evicted_slot", ctypes.c_int * 4),
                ("n_bank", ctypes.c_int), ("nR", ctypes.c_int), ("pad", ctypes.c_int),
                ("R", ctypes.c_int * BANK_MAX), ("R_slot", ctypes.c_int * BANK_MAX)]


_ENV_VARIANTS = ("BANKV2_ADMIT_STRIDE_STEPS", "BANKV2_RETRIEVE_MIN_AGE", "BANKV2_RETRIEVE_FAR_GATE",
                 "BANKV2_RETRIEVE_DIVERSE_SEP")


def _check_env():
    for k in _ENV_VARIANTS:
        if float(os.environ.get(k, "0") or 0) != 0:
            raise NotImplementedError(f"{k} (an opt-in retrieval/admission variant) is not implemented")
    if os.environ.get("BANKV2_ROPE_REMAP", "0") == "1":
        raise NotImplementedError("BANKV2_ROPE_REMAP (virtual RoPE time axis) is not implemented")


def pose_record(pose):
    """rw_pose_t of a 4x4 pose: translation, the retrieval yaw (Python math, as
    landmark_cache.py:27-28) and the eviction yaw (numpy, as
    landmark_cache_v2.py:93-94), and whether the pose array is float32."""
    p = np.asarray(pose)
    r02, r22 = p[0, 2], p[2, 2]
    yaw_r = math.degrees(math.atan2(r02, r22))
    P64 = p.astype(np.float64)
    yaw_e = float(np.degrees(np.arctan2(P64[0, 2], P64[2, 2])))
    return RwPose(float(P64[0, 3]), float(P64[1, 3]), float(P64[2, 3]), yaw_r, yaw_e,
                  1.0 if p.dtype == np.float32 else 0.0, 0.0, 0.0)


class DeviceBankDecisions:
    """Bank membership (pose, born, slot, protected) kept in device memory and
    updated by rw_bank_step; a host mirror of the list is kept for the API."""

    def __init__(self, K, retrieve_k, mode="b", protect_n=2, device="cuda"):
        if K > BANK_MAX:
            raise ValueError(f"bank capacity {K} exceeds {BANK_MAX}")
        self.K, self.retrieve_k, self.protect_n = int(K), int(retrieve_k), int(protect_n)
        self.mode = 1 if mode == "b" else 0
        self.device = torch.device(device)
        self.state = torch.zeros(ctypes.sizeof(RwBankState), dtype=torch.uint8, device=self.device)
        self.result = torch.zeros(ctypes.sizeof(RwBankResult), dtype=torch.uint8, device=self.device)
        self.poses = torch.zeros(2 * ctypes.sizeof(RwPose), dtype=torch.uint8, device=self.device)
        self.members = []          # host mirror: list of (born, slot, pose)
        self._admitted = 0

    def step(self, admit=None, target=None):
        """admit = (pose, born, slot) or None; target = pose for mode 'b'.
        Returns (evicted [(born, slot)], R, R_slots)."""
        recs = (RwPose * 2)()
        if admit is not None:
            recs[0] = pose_record(admit[0])
        if target is not None:
            recs[1] = pose_record(target)
        host = torch.frombuffer(bytearray(bytes(recs)), dtype=torch.uint8)
        self.poses.copy_(host)
        p0 = self.poses.data_ptr()
        ps = ctypes.sizeof(RwPose)
        lib = _native.lib()
        with torch.cuda.device(self.device):
            code = lib.rw_bank_step(
                c_vp(self.state.data_ptr()), self.K, self.protect_n, 1 if admit is not None else 0,
                c_vp(p0), int(admit[1]) if admit is not None else -1, int(admit[2]) if admit is not None else -1,
                c_vp(p0 + ps) if target is not None else None, self.retrieve_k, self.mode,
                c_vp(self.result.data_ptr()), _native.stream_ptr(self.device))
        _native.check(code, "rw_bank_step")
        res = RwBankResult.from_buffer_copy(self.result.cpu().numpy().tobytes())
        evicted = [(res.evicted_born[i], res.evicted_slot[i]) for i in range(min(res.n_evicted, 4))]
        if res.n_evicted > 4:
            raise RuntimeError("more than 4 evictions in one step")
        for born, _slot in evicted:
            idx = [m[0] for m in self.members].index(born)
            self.members.pop(idx)
        if admit is not None:
            self.members.append((int(admit[1]), int(admit[2]), np.asarray(admit[0]).copy()))
            self._admitted += 1
        if res.n_bank != len(self.members):
            raise RuntimeError(f"bank mirror out of sync: device {res.n_bank} vs host {len(self.members)}")
        R = [res.R[i] for i in range(res.nR)]
        R_slots = [res.R_slot[i] for i in range(res.nR)]
        return evicted, R, R_slots


class _Entry:
    """Host view of a sink / recent / bank chunk (born index, pose, pool slot)."""
    __slots__ = ("born", "pose", "slot", "protected", "visit", "phase_f")

    def __init__(self, born, pose, slot):
        self.born, self.pose, self.slot = born, np.asarray(pose).copy(), slot
        self.protected, self.visit, self.phase_f = False, 1, None

    @property
    def member_id(self):
        return self.born


class _ChunkPool:
    """[n_slots, n_layers, 2, ct, H, D] bf16 pool with a slot free list."""

    def __init__(self, n_slots, n_layers, ct, H, D, device, dtype=torch.bfloat16):
        self.pool = torch.empty((n_slots, n_layers, 2, ct, H, D), dtype=dtype, device=device)
        self.free = list(range(n_slots))
        self.ct, self.H, self.D, self.n_layers = ct, H, D, n_layers
        self.chunk_bytes = ct * H * D * self.pool.element_size()

    def acquire(self):
        if not self.free:
            raise RuntimeError("chunk pool exhausted")
        return self.free.pop(0)

    def release(self, slot):
        self.free.append(slot)

    def ptr(self, slot, layer, kv):
        return self.pool[slot, layer, kv].data_ptr()


def copy_jobs(jobs, device, status=None):
    """Runs [(src_ptr, dst_ptr, nbytes), ...] with one rw_copy_chunks launch."""
    if not jobs:
        return
    arr = torch.tensor(np.asarray(jobs, dtype=np.int64).reshape(-1, 3), dtype=torch.int64)
    d = arr.to(device, non_blocking=False)
    st = status if status is not None else _native.status_tensor(torch.device(device))
    lib = _native.lib()
    with torch.cuda.device(device):
        code = lib.rw_copy_chunks(c_vp(d.data_ptr()), len(jobs), c_vp(st.data_ptr()), _native.stream_ptr(device))
    _native.check(code, "rw_copy_chunks")
    # `d` is released to the caching allocator on this stream, so it cannot be
    # reused before the copy kernel (queued earlier on the same stream) has read it.


class LandmarkBankStack:
    """Landmark bank shared by all layers (one decision per chunk, one gather
    launch for every layer).  Same policy as LandmarkCacheV2: sink chunks,
    a recent window of recent_w chunks, an always-admit bank of capacity K with
    protect-earliest-protect_n + most-redundant eviction and top-retrieve_k
    pose retrieval (mode 'b') or the whole bank (mode 'a')."""

    def __init__(self, chunk_tokens, n_layers, num_heads, head_dim, n_sink=1, recent_w=5, K=30, retrieve_k=6,
                 mode="b", protect_n=2, device="cuda", dtype=torch.bfloat16):
        _check_env()
        assert mode in ("a", "b")
        self.ct, self.n_layers, self.H, self.D = chunk_tokens, n_layers, num_heads, head_dim
        self.n_sink, self.recent_w, self.K, self.retrieve_k, self.mode = n_sink, recent_w, K, retrieve_k, mode
        self.protect_n = protect_n
        self.device = torch.device(device)
        self.pool = _ChunkPool(n_sink + recent_w + K + 1, n_layers, chunk_tokens, num_heads, head_dim,
                               self.device, dtype)
        self.dec = DeviceBankDecisions(K, retrieve_k, mode, protect_n, self.device)
        self.sink, self.recent, self.bank = [], [], []
        self.events = []
        self._n = 0

    # -- chunk admission ----------------------------------------------------
    def add_chunk_from(self, src_k, src_v, pose, pose_next=None):
        """src_k/src_v: per-layer lists of [ct, H, D] views (e.g. the cache rows
        the chunk was just written to).  Packs them into a pool slot (one launch)
        and runs the bank decision.  Returns R (bank indices, ascending)."""
        c = self._n
        self._n += 1
        slot = self.pool.acquire()
        jobs = []
        nb = self.pool.chunk_bytes
        for layer in range(self.n_layers):
            for kv, src in ((0, src_k[layer]), (1, src_v[layer])):
                if src.dtype != self.pool.pool.dtype or not src.is_contiguous():
                    raise ValueError("chunk K/V must be contiguous and of the pool dtype")
                jobs.append((src.data_ptr(), self.pool.ptr(slot, layer, kv), nb))
        copy_jobs(jobs, self.device)
        e = _Entry(c, pose, slot)
        admit = None
        if c < self.n_sink:
            self.sink.append(e)
        else:
            self.recent.append(e)
            while len(self.recent) > self.recent_w:
                old = self.recent.pop(0)
                if admit is not None:
                    raise RuntimeError("more than one chunk aged out in one step")
                admit = old
        target = pose_next if pose_next is not None else pose
        evicted, R, _ = self.dec.step(
            admit=(admit.pose, admit.born, admit.slot) if admit is not None else None,
            target=target if self.mode == "b" else None)
        for born, slot_ev in evicted:
            j = [m.born for m in self.bank].index(born)
            self.bank.pop(j)
            self.pool.release(slot_ev)
            self.events.append(("evict", born))
        if admit is not None:
            admit.protected = self.dec._admitted <= self.protect_n
            self.bank.append(admit)
            self.events.append(("add", admit.born, len(self.bank)))
        return R

    # -- cache assembly ------------------------------------------------------
    def layout(self, R):
        return list(self.sink) + list(self.recent) + [self.bank[i] for i in R]

    def write_into_caches(self, caches_k, caches_v, R, offset=0):
        """Assembles sink | recent | bank[R] at tokens [offset, offset + tot) of
        every layer's cache (caches_k[l]: [B=1, cap, H, D] or [cap, H, D]) in one
        gather launch; returns tot (tokens)."""
        chunks = self.layout(R)
        tot = len(chunks) * self.ct
        if tot == 0:
            return 0
        nb = self.pool.chunk_bytes
        jobs = []
        for layer in range(self.n_layers):
            ck, cv = caches_k[layer], caches_v[layer]
            ck2 = ck[0] if ck.dim() == 4 else ck
            cv2 = cv[0] if cv.dim() == 4 else cv
            if offset + tot > ck2.shape[0]:
                raise RuntimeError(f"landmark active {tot} > cache capacity {ck2.shape[0]}")
            if not (ck2.is_contiguous() and cv2.is_contiguous()):
                raise ValueError("per-layer cache rows must be contiguous [cap, H, D]")
            row = ck2.stride(0) * ck2.element_size()
            for i, ch in enumerate(chunks):
                dst = (offset + i * self.ct) * row
                jobs.append((self.pool.ptr(ch.slot, layer, 0), ck2.data_ptr() + dst, nb))
                jobs.append((self.pool.ptr(ch.slot, layer, 1), cv2.data_ptr() + dst, nb))
        copy_jobs(jobs, self.device)
        return tot

    def stats(self, R):
        return dict(sink=len(self.sink), recent=len(self.recent), bank=len(self.bank),
                    attended=len(self.sink) + len(self.recent) + len(R),
                    pool_slots_used=self.pool.pool.shape[0] - len(self.pool.free),
                    pool_slots_total=self.pool.pool.shape[0])


class LandmarkCacheV2:
    """Per-layer drop-in for longctx/inference/landmark_cache_v2.py:413 LandmarkCacheV2.

    Same constructor (eps / diverse / hot_gpu / gpu_spare are accepted for
    compatibility and have no effect: there is no host tier) and the same
    methods.  K/V are device tensors; the pool is created at the first
    add_chunk from the chunk's shape."""

    def __init__(self, chunk_tokens, n_sink=1, recent_w=5, K=30, retrieve_k=6, eps=0.5, mode="b", diverse=False,
                 protect_n=2, hot_gpu=None, gpu_spare=None):
        _check_env()
        assert mode in ("a", "b")
        self.ct, self.n_sink, self.recent_w, self.K = chunk_tokens, n_sink, recent_w, K
        self.retrieve_k, self.mode, self.protect_n = retrieve_k, mode, protect_n
        self.eps, self.diverse = eps, diverse
        self._stack = None
        self.events = []

    def _ensure(self, k):
        if self._stack is None:
            ct, H, D = k.shape
            if ct != self.ct:
                raise ValueError(f"chunk has {ct} tokens, expected {self.ct}")
            self._stack = LandmarkBankStack(ct, 1, H, D, self.n_sink, self.recent_w, self.K, self.retrieve_k,
                                            self.mode, self.protect_n, device=k.device, dtype=k.dtype)
            self._stack.events = self.events

    @property
    def sink(self):
        return self._stack.sink if self._stack else []

    @property
    def recent(self):
        return self._stack.recent if self._stack else []

    @property
    def bank(self):
        return self._stack.bank if self._stack else []

    def add_chunk(self, k, v, pose, pose_next=None, phase_f=None):
        """k, v: [ct, H, D] device tensors; pose, pose_next: (4, 4).  Returns the
        retrieved bank indices for the next chunk (ascending)."""
        self._ensure(k)
        return self._stack.add_chunk_from([k.detach().contiguous()], [v.detach().contiguous()], pose, pose_next)

    def write_into_cache(self, kv_cache, R):
        if self._stack is None:
            return 0
        return self._stack.write_into_caches([kv_cache["k"]], [kv_cache["v"]], R)

    def active_layout(self, R):
        return self._stack.layout(R) if self._stack else []

    def get_active_kv(self, R):
        chunks = self.active_layout(R)
        if not chunks:
            return None, None, 0
        pool = self._stack.pool.pool
        k = torch.cat([pool[c.slot, 0, 0] for c in chunks], 0)
        v = torch.cat([pool[c.slot, 0, 1] for c in chunks], 0)
        return k, v, k.shape[0]

    def stats(self, R):
        if self._stack is None:
            return dict(sink=0, recent=0, bank=0, attended=0)
        return self._stack.stats(R)
