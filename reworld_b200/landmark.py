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
free list, so by default every member stays resident in HBM (a 30-member bank
of the 5B model is 29 GB).  With host_tier=True the bank members' master copies
live in a pinned host pool instead, as in the reference's _TieredMemberStore
(landmark_cache_v2.py:137-411): write-through D2H on admission, an LRU hot set
of device slots, H2D prefetch of the retrieved members on a dedicated stream,
or (hot_gpu = 0) direct host-to-cache copies.
"""
import collections
import ctypes
import math
import os
import warnings
from typing import NamedTuple

import numpy as np
import torch

from . import _native
from ._native import c_vp

BANK_MAX = 1024


# ---------------------------------------------------------------- rollout-side sizing and poses
# kv_compression policies that run the landmark bank (compressed.py:302-306):
# policy -> (mode, diverse).  'a' attends the whole bank, 'b' retrieves top-k.
LANDMARK_POLICIES = {"consol": ("a", False), "consol_div": ("a", True), "v15a": ("a", False),
                     "v15b": ("b", False), "v15c": ("b", True)}


class BudgetSplit(NamedTuple):
    """How a KV budget of `budget` chunks is spent: sink + recent + landmarks."""
    budget: int          # effective budget (capped to what the cache holds)
    n_sink: int
    recent_w: int        # effective recent window
    n_landmark: int      # landmarks attended per chunk (retrieve_k)
    K: int               # bank capacity
    mode: str
    diverse: bool


def budget_split(budget_chunks, n_sink, recent_w, landmark_k=30, policy="v15b", cache_tokens=None,
                 chunk_tokens=None):
    """The compressed pipeline's budget split (pipeline/
    causal_diffusion_inference_compressed.py:273-282 and :302-322): the budget is
    capped to the chunks the pre-allocated cache holds (cache_tokens //
    chunk_tokens, when given); the recent window is capped so at least one
    landmark slot survives, eff_recent = min(recent_w, max(1, B - n_sink - 1));
    the landmarks fill the rest, n_landmark = max(1, B - n_sink - eff_recent);
    the bank holds K = max(landmark_k, n_landmark) for the top-k policies and
    exactly n_landmark for the attend-all ones.  Raises ValueError for a policy
    that does not use the landmark bank."""
    if policy not in LANDMARK_POLICIES:
        raise ValueError(f"policy {policy!r} does not use the landmark bank (one of {sorted(LANDMARK_POLICIES)})")
    mode, diverse = LANDMARK_POLICIES[policy]
    budget = int(budget_chunks)
    if cache_tokens is not None:
        if not chunk_tokens:
            raise ValueError("cache_tokens needs chunk_tokens")
        budget = min(budget, int(cache_tokens) // int(chunk_tokens))
    n_sink = int(n_sink)
    eff_recent = min(int(recent_w), max(1, budget - n_sink - 1))
    n_landmark = max(1, budget - n_sink - eff_recent)
    K = max(int(landmark_k), n_landmark) if mode == "b" else n_landmark
    return BudgetSplit(budget, n_sink, eff_recent, n_landmark, K, mode, diverse)


def chunk_pose(prope_ctx, num_frame_per_block):
    """One (4, 4) float32 pose for the chunk just generated, as the compressed
    pipeline's _compute_chunk_pose forms it (causal_diffusion_inference_
    compressed.py:355-377): the rotation of the chunk's first frame and the mean
    translation over its frames, from the last num_frame_per_block entries of
    prope_ctx [B, T_seen, 4, 4] (batch 0), in fp32 with numpy's reduction.  The
    pose is host data for the bank's decision (pose_record), so the few bytes
    are read back here as the reference reads them."""
    if prope_ctx is None:
        raise RuntimeError("chunk_pose: prope_context is None; the landmark bank needs the model's "
                           "camera context (use_prope)")
    cur = prope_ctx[0, -num_frame_per_block:].detach().to(torch.float32).cpu().numpy()
    out = np.eye(4, dtype=np.float32)
    out[:3, :3] = cur[0, :3, :3]
    out[:3, 3] = cur[:, :3, 3].mean(axis=0)
    return out


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
        return self.collect(self.issue(admit, target))

    def issue(self, admit=None, target=None):
        """Queues the decision (rw_bank_step) and the copy of its result to pinned
        host memory without waiting for either; returns the ticket that collect()
        turns into step()'s result.  Tickets are collected in the order issued."""
        recs = (RwPose * 2)()
        if admit is not None:
            recs[0] = pose_record(admit[0])
        if target is not None:
            recs[1] = pose_record(target)
        # pinned staging: the copy is queued without a host wait; the pinned block is
        # not reused before the copy has run (torch's pinned allocator records it)
        host = torch.empty(len(bytes(recs)), dtype=torch.uint8, pin_memory=True)
        host.numpy()[:] = np.frombuffer(bytes(recs), dtype=np.uint8)
        self.poses.copy_(host, non_blocking=True)
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
        host_res = torch.empty(self.result.numel(), dtype=torch.uint8, pin_memory=True)
        host_res.copy_(self.result, non_blocking=True)
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(self.device))
        return host_res, done, admit

    def collect(self, ticket):
        """Waits for an issued decision (only for it and the work queued before it)
        and applies it to the host mirror; returns (evicted, R, R_slots)."""
        host_res, done, admit = ticket
        done.synchronize()
        res = RwBankResult.from_buffer_copy(host_res.numpy().tobytes())
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
        self.ev = {}   # slot -> last event of a copy stream that read or wrote it (host tier)

    def acquire(self, stream=None):
        """A free slot; `stream` (the one that will write it) first waits for the
        slot's last use on a copy stream."""
        if not self.free:
            raise RuntimeError("chunk pool exhausted")
        slot = self.free.pop(0)
        ev = self.ev.get(slot)
        if ev is not None and stream is not None:
            stream.wait_event(ev)
        return slot

    def release(self, slot):
        self.free.append(slot)

    def ptr(self, slot, layer, kv):
        return self.pool[slot, layer, kv].data_ptr()


def copy_jobs(jobs, device, status=None):
    """Runs [(src_ptr, dst_ptr, nbytes), ...] with one rw_copy_chunks launch."""
    if not jobs:
        return
    # descriptors through pinned memory: the host-to-device copy is queued without
    # a host wait (torch's pinned allocator keeps the block until the copy ran)
    arr = torch.empty((len(jobs), 3), dtype=torch.int64, pin_memory=True)
    arr.numpy()[:] = np.asarray(jobs, dtype=np.int64).reshape(-1, 3)
    d = arr.to(device, non_blocking=True)
    st = status if status is not None else _native.status_tensor(torch.device(device))
    lib = _native.lib()
    with torch.cuda.device(device):
        code = lib.rw_copy_chunks(c_vp(d.data_ptr()), len(jobs), c_vp(st.data_ptr()), _native.stream_ptr(device))
    _native.check(code, "rw_copy_chunks")
    # `d` is released to the caching allocator on this stream, so it cannot be
    # reused before the copy kernel (queued earlier on the same stream) has read it.


def _available_ram():
    try:
        import psutil
        return psutil.virtual_memory().available
    except Exception:  # noqa: BLE001 - no psutil / no /proc: no cap
        return None


def host_pool(n_slots, member_shape, dtype):
    """Pinned host pool [n, *member_shape] for the tiered bank, sized as the
    reference sizes its host tier (landmark_cache_v2.py:176-203): at most half of
    the free RAM, and halved while a pinned allocation fails; when even one pinned
    slot cannot be had, one pageable slot (the reference's last resort: its copies
    then block the host).  The returned pool's length is the bank capacity that
    fits (the caller lowers K to it)."""
    member_bytes = int(np.prod(member_shape)) * torch.empty((), dtype=dtype).element_size()
    n = int(n_slots)
    avail = _available_ram()
    if avail is not None and member_bytes * n > 0.5 * avail:
        n = max(1, int((0.5 * avail) // max(member_bytes, 1)))
        warnings.warn(f"[tiered-store] host pool capped by free RAM: {n_slots} -> {n} slots")
    pin = True
    while True:
        try:
            return torch.empty((n,) + tuple(member_shape), dtype=dtype, pin_memory=pin)
        except RuntimeError:
            if pin and n > 1:
                n //= 2
                warnings.warn(f"[tiered-store] pinned alloc failed, retry with {n} slots")
            elif pin:
                pin = False
                warnings.warn("[tiered-store] pinned alloc impossible; pageable host memory + blocking copies")
            else:
                raise


class _HostTier:
    """Pinned host master copies of the bank members and the device hot set.

    Same protocol as the reference's _TieredMemberStore
    (longctx/inference/landmark_cache_v2.py:137-411): put = write-through D2H on
    a dedicated stream, the admitted chunk's device slot kept as a warm hot
    entry; prefetch = H2D of misses on a second stream into device slots, each
    transfer tracked by an event; an LRU hot set of hot_capacity members (the
    host copy is the master, so dropping a hot entry needs no copy back);
    hot_capacity 0 = direct mode (members go host -> cache rows on the compute
    stream).  A member is one contiguous [n_layers, 2, ct, H, D] block on both
    sides, so each transfer is one cudaMemcpyAsync.  No CPU waits: every reuse of
    a host or device slot is ordered by events."""

    def __init__(self, n_slots, pool, hot_capacity):
        member = tuple(pool.pool.shape[1:])
        self.host = host_pool(n_slots, member, pool.pool.dtype)
        self.pool = pool
        self.hot_capacity = hot_capacity
        self.free = collections.deque(range(self.host.shape[0]))
        self.m2s = {}                          # member id -> host slot
        self.slot_ev = {}                      # host slot -> last transfer event touching it
        self.master_ev = {}                    # member id -> write-through event
        self.fetch_ev = {}                     # member id -> H2D event of its hot copy
        self.hot = collections.OrderedDict()   # member id -> device slot, LRU first
        dev = pool.pool.device
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.member_bytes = pool.pool[0].numel() * pool.pool.element_size()
        self.counters = dict(hits=0, misses=0, warm_inserts=0, hot_evictions=0, bytes_h2d=0, bytes_d2h=0,
                             waits_pending=0)

    @property
    def slots_in_use(self):
        return self.host.shape[0] - len(self.free)

    def _hot_insert(self, mid, dslot):
        old = self.hot.pop(mid, None)
        if old is not None and old != dslot:
            self.pool.release(old)
        self.hot[mid] = dslot
        while len(self.hot) > self.hot_capacity:
            _, s = self.hot.popitem(last=False)
            self.counters["hot_evictions"] += 1
            self.pool.release(s)               # host is master: no copy back

    def put(self, mid, dslot):
        """Admits member mid from device slot dslot (written on the compute stream)."""
        if not self.free:
            raise RuntimeError("host tier: no free slot (evict a bank member first)")
        hs = self.free.popleft()
        comp = torch.cuda.current_stream(self.pool.pool.device)
        self.d2h.wait_stream(comp)                      # the chunk is fully packed
        prev = self.slot_ev.get(hs)
        if prev is not None:
            self.d2h.wait_event(prev)                   # last read of the host slot is done
        with torch.cuda.stream(self.d2h):
            self.host[hs].copy_(self.pool.pool[dslot], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.d2h)
        self.slot_ev[hs] = ev
        self.master_ev[mid] = ev
        self.pool.ev[dslot] = ev                        # the next writer of dslot waits for this read
        self.m2s[mid] = hs
        self.counters["bytes_d2h"] += self.member_bytes
        if self.hot_capacity > 0:
            self._hot_insert(mid, dslot)                # warm: the original device copy
            self.counters["warm_inserts"] += 1
        else:
            self.pool.release(dslot)

    def free_member(self, mid):
        """Bank eviction: the host slot returns to the free list (its next writer
        waits for its last transfer) and a hot copy is dropped."""
        self.free.append(self.m2s.pop(mid))
        self.master_ev.pop(mid, None)
        self.fetch_ev.pop(mid, None)
        s = self.hot.pop(mid, None)
        if s is not None:
            self.pool.release(s)

    def prefetch(self, mids):
        """H2D of the members not in the hot set, on the h2d stream; returns at once."""
        if self.hot_capacity <= 0:
            return
        comp = torch.cuda.current_stream(self.pool.pool.device)
        waited = False
        for mid in mids:
            if mid in self.hot:
                self.hot.move_to_end(mid)
                self.counters["hits"] += 1
                continue
            self.counters["misses"] += 1
            if not waited:
                self.h2d.wait_stream(comp)              # reads of recycled device slots queued so far
                waited = True
            ds = self.pool.acquire(self.h2d)
            hs = self.m2s[mid]
            mev = self.master_ev.get(mid)
            if mev is not None:
                self.h2d.wait_event(mev)                # the master copy has landed
            with torch.cuda.stream(self.h2d):
                self.pool.pool[ds].copy_(self.host[hs], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.h2d)
            self.slot_ev[hs] = ev
            self.pool.ev[ds] = ev
            self.fetch_ev[mid] = ev
            self._hot_insert(mid, ds)
            self.counters["bytes_h2d"] += self.member_bytes

    def device_slot(self, mid):
        """The hot copy's device slot, with the compute stream ordered after its fetch."""
        ev = self.fetch_ev.pop(mid, None)
        if ev is not None:
            if not ev.query():
                self.counters["waits_pending"] += 1
            torch.cuda.current_stream(self.pool.pool.device).wait_event(ev)
        self.hot.move_to_end(mid)
        return self.hot[mid]

    def copy_to_rows(self, mid, layer, dst_k, dst_v):
        """Direct mode: one member's K and V of one layer from the host slot into
        cache rows, on the compute stream."""
        comp = torch.cuda.current_stream(self.pool.pool.device)
        mev = self.master_ev.get(mid)
        if mev is not None:
            comp.wait_event(mev)
        hs = self.m2s[mid]
        dst_k.copy_(self.host[hs, layer, 0], non_blocking=True)
        dst_v.copy_(self.host[hs, layer, 1], non_blocking=True)

    def mark_read(self, mids):
        """After direct copies on the compute stream: the next write-through into
        these members' host slots waits for them."""
        if not mids:
            return
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.pool.pool.device))
        for mid in mids:
            self.slot_ev[self.m2s[mid]] = ev
            self.counters["misses"] += 1
            self.counters["bytes_h2d"] += self.member_bytes

    def stats(self):
        d = dict(host_slots_used=self.slots_in_use, host_slots_total=self.host.shape[0], pinned=bool(self.host.is_pinned()),
                 hot=len(self.hot), hot_capacity=self.hot_capacity)
        d.update({f"io_{k}": v for k, v in self.counters.items()})
        return d


class LandmarkBankStack:
    """Landmark bank shared by all layers (one decision per chunk, one gather
    launch for every layer).  Same policy as LandmarkCacheV2: sink chunks,
    a recent window of recent_w chunks, an always-admit bank of capacity K with
    protect-earliest-protect_n + most-redundant eviction and top-retrieve_k
    pose retrieval (mode 'b') or the whole bank (mode 'a')."""

    def __init__(self, chunk_tokens, n_layers, num_heads, head_dim, n_sink=1, recent_w=5, K=30, retrieve_k=6,
                 mode="b", protect_n=2, device="cuda", dtype=torch.bfloat16, host_tier=False, hot_gpu=None,
                 gpu_spare=None):
        """host_tier=True keeps the bank members' master copies in pinned host
        memory (the reference's tiered store): hot_gpu None or 0 = direct mode
        (members copied host -> cache rows each chunk, no device copies of the
        bank); hot_gpu > 0 = an LRU hot set of max(hot_gpu, retrieve_k) device
        slots plus gpu_spare (default retrieve_k) staging slots, filled by H2D
        prefetch right after each decision."""
        _check_env()
        assert mode in ("a", "b")
        self.ct, self.n_layers, self.H, self.D = chunk_tokens, n_layers, num_heads, head_dim
        self.n_sink, self.recent_w, self.K, self.retrieve_k, self.mode = n_sink, recent_w, K, retrieve_k, mode
        self.protect_n = protect_n
        self.device = torch.device(device)
        self.tier = None
        if host_tier:
            hot = 0 if not hot_gpu or int(hot_gpu) <= 0 else max(int(hot_gpu), retrieve_k)
            spare = 0 if hot == 0 else (int(gpu_spare) if gpu_spare is not None else retrieve_k)
            n_dev = n_sink + recent_w + 1 + hot + max(spare, 1 if hot else 0)
        else:
            n_dev = n_sink + recent_w + K + 1
        self.pool = _ChunkPool(n_dev, n_layers, chunk_tokens, num_heads, head_dim, self.device, dtype)
        if host_tier:
            self.tier = _HostTier(K, self.pool, hot)
            if self.tier.host.shape[0] < K:   # the host pool was capped: keep the capacity honest
                K = self.K = self.tier.host.shape[0]
                if K < retrieve_k:
                    raise RuntimeError(f"host memory holds only {K} bank members, fewer than the "
                                       f"{retrieve_k} landmarks retrieved per chunk")
        self.dec = DeviceBankDecisions(K, retrieve_k, mode, protect_n, self.device)
        self.sink, self.recent, self.bank = [], [], []
        self.events = []
        self._n = 0
        self._pending = None   # a decision queued by prepare() for chunk self._n

    @classmethod
    def from_budget(cls, chunk_tokens, n_layers, num_heads, head_dim, budget_chunks, n_sink=1, recent_w=5,
                    landmark_k=30, policy="v15b", cache_tokens=None, **kw):
        """The bank the compressed pipeline builds for a KV budget (budget_split:
        sink, effective recent window, retrieve_k = n_landmark, bank capacity K,
        mode from the policy); `split` on the result records the split."""
        sp = budget_split(budget_chunks, n_sink, recent_w, landmark_k, policy, cache_tokens, chunk_tokens)
        st = cls(chunk_tokens, n_layers, num_heads, head_dim, n_sink=sp.n_sink, recent_w=sp.recent_w, K=sp.K,
                 retrieve_k=sp.n_landmark, mode=sp.mode, **kw)
        st.split = sp
        return st

    # -- chunk admission ----------------------------------------------------
    def _aging_out(self):
        """The recent-window entry that leaves the window when the next chunk joins."""
        if self._n < self.n_sink or len(self.recent) + 1 <= self.recent_w:
            return None
        return self.recent[0]

    def prepare(self, pose, pose_next=None):
        """Queues the bank decision of the next add_chunk_from (same pose and
        pose_next) ahead of time: the decision depends only on poses and bank
        membership, not on the chunk's K/V, so it can run before the forwards that
        produce them, and add_chunk_from then finds its result on the host instead
        of waiting for the device to drain.  Optional; the results are the same."""
        if self._pending is not None:
            raise RuntimeError("a prepared bank decision is still pending")
        admit = self._aging_out()
        target = pose_next if pose_next is not None else pose
        ticket = self.dec.issue(admit=(admit.pose, admit.born, admit.slot) if admit is not None else None,
                                target=target if self.mode == "b" else None)
        self._pending = (self._n, bytes(pose_record(target)), admit, ticket)

    def add_chunk_from(self, src_k, src_v, pose, pose_next=None):
        """src_k/src_v: per-layer lists of [ct, H, D] views (e.g. the cache rows
        the chunk was just written to).  Packs them into a pool slot (one launch)
        and runs the bank decision.  Returns R (bank indices, ascending)."""
        c = self._n
        self._n += 1
        slot = self.pool.acquire(torch.cuda.current_stream(self.device))
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
        if self._pending is not None:
            pc, ptarget, padmit, ticket = self._pending
            self._pending = None
            if pc != c or padmit is not admit or ptarget != bytes(pose_record(target)):
                raise RuntimeError("the prepared bank decision was for another chunk or pose")
            evicted, R, _ = self.dec.collect(ticket)
        else:
            evicted, R, _ = self.dec.step(
                admit=(admit.pose, admit.born, admit.slot) if admit is not None else None,
                target=target if self.mode == "b" else None)
        for born, slot_ev in evicted:
            j = [m.born for m in self.bank].index(born)
            self.bank.pop(j)
            if self.tier is not None:
                self.tier.free_member(born)
            else:
                self.pool.release(slot_ev)
            self.events.append(("evict", born))
        if admit is not None:
            admit.protected = self.dec._admitted <= self.protect_n
            if self.tier is not None:
                self.tier.put(admit.born, admit.slot)   # the device slot now belongs to the tier
                admit.slot = None
            self.bank.append(admit)
            self.events.append(("add", admit.born, len(self.bank)))
        if self.tier is not None:
            self.tier.prefetch([self.bank[i].born for i in R])   # overlaps the next chunk's compute
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
        # device slot of every chunk; None = a bank member read from the host tier (direct mode)
        slots = [ch.slot for ch in chunks]
        if self.tier is not None:
            for i, ch in enumerate(chunks):
                if ch.slot is None and self.tier.hot_capacity > 0:
                    slots[i] = self.tier.device_slot(ch.born)
        jobs, direct = [], []
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
                if slots[i] is None:
                    r0 = offset + i * self.ct
                    direct.append((ch.born, layer, ck2[r0:r0 + self.ct], cv2[r0:r0 + self.ct]))
                    continue
                jobs.append((self.pool.ptr(slots[i], layer, 0), ck2.data_ptr() + dst, nb))
                jobs.append((self.pool.ptr(slots[i], layer, 1), cv2.data_ptr() + dst, nb))
        copy_jobs(jobs, self.device)
        for born, layer, dk, dv in direct:
            self.tier.copy_to_rows(born, layer, dk, dv)
        if direct:
            self.tier.mark_read(sorted({d[0] for d in direct}))
        return tot

    def stats(self, R):
        d = dict(sink=len(self.sink), recent=len(self.recent), bank=len(self.bank),
                 attended=len(self.sink) + len(self.recent) + len(R),
                 pool_slots_used=self.pool.pool.shape[0] - len(self.pool.free),
                 pool_slots_total=self.pool.pool.shape[0])
        if self.tier is not None:
            d.update(self.tier.stats())
        return d


class LandmarkCacheV2:
    """Per-layer drop-in for longctx/inference/landmark_cache_v2.py:413 LandmarkCacheV2.

    Same constructor (eps / diverse are accepted for compatibility and have no
    effect, as in the reference's v2) and the same methods.  K/V are device
    tensors; the pool is created at the first add_chunk from the chunk's shape.
    By default every bank member stays in HBM.  host_tier=True selects the
    reference's tiered store: hot_gpu / gpu_spare (or BANKV2_HOT_GPU /
    BANKV2_GPU_SPARE, read as the reference reads them,
    landmark_cache_v2.py:431-451) choose direct mode (hot_gpu None or 0) or the
    staged hot set."""

    def __init__(self, chunk_tokens, n_sink=1, recent_w=5, K=30, retrieve_k=6, eps=0.5, mode="b", diverse=False,
                 protect_n=2, hot_gpu=None, gpu_spare=None, host_tier=False):
        _check_env()
        assert mode in ("a", "b")
        self.ct, self.n_sink, self.recent_w, self.K = chunk_tokens, n_sink, recent_w, K
        self.retrieve_k, self.mode, self.protect_n = retrieve_k, mode, protect_n
        self.eps, self.diverse = eps, diverse
        if host_tier:
            if hot_gpu is None and os.environ.get("BANKV2_HOT_GPU"):
                hot_gpu = int(os.environ["BANKV2_HOT_GPU"])
            if gpu_spare is None and os.environ.get("BANKV2_GPU_SPARE"):
                gpu_spare = int(os.environ["BANKV2_GPU_SPARE"])
        self.host_tier, self.hot_gpu, self.gpu_spare = host_tier, hot_gpu, gpu_spare
        self._stack = None
        self.events = []

    def _ensure(self, k):
        if self._stack is None:
            ct, H, D = k.shape
            if ct != self.ct:
                raise ValueError(f"chunk has {ct} tokens, expected {self.ct}")
            self._stack = LandmarkBankStack(ct, 1, H, D, self.n_sink, self.recent_w, self.K, self.retrieve_k,
                                            self.mode, self.protect_n, device=k.device, dtype=k.dtype,
                                            host_tier=self.host_tier, hot_gpu=self.hot_gpu,
                                            gpu_spare=self.gpu_spare)
            self._stack.events = self.events
            self.K = self._stack.K             # lowered when the host pool was capped

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
        st = self._stack
        pool = st.pool.pool
        parts = []
        for c in chunks:
            if c.slot is not None:
                parts.append(pool[c.slot, 0])
            elif st.tier.hot_capacity > 0:
                parts.append(pool[st.tier.device_slot(c.born), 0])
            else:
                mev = st.tier.master_ev.get(c.born)
                if mev is not None:
                    torch.cuda.current_stream(st.device).wait_event(mev)
                parts.append(st.tier.host[st.tier.m2s[c.born], 0].to(st.device, non_blocking=True))
        k = torch.cat([p_[0] for p_ in parts], 0)
        v = torch.cat([p_[1] for p_ in parts], 0)
        if st.tier is not None and st.tier.hot_capacity == 0:
            st.tier.mark_read([c.born for c in chunks if c.slot is None])
        return k, v, k.shape[0]

    def stats(self, R):
        if self._stack is None:
            return dict(sink=0, recent=0, bank=0, attended=0)
        return self._stack.stats(R)
