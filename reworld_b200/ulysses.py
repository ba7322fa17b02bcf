"""Ulysses sequence parallelism for the cached chunk attention (heads sharded).

Reference pattern: wan_5b/distributed/ulysses.py:17-55 distributed_attention —
all_to_all(q/k/v, scatter_dim=2 (heads), gather_dim=1 (sequence)) so each rank
holds the whole sequence for H/P heads, attention, then all_to_all(x,
scatter_dim=1, gather_dim=2) back; all_to_all itself is
wan_5b/distributed/util.py:52-64 (chunk + contiguous + dist.all_to_all + cat).
The reference has no cached-inference variant (sequence_parallel.py:550-551
raises); this module extends the pattern to the KV-cached chunk attention:
every rank keeps the KV cache, landmark pool and gather for its own H/P heads
(head-resident cache), so per chunk only the new q/k/v and the output cross
NVLink.

Exchange: one NCCL all_to_all_single over a contiguous buffer per tensor, with
the layout transforms done by the package's kernels (rw_a2a_pack /
rw_a2a_unpack) instead of chunk/contiguous/cat copies.
"""
import math
import torch
import torch.distributed as dist

from . import _native
from ._native import c_vp


def a2a_pack(x, P, out=None):
    """[B, Ls, H, D] -> [P, B, Ls, H/P, D] (block p = head group p)."""
    B, Ls, H, D = x.shape
    x = x.contiguous()
    if out is None:
        out = torch.empty((P, B, Ls, H // P, D), dtype=x.dtype, device=x.device)
    lib = _native.lib()
    with torch.cuda.device(x.device):
        code = lib.rw_a2a_pack(c_vp(x.data_ptr()), c_vp(out.data_ptr()), B, Ls, H, D, P,
                               _native.stream_ptr(x.device))
    _native.check(code, "rw_a2a_pack")
    return out


def a2a_unpack(blocks, H, out=None):
    """[P, B, Ls, H/P, D] (block p = head group p) -> [B, Ls, H, D]."""
    P, B, Ls, Hp, D = blocks.shape
    assert Hp * P == H
    blocks = blocks.contiguous()
    if out is None:
        out = torch.empty((B, Ls, H, D), dtype=blocks.dtype, device=blocks.device)
    lib = _native.lib()
    with torch.cuda.device(blocks.device):
        code = lib.rw_a2a_unpack(c_vp(blocks.data_ptr()), c_vp(out.data_ptr()), B, Ls, H, D, P,
                                 _native.stream_ptr(blocks.device))
    _native.check(code, "rw_a2a_unpack")
    return out


def exchange_blocks(send, group=None):
    """One all_to_all_single over a contiguous [P, ...] buffer: block p goes to
    rank p, and block p of the result came from rank p."""
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send.contiguous(), group=group)
    return recv


def blocks_to_seq(recv):
    """[P(src), B, Ls, H/P, D] received head-group blocks -> [B, P*Ls, H/P, D]
    (source rank p holds tokens [p*Ls, (p+1)*Ls))."""
    P, B, Ls, Hp, D = recv.shape
    return recv.permute(1, 0, 2, 3, 4).reshape(B, P * Ls, Hp, D)


def seq_to_blocks(x, P):
    """[B, L, H/P, D] -> [P(dst), B, L/P, H/P, D]: block p holds rank p's tokens
    (a view without copying when B = 1)."""
    B, L, Hp, D = x.shape
    return x.reshape(B, P, L // P, Hp, D).permute(1, 0, 2, 3, 4)


def seq_to_head(x, group=None):
    """util.all_to_all(x, scatter_dim=2, gather_dim=1): [B, L/P, H, D] -> [B, L, H/P, D].
    Rank r ends up with heads [r*H/P, (r+1)*H/P) for the whole sequence."""
    P = dist.get_world_size(group)
    if P == 1:
        return x
    return blocks_to_seq(exchange_blocks(a2a_pack(x, P), group))


def head_to_seq(x, H, group=None):
    """util.all_to_all(x, scatter_dim=1, gather_dim=2): [B, L, H/P, D] -> [B, L/P, H, D]."""
    P = dist.get_world_size(group)
    if P == 1:
        return x
    return a2a_unpack(exchange_blocks(seq_to_blocks(x, P), group), H)


def all_to_all(x, scatter_dim, gather_dim, group=None):
    """Drop-in for wan_5b/distributed/util.py:52-64 for the two uses of Ulysses
    ([B, L, H, D] tensors: heads -> sequence and back)."""
    if scatter_dim == 2 and gather_dim == 1:
        return seq_to_head(x, group)
    if scatter_dim == 1 and gather_dim == 2:
        P = dist.get_world_size(group)
        return head_to_seq(x, x.shape[2] * P, group)
    raise NotImplementedError("only the Ulysses (2,1) and (1,2) exchanges are supported")


def distributed_attention(q, k, v, seq_lens=None, window_size=(-1, -1), group=None):
    """Drop-in for wan_5b/distributed/ulysses.py:17-55 (non-cached): q/k/v
    sequence-sharded [B, L/P, H, D] in, output sequence-sharded out."""
    from .attention import attention
    H = q.shape[2]
    qh, kh, vh = seq_to_head(q, group), seq_to_head(k, group), seq_to_head(v, group)
    x = attention(qh, kh, vh, k_lens=seq_lens, window_size=window_size)
    return head_to_seq(x, H, group)


def sp_chunk_attention(q, k, v, cache_k, cache_v, dst_start, rope=None, group=None, out=None):
    """One layer of the cached chunk attention under Ulysses head parallelism.

    q, k, v: this rank's sequence shard [B, L/P, H, D] of the chunk (all heads);
    cache_k / cache_v: this rank's head-resident cache [B, cap, H/P, D] (heads
    [r*H/P, (r+1)*H/P)).  The chunk's q/k/v go seq -> head, the chunk's roped K
    and V are written into the local cache at dst_start, the chunk's queries
    attend cache[:, :dst_start + L] for the local heads (q's RoPE applied in the
    kernel), and the result goes head -> seq.  Returns [B, L/P, H, D].
    """
    from .attention import chunk_attention
    from .kv_cache import rope_kv_store
    H = q.shape[2]
    qh, kh, vh = seq_to_head(q, group), seq_to_head(k, group), seq_to_head(v, group)
    L = qh.shape[1]
    rope_kv_store(kh, vh, cache_k, cache_v, dst_start, rope=rope)
    o = chunk_attention(qh, cache_k[:, :dst_start + L], cache_v[:, :dst_start + L], rope=rope)
    res = head_to_seq(o, H, group)
    if out is not None:
        out.copy_(res)
        return out
    return res


def sp_chunk_attention_seq_kv(q, k, v, kv_k, kv_v, rope=None, group=None, work=None):
    """One layer of the cached chunk attention with the cache sharded along the
    sequence too (every rank holds a slice of the cached keys for all heads), the
    other way to lay the 12-chunk cache over P GPUs.

    q, k, v: this rank's sequence shard [B, L/P, H, D] of the chunk (all heads);
    kv_k / kv_v: this rank's slice [B, Lc/P, H, D] of the cached, already roped
    keys and values (rank r: cached keys [r*Lc/P, (r+1)*Lc/P), all heads).  Each
    call moves the cache seq -> head with the chunk's q/k/v (util.all_to_all's
    scatter_dim=2, gather_dim=1, as wan_5b/distributed/ulysses.py:40-45 does for
    q/k/v), so every rank then holds all Lc cached keys plus the chunk's roped
    keys for its H/P heads; attention over them (q's RoPE in the kernel); the
    output goes head -> seq.  Returns [B, L/P, H, D].  Compared with the
    head-resident cache (sp_chunk_attention, UlyssesP2P) every layer here also
    sends (P-1)/P of this rank's cache slice over NVLink.  work = (buf_k, buf_v),
    [B, >= Lc + L, H/P, D] key buffers reused across calls (allocated when None).
    """
    from .attention import chunk_attention
    from .kv_cache import rope_kv_store
    P = dist.get_world_size(group)
    B, Ls, H, D = q.shape
    Lcs = kv_k.shape[1]
    Lc, L, Hp = Lcs * P, Ls * P, H // P
    if kv_v.shape != kv_k.shape or kv_k.shape[0] != B or kv_k.shape[2] != H:
        raise ValueError("cache slices must be [B, Lc/P, H, D] like q's batch and heads")
    if work is None:
        work = tuple(torch.empty((B, Lc + L, Hp, D), dtype=torch.bfloat16, device=q.device) for _ in range(2))
    buf_k, buf_v = work
    if buf_k.shape[1] < Lc + L or buf_k.shape[2] != Hp or buf_v.shape != buf_k.shape:
        raise ValueError("work buffers must be [B, >= Lc + L, H/P, D]")
    qh = seq_to_head(q, group)
    for src, dst in ((kv_k, buf_k), (kv_v, buf_v)):
        if P == 1:
            dst[:, :Lc].copy_(src)
        elif B == 1 and dst.is_contiguous():
            # block p of the exchange = rank p's cached keys = rows [p*Lc/P, (p+1)*Lc/P) of
            # the buffer: received in place
            recv = dst[:, :Lc].view(P, 1, Lcs, Hp, D)
            dist.all_to_all_single(recv, a2a_pack(src, P), group=group)
        else:
            dst[:, :Lc].copy_(blocks_to_seq(exchange_blocks(a2a_pack(src, P), group)))
    kh, vh = seq_to_head(k, group), seq_to_head(v, group)
    rope_kv_store(kh, vh, buf_k, buf_v, Lc, rope=rope)
    o = chunk_attention(qh, buf_k[:, :Lc + L], buf_v[:, :Lc + L], rope=rope)
    return head_to_seq(o, H, group)


class UlyssesP2P:
    """Head-parallel cached chunk attention with the exchanges done by this
    package's kernels over peer memory (NVLink) instead of a collective library.

    Per layer, two launches: rw_sp_scatter_qkv (each rank writes its sequence
    shard's q into the owning rank's q buffer and its roped k and v straight into
    the owning rank's KV cache; its last CTA then signals every rank), and
    rw_sp_attn_fwd (every CTA first waits, bounded, for all ranks' scatter signals,
    then runs the chunk attention on the local heads over the local, head-resident
    cache; its epilogue stores every output row straight into the buffer of the
    rank that owns the token, and its last CTA — or the merge kernel's, when the
    key split needs one — signals every rank again).  The cross-rank ordering thus
    rides on the two kernels (no barrier launches).  The q and output buffers
    alternate between two copies from call to call: when a rank scatters call
    n + 2 into q copy n % 2, every rank has passed call n + 1's wait, i.e. finished
    call n's attention, so nothing still reads that copy.  `layer(...,
    sync_output=True)` adds a wait for every rank's output rows (rw_sp_wait) before
    returning; a caller that reads the output later calls `finish()` first.  The q
    buffers, output buffers, all layers' caches and the signal array are symmetric
    memory, so every rank holds the peers' device pointers.  One sequence (B = 1),
    as in the streaming rollout.
    """

    SLOT_SCATTER, SLOT_ATTN, SLOT_BARRIER = 0, 1, 2     # signal slots, in units of P

    def __init__(self, group, n_layers, cap_tokens, chunk_tokens, heads, head_dim=128, device=None,
                 barrier_timeout_ms=10000):
        import torch.distributed._symmetric_memory as symm
        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if heads % self.P or chunk_tokens % self.P:
            raise ValueError("heads and chunk tokens must divide by the number of ranks")
        self.H, self.Hp, self.D = heads, heads // self.P, head_dim
        self.L, self.Ls, self.cap, self.n_layers = chunk_tokens, chunk_tokens // self.P, cap_tokens, n_layers
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.timeout_ms = barrier_timeout_ms
        bf16 = torch.bfloat16
        self.caches = symm.empty(n_layers, 2, cap_tokens, self.Hp, head_dim, dtype=bf16, device=self.device)
        self.qbuf = symm.empty(2, chunk_tokens, self.Hp, head_dim, dtype=bf16, device=self.device)
        self.obuf = symm.empty(2, self.Ls, heads, head_dim, dtype=bf16, device=self.device)
        self.sig = symm.empty(4 * self.P, dtype=torch.int32, device=self.device)   # signal slots
        self.counters = torch.zeros(2, dtype=torch.int32, device=self.device)     # scatter, attention
        self.caches.zero_()
        self.sig.zero_()
        torch.cuda.synchronize(self.device)   # zeroed on every rank before any peer can signal into it
        self.h_c = symm.rendezvous(self.caches, group)
        self.h_s = symm.rendezvous(self.sig, group)
        self.sig_ptrs = torch.tensor(list(self.h_s.buffer_ptrs), dtype=torch.int64, device=self.device)
        self.epoch = 0
        self.h_q = symm.rendezvous(self.qbuf, group)
        self.h_o = symm.rendezvous(self.obuf, group)
        per_tensor = cap_tokens * self.Hp * head_dim * 2
        base = list(self.h_c.buffer_ptrs)
        ptrs = [[[b + (l * 2 + kv) * per_tensor for b in base] for kv in range(2)] for l in range(n_layers)]
        self.cache_ptrs = torch.tensor(ptrs, dtype=torch.int64, device=self.device)   # [layer, k/v, P]
        qsz, osz = self.qbuf[0].numel() * 2, self.obuf[0].numel() * 2
        self.q_ptrs = torch.tensor([[b + c * qsz for b in self.h_q.buffer_ptrs] for c in range(2)], dtype=torch.int64,
                                   device=self.device)                             # [copy, P]
        self.o_ptrs = torch.tensor([[b + c * osz for b in self.h_o.buffer_ptrs] for c in range(2)], dtype=torch.int64,
                                   device=self.device)

    def cache_k(self, layer):
        return self.caches[layer, 0].unsqueeze(0)

    def cache_v(self, layer):
        return self.caches[layer, 1].unsqueeze(0)

    def _sync(self, counter=None, wait_slot=0, wait_epoch=0, signal_slot=0, signal_epoch=0):
        return _native.RwSpSync(c_vp(self.sig_ptrs.data_ptr()),
                                c_vp(self.counters[counter].data_ptr()) if counter is not None else None,
                                self.P, self.rank, wait_slot * self.P, wait_epoch, signal_slot * self.P,
                                signal_epoch, self.timeout_ms, 0)

    def scatter_qkv(self, layer, q, k, v, dst_start, rope=None, copy=0, sync=None):
        """q, k, v: [1, Ls, H, D] bf16 (this rank's tokens, all heads)."""
        import ctypes
        lib = _native.lib()
        rs = rope.struct() if rope is not None else None
        st = _native.status_tensor(self.device)
        code = lib.rw_sp_scatter_qkv(
            c_vp(q.data_ptr()), c_vp(k.data_ptr()), c_vp(v.data_ptr()),
            q.stride(1), q.stride(2), k.stride(1), k.stride(2), v.stride(1), v.stride(2),
            c_vp(self.q_ptrs[copy].data_ptr()), c_vp(self.cache_ptrs[layer, 0].data_ptr()),
            c_vp(self.cache_ptrs[layer, 1].data_ptr()), self.Ls, self.H, self.D, self.P, self.rank,
            int(dst_start), self.cap, ctypes.byref(rs) if rs is not None else None,
            ctypes.byref(sync) if sync is not None else None, c_vp(st.data_ptr()), _native.stream_ptr(self.device))
        _native.check(code, "rw_sp_scatter_qkv")

    def barrier(self, slot_base=None):
        """Stream-ordered barrier of the group over the peer-mapped signal array
        (rw_sp_barrier); everything each rank enqueued before it is visible to all
        ranks after it."""
        if slot_base is None:
            slot_base = self.SLOT_BARRIER * self.P
        lib = _native.lib()
        st = _native.status_tensor(self.device)
        self.epoch += 1
        code = lib.rw_sp_barrier(c_vp(self.sig_ptrs.data_ptr()), slot_base, self.P, self.rank, self.epoch,
                                 self.timeout_ms, c_vp(st.data_ptr()), _native.stream_ptr(self.device))
        _native.check(code, "rw_sp_barrier")

    def attend(self, layer, lk, rope=None, copy=0, sync=None):
        """Attention of this rank's heads over cache rows [0, lk) with the output
        rows sent to their owner ranks' output buffers."""
        import ctypes
        from .attention import _workspace
        lib = _native.lib()
        q = self.qbuf[copy]
        kc, vc = self.caches[layer, 0], self.caches[layer, 1]
        rs = rope.struct() if rope is not None else None
        st = _native.status_tensor(self.device)
        ws = _workspace(self.device, lib.rw_attn_workspace_bytes(1, self.L, lk, self.Hp))
        code = lib.rw_sp_attn_fwd(
            c_vp(q.data_ptr()), c_vp(kc.data_ptr()), c_vp(vc.data_ptr()), self.L, lk, self.Hp, self.D,
            q.stride(0), q.stride(1), kc.stride(0), kc.stride(1), vc.stride(0), vc.stride(1),
            c_vp(self.o_ptrs[copy].data_ptr()), self.P, self.rank, self.H, 1.0 / math.sqrt(self.D),
            ctypes.byref(rs) if rs is not None else None,
            c_vp(ws.data_ptr()) if ws is not None else None, ws.numel() if ws is not None else 0,
            ctypes.byref(sync) if sync is not None else None, c_vp(st.data_ptr()), _native.stream_ptr(self.device))
        _native.check(code, "rw_sp_attn_fwd")

    def finish(self):
        """Waits on this rank's stream until every rank's output rows of the last
        layer() call have arrived (rw_sp_wait)."""
        if self.epoch == 0:
            return
        s = self._sync(wait_slot=self.SLOT_ATTN, wait_epoch=self.epoch)
        import ctypes
        st = _native.status_tensor(self.device)
        code = _native.lib().rw_sp_wait(ctypes.byref(s), c_vp(st.data_ptr()), _native.stream_ptr(self.device))
        _native.check(code, "rw_sp_wait")

    def layer(self, layer, q, k, v, dst_start, rope=None, attn_events=None, sync_output=True, scatter_events=None):
        """One layer's cached chunk attention; returns [1, Ls, H, D] (this rank's
        tokens, all heads), complete on return when sync_output, else after
        finish() (valid until the call after next, which reuses its copy).
        attn_events / scatter_events: optional CUDA event pairs recorded around the
        attention and the scatter launches."""
        for t in (q, k, v):
            if t.dtype != torch.bfloat16 or t.shape != (1, self.Ls, self.H, self.D) or t.stride(-1) != 1:
                raise ValueError("q, k, v must be bf16 [1, L/P, H, D] with a contiguous head dim")
        self.epoch += 1
        e, copy = self.epoch, self.epoch & 1
        if scatter_events is not None:
            scatter_events[0].record()
        self.scatter_qkv(layer, q, k, v, dst_start, rope, copy,
                         self._sync(counter=0, signal_slot=self.SLOT_SCATTER, signal_epoch=e))
        if scatter_events is not None:
            scatter_events[1].record()
        lk = dst_start + self.L
        if attn_events is not None:
            attn_events[0].record()
        self.attend(layer, lk, rope, copy,
                    self._sync(counter=1, wait_slot=self.SLOT_SCATTER, wait_epoch=e, signal_slot=self.SLOT_ATTN,
                               signal_epoch=e))
        if attn_events is not None:
            attn_events[1].record()
        if sync_output:
            self.finish()
        return self.obuf[copy].unsqueeze(0)
