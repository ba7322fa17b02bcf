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
