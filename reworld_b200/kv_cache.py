"""KV-cache write of the new chunk with the RoPE (and the q/k RMSNorm) applied in the same pass.

Replaces wan_5b/modules/action_model.py:265-292 (apply_rope on q and the new k
at the chunk's start frame, then kv_cache["k"/"v"][:, local_start:local_end] =
k_f / v) with one launch of rw_rope_kv_store; qkv_norm_rope_store also takes in
the RMSNorm of q and k (action_model.py:164-166) and launches
rw_qkv_norm_rope_store.
"""
import ctypes

import torch

from . import _native
from ._native import c_vp


def _ok(t):
    return t.dtype == torch.bfloat16 and t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and \
        all(s % 8 == 0 for s in t.stride()[:-1])


def rope_kv_store(k, v, cache_k, cache_v, dst_start, rope=None, q=None, q_out=None):
    """cache_k[:, dst_start:dst_start+L] = rope(k); cache_v[...] = v; optionally
    q_out = rope(q).  k, v, q: [B, L, H, 128] bf16; caches [B, cap, H, 128] bf16."""
    B, L, H, D = k.shape
    if v.shape != k.shape or cache_k.shape[0] != B or cache_k.shape[2:] != (H, D) or cache_v.shape != cache_k.shape:
        raise ValueError("shape mismatch between k/v and the cache")
    if dst_start < 0 or dst_start + L > cache_k.shape[1]:
        raise RuntimeError(f"cache write [{dst_start}, {dst_start + L}) exceeds capacity {cache_k.shape[1]}")
    if not (_ok(cache_k) and _ok(cache_v)):
        raise ValueError("caches must be bf16 with a contiguous head dim")
    k = k if _ok(k) else k.to(torch.bfloat16).contiguous()
    v = v if _ok(v) else v.to(torch.bfloat16).contiguous()
    if q is not None:
        q = q if _ok(q) else q.to(torch.bfloat16).contiguous()
        if q_out is None:
            q_out = torch.empty_like(q)
    rs = rope.struct() if rope is not None else None
    z = (0, 0, 0)
    lib = _native.lib()
    with torch.cuda.device(k.device):
        code = lib.rw_rope_kv_store(
            c_vp(k.data_ptr()), c_vp(v.data_ptr()),
            c_vp(q.data_ptr()) if q is not None else None, c_vp(q_out.data_ptr()) if q is not None else None,
            c_vp(cache_k.data_ptr()), c_vp(cache_v.data_ptr()), B, L, H, D, int(dst_start),
            *k.stride()[:3], *v.stride()[:3],
            *(q.stride()[:3] if q is not None else z), *(q_out.stride()[:3] if q is not None else z),
            *cache_k.stride()[:3], *cache_v.stride()[:3],
            ctypes.byref(rs) if rs is not None else None, _native.stream_ptr(k.device))
    _native.check(code, "rw_rope_kv_store")
    return q_out


def _rows_ok(t):
    return t.dtype == torch.bfloat16 and t.dim() == 3 and t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and \
        all(s % 8 == 0 for s in t.stride()[:-1])


def qkv_norm_rope_store(q, k, v, w_q, w_k, cache_k, cache_v, dst_start, eps_q, eps_k=None, rope=None,
                        q_out=None):
    """RMSNorm of the projected q and k rows over all heads (WanRMSNorm,
    wan_5b/modules/model.py:73-89, as norm_q / norm_k at
    wan_5b/modules/action_model.py:164-166), RoPE of k, and the cache write of k
    and v (:265-292), in one launch of rw_qkv_norm_rope_store.

    q, k, v: bf16 [B, L, H*128] (e.g. column slices of one fused q|k|v
    projection); w_q, w_k, eps_q, eps_k: the two norms' weights [H*128] and
    epsilons (eps_k defaults to eps_q); caches [B, cap, H, 128] bf16.  Returns q_out = rmsnorm(q) * w_q as [B, L, H, 128] (without RoPE).
    """
    B, L, C = q.shape
    H, D = cache_k.shape[2], cache_k.shape[3]
    if k.shape != q.shape or v.shape != q.shape or C != H * D:
        raise ValueError(f"q/k/v rows {tuple(q.shape)} {tuple(k.shape)} {tuple(v.shape)} do not match "
                         f"the cache heads {H}x{D}")
    if cache_k.shape[0] != B or cache_v.shape != cache_k.shape:
        raise ValueError("shape mismatch between the rows and the cache")
    if dst_start < 0 or dst_start + L > cache_k.shape[1]:
        raise RuntimeError(f"cache write [{dst_start}, {dst_start + L}) exceeds capacity {cache_k.shape[1]}")
    if not (_ok(cache_k) and _ok(cache_v)):
        raise ValueError("caches must be bf16 with a contiguous head dim")
    q, k, v = (t if _rows_ok(t) else t.to(torch.bfloat16).contiguous() for t in (q, k, v))
    if w_q.dtype != torch.bfloat16 or w_k.dtype != torch.bfloat16:
        raise ValueError("norm weights must be bf16 (the module's dtype)")
    w_q, w_k = w_q.detach().contiguous(), w_k.detach().contiguous()
    if w_q.numel() != C or w_k.numel() != C:
        raise ValueError("norm weights must have H*D elements")
    if q_out is None:
        q_out = torch.empty((B, L, H, D), dtype=torch.bfloat16, device=q.device)
    elif not (_ok(q_out) and q_out.shape == (B, L, H, D)):
        raise ValueError("q_out must be a bf16 [B, L, H, D] tensor with a contiguous head dim")
    if rope is not None and rope.delta_cs is not None and rope.delta_cs.shape[0] < B:
        raise ValueError("the PM-RoPE phase needs one row per batch element")
    rs = rope.struct() if rope is not None else None
    lib = _native.lib()
    with torch.cuda.device(q.device):
        code = lib.rw_qkv_norm_rope_store(
            c_vp(q.data_ptr()), c_vp(k.data_ptr()), c_vp(v.data_ptr()), c_vp(w_q.data_ptr()),
            c_vp(w_k.data_ptr()), c_vp(q_out.data_ptr()), c_vp(cache_k.data_ptr()), c_vp(cache_v.data_ptr()),
            B, L, H, D, int(dst_start), float(eps_q), float(eps_q if eps_k is None else eps_k),
            *q.stride()[:2], *k.stride()[:2], *v.stride()[:2], *q_out.stride()[:3],
            *cache_k.stride()[:3], *cache_v.stride()[:3],
            ctypes.byref(rs) if rs is not None else None, c_vp(_native.status_tensor(q.device).data_ptr()),
            _native.stream_ptr(q.device))
    _native.check(code, "rw_qkv_norm_rope_store")
    return q_out
