"""KV-cache write of the new chunk with the RoPE applied in the same pass.

Replaces wan_5b/modules/action_model.py:265-292 (apply_rope on q and the new k
at the chunk's start frame, then kv_cache["k"/"v"][:, local_start:local_end] =
k_f / v) with one launch of rw_rope_kv_store.
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
