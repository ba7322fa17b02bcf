"""Chunk attention: drop-in for the reference's `attention()` on the cached chunk.

`attention(q, k, v, ...)` has the signature and argument meaning of
wan_5b/modules/attention.py:133-179 and returns [B, Lq, H, D] in q's dtype, as
the reference's flash-attention branch does (:127-130).  The computation is the
package's tcgen05 kernel (rw_attn_fwd); there is no other backend.
"""
import ctypes
import math

import torch

from . import _native
from ._native import RwRope, c_vp


def _strides_ok(t):
    return t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 16 == 0


def _prep(t):
    if t.dtype != torch.bfloat16:
        t = t.to(torch.bfloat16)
    if not _strides_ok(t):
        t = t.contiguous()
    return t


_workspaces = {}


def _workspace(device, nbytes):
    """Per-device scratch for the key-split tail of the attention kernel (grown on demand)."""
    if nbytes <= 0:
        return None
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[idx] = ws
    return ws


def chunk_attention(q, k, v, softmax_scale=None, rope=None, out=None, se3=None):
    """softmax(q k^T * scale) v over every key (no mask), bf16, fp32 accumulation.

    q: [B, Lq, H, 128]; k, v: [B, Lk, H, 128] (any strides with a contiguous head
    dim, e.g. kv_cache["k"][:, :local_end]).  `rope` (a RopeArgs) applies the
    3-D RoPE (+ PM-RoPE phase) to q inside the kernel.  Returns bf16 [B, Lq, H, 128].

    se3 = (mats, frame_seqlen, po): the kernel also writes po = P y, the PRoPE
    O-side transform of its output (mats: fp32 [B, Lq / frame_seqlen, 4, 4]; po:
    bf16 [B, Lq, H, 128], e.g. the right half of the [y | P y] rows), as
    rw_se3_block_apply would from y (rw_attn_fwd_prope).
    """
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("chunk_attention runs on CUDA tensors only")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be [B, L, H, D]")
    B, Lq, H, D = q.shape
    if k.shape[0] != B or v.shape != k.shape or k.shape[2] != H or k.shape[3] != D:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    Lk = k.shape[1]
    q, k, v = _prep(q), _prep(k), _prep(v)
    if out is None:
        out = torch.empty((B, Lq, H, D), dtype=torch.bfloat16, device=q.device)
    elif out.dtype != torch.bfloat16 or out.shape != (B, Lq, H, D) or not _strides_ok(out):
        raise ValueError("out must be a bf16 [B, Lq, H, D] tensor with a contiguous head dim")
    scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(D)
    rope_struct = rope.struct() if rope is not None else None
    lib = _native.lib()
    if se3 is not None:
        mats, fs, po = se3
        if mats.dtype != torch.float32 or not mats.is_contiguous() or mats.device != q.device or \
                mats.shape != (B, Lq // int(fs), 4, 4) or Lq % int(fs) != 0:
            raise ValueError("se3 matrices must be fp32 [B, Lq / frame_seqlen, 4, 4] on q's device")
        if po.dtype != torch.bfloat16 or po.shape != (B, Lq, H, D) or not _strides_ok(po):
            raise ValueError("se3 output must be a bf16 [B, Lq, H, D] tensor with a contiguous head dim")
    with torch.cuda.device(q.device):
        st = _native.status_tensor(q.device)
        ws = _workspace(q.device, lib.rw_attn_workspace_bytes(B, Lq, Lk, H))
        common = (B, Lq, Lk, H, D,
                  q.stride(0), q.stride(1), q.stride(2),
                  k.stride(0), k.stride(1), k.stride(2),
                  v.stride(0), v.stride(1), v.stride(2),
                  out.stride(0), out.stride(1), out.stride(2))
        tail = (scale, ctypes.byref(rope_struct) if rope_struct is not None else None,
                c_vp(ws.data_ptr()) if ws is not None else None, ws.numel() if ws is not None else 0,
                c_vp(st.data_ptr()), _native.stream_ptr(q.device))
        if se3 is None:
            name = "rw_attn_fwd"
            code = lib.rw_attn_fwd(c_vp(q.data_ptr()), c_vp(k.data_ptr()), c_vp(v.data_ptr()),
                                   c_vp(out.data_ptr()), *common, *tail)
        else:
            name = "rw_attn_fwd_prope"
            code = lib.rw_attn_fwd_prope(c_vp(q.data_ptr()), c_vp(k.data_ptr()), c_vp(v.data_ptr()),
                                         c_vp(out.data_ptr()), c_vp(po.data_ptr()), c_vp(mats.data_ptr()), int(fs),
                                         *common, po.stride(0), po.stride(1), po.stride(2), *tail)
    _native.check(code, name)
    return out


def attention(q, k, v, q_lens=None, k_lens=None, dropout_p=0., softmax_scale=None, q_scale=None,
              causal=False, window_size=(-1, -1), deterministic=False, dtype=torch.bfloat16,
              fa_version=None):
    """Drop-in for wan_5b/modules/attention.py:133 `attention` (cached-chunk use).

    q: [B, Lq, Nq, C], k/v: [B, Lk, Nk, C].  Inputs that are not fp16/bf16 are
    cast to bf16 (the reference casts them to `dtype`); the result is returned
    in q's dtype like the reference's flash-attention branch.  k_lens restricts
    each batch element to its first k_lens[b] keys.  Options the cached-chunk
    call never uses (dropout, causal masking, sliding windows, ragged q_lens)
    raise NotImplementedError instead of silently computing something else.
    """
    half_dtypes = (torch.float16, torch.bfloat16)
    assert dtype in half_dtypes
    assert q.device.type == "cuda" and q.size(-1) <= 256
    if dropout_p:
        raise NotImplementedError("dropout is not supported by the chunk-attention kernel")
    if causal:
        raise NotImplementedError("causal masking is not supported (the cached chunk attends all keys)")
    if tuple(window_size) != (-1, -1):
        raise NotImplementedError("sliding-window attention is not supported")
    if k.size(2) != q.size(2):
        raise NotImplementedError("grouped-query attention (Nk != Nq) is not supported")
    b, lq = q.size(0), q.size(1)
    out_dtype = q.dtype
    if q_lens is not None:
        ql = torch.as_tensor(q_lens).tolist()
        if any(int(x) != lq for x in ql):
            raise NotImplementedError("ragged q_lens are not supported")
    if q_scale is not None:
        q = q * q_scale
    if k_lens is None:
        out = chunk_attention(q, k, v, softmax_scale=softmax_scale)
    else:
        kl = [int(x) for x in torch.as_tensor(k_lens).tolist()]
        if len(set(kl)) == 1:
            # one length for the whole batch (padded text contexts): one launch over the
            # leading keys of every element
            out = chunk_attention(q, k[:, :kl[0]], v[:, :kl[0]], softmax_scale=softmax_scale)
        else:
            out = torch.empty((b, lq, q.size(2), q.size(3)), dtype=torch.bfloat16, device=q.device)
            for i in range(b):
                chunk_attention(q[i:i + 1], k[i:i + 1, :kl[i]], v[i:i + 1, :kl[i]], softmax_scale=softmax_scale,
                                out=out[i:i + 1])
    return out.type(out_dtype)


flash_attention = attention
