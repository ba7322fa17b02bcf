"""Attention oracle (TEST INFRASTRUCTURE, see oracle/__init__.py).

reference_attention_cpu is the reference's own CPU path: wan_5b/modules/
attention.py:133-179 `attention()` with the flash-attention flags off, i.e.
q/k/v transposed to [B, H, L, D], cast to `dtype` (bf16 by default) and run
through torch's scaled_dot_product_attention, non-causal, no mask (:164-179).
attention_f64 restates the same math in numpy float64 for tolerance checks.
"""
import math

import numpy as np
import torch


def reference_attention_cpu(q, k, v, dtype=torch.bfloat16, softmax_scale=None):
    """wan_5b/modules/attention.py:164-179 (SDPA branch), CPU tensors [B, L, H, D]."""
    q = q.transpose(1, 2).to(dtype)
    k = k.transpose(1, 2).to(dtype)
    v = v.transpose(1, 2).to(dtype)
    out = torch.nn.functional.scaled_dot_product_attention(
        q, k, v, attn_mask=None, is_causal=False, dropout_p=0.0, scale=softmax_scale)
    return out.transpose(1, 2).contiguous()


def attention_f64(q, k, v, softmax_scale=None):
    """softmax(q k^T * scale) v per (batch, head) in float64.  q: [B, Lq, H, D],
    k/v: [B, Lk, H, D] float arrays (e.g. bf16 values as float32)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    qh = q.transpose(0, 2, 1, 3)
    kh = k.transpose(0, 2, 1, 3)
    vh = v.transpose(0, 2, 1, 3)
    s = np.matmul(qh, kh.transpose(0, 1, 3, 2)) * scale
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.matmul(p, vh).transpose(0, 2, 1, 3)


def attention_flops(B, Lq, Lk, H, D):
    """QK^T + PV multiply-adds counted as 2 FLOPs each."""
    return 4.0 * B * Lq * Lk * H * D
