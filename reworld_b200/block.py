"""Drop-ins for the rest of the DiT block around the cached self-attention: the
text cross-attention with cached K/V, the two LayerNorms and the FFN.

Reference: the block's `cross_attn_ffn` (wan_5b/modules/action_model.py:547-556)

    x = x + cross_attn(norm3(x), context, context_lens, crossattn_cache)
    y = ffn(norm2(x) * (1 + e[4]) + e[3])          # per frame
    x = x + y * e[5]

with norm3 / norm2 WanLayerNorm (model.py:92-102), cross_attn a
MultiShotT2VCrossAttention (causal_model.py:186-289; WanCrossAttention,
model.py:162-197) and ffn Linear(dim, ffn_dim) -> GELU(tanh) -> Linear(ffn_dim, dim)
(action_model.py:404-406).  `install(model)` swaps, per block, norm2 / norm3 for
`RowLayerNorm` (rw_row_norm), ffn for `GeluFFN` (the package's tcgen05 GEMM,
rw_gemm_bf16, with the GELU in the first GEMM's epilogue, then the second GEMM)
and cross_attn.forward for `cross_attn_forward` (its q/k/v/o projections on the
same GEMM, norm_q / norm_k on rw_row_norm, the attention on the package's kernel
with k_lens).  The modulation and the residual adds stay the reference's own
elementwise ops.  CUDA tensors only; bf16 modules run the kernels, modules in
other dtypes keep their own computation.
"""
import types

import torch
import torch.nn as nn

from . import _native
from . import gemm
from ._native import c_vp
from .attention import attention

RW_NORM_RMS, RW_NORM_LAYER = 0, 1


def row_norm(x, weight=None, bias=None, eps=1e-6, mode="layer", out=None):
    """WanRMSNorm (mode 'rms', weight required) or WanLayerNorm (mode 'layer',
    affine optional) over the last dim of a bf16 CUDA tensor, one rw_row_norm launch."""
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError("row_norm runs on bf16 CUDA tensors")
    C = x.shape[-1]
    x2 = x.reshape(-1, C)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    o2 = out.view(-1, C)
    if not _bf16_or_none(weight, bias):
        raise ValueError("row_norm weights must be bf16 (the module's dtype)")
    w = weight.detach().contiguous() if weight is not None else None
    b = bias.detach().contiguous() if bias is not None else None
    code = _native.lib().rw_row_norm(
        c_vp(x2.data_ptr()), c_vp(o2.data_ptr()), c_vp(w.data_ptr()) if w is not None else None,
        c_vp(b.data_ptr()) if b is not None else None, x2.shape[0], C, x2.stride(0), o2.stride(0), float(eps),
        RW_NORM_RMS if mode == "rms" else RW_NORM_LAYER, _native.stream_ptr(x.device))
    _native.check(code, "rw_row_norm")
    return out


def _bf16_or_none(*ts):
    return all(t is None or t.dtype == torch.bfloat16 for t in ts)


class RowLayerNorm(nn.Module):
    """WanLayerNorm on rw_row_norm; keeps the wrapped module's eps, weight and bias."""

    def __init__(self, ln):
        super().__init__()
        self.inner = ln

    def forward(self, x):
        ln = self.inner
        if not x.is_cuda:
            raise ValueError("RowLayerNorm runs on CUDA tensors (no CPU path)")
        if x.dtype != torch.bfloat16 or not _bf16_or_none(ln.weight, ln.bias):
            return ln(x)   # outside the kernel's domain: the module's own computation
        return row_norm(x, ln.weight, ln.bias, ln.eps, "layer")


class GeluFFN(nn.Module):
    """Linear -> GELU(tanh) -> Linear on rw_gemm_bf16, the GELU applied in the first
    GEMM's epilogue (on the fp32 accumulator: one rounding instead of the
    reference's two); keeps the wrapped Sequential's parameters."""

    def __init__(self, seq):
        super().__init__()
        self.inner = seq

    def forward(self, x):
        lin1, act, lin2 = self.inner[0], self.inner[1], self.inner[2]
        if not x.is_cuda:
            raise ValueError("GeluFFN runs on CUDA tensors (no CPU path)")
        if x.dtype != torch.bfloat16 or getattr(act, "approximate", "none") != "tanh" or \
                not _bf16_or_none(lin1.weight, lin1.bias, lin2.weight, lin2.bias):
            return self.inner(x)
        h = gemm.module_linear(lin1, x, gelu=True)
        return gemm.module_linear(lin2, h)


def cross_attn_forward(self, x, context, context_lens, is_teacher_forcing=False, crossattn_cache=None):
    """MultiShotT2VCrossAttention.forward (causal_model.py:188-289; with one context
    chunk per video it is WanCrossAttention.forward, model.py:164-197)."""
    b_orig, L1, C = x.size()
    n, d = self.num_heads, self.head_dim
    b_ctx = context.size(0)
    assert b_ctx % b_orig == 0, f"context batch ({b_ctx}) must be a multiple of x batch ({b_orig})"
    num_chunks = b_ctx // b_orig
    if context_lens is not None and context_lens.numel() == b_orig:
        context_lens = context_lens.repeat_interleave(num_chunks)
    elif context_lens is not None:
        assert context_lens.numel() == b_ctx
    fused = x.dtype == torch.bfloat16 and x.is_cuda and self.q.weight.dtype == torch.bfloat16

    def norm(t, mod):
        # WanRMSNorm with a bf16 weight on the kernel (an fp32 weight makes the
        # reference's product fp32: the module's own computation then)
        if fused and hasattr(mod, "weight") and hasattr(mod, "eps") and _bf16_or_none(mod.weight):
            return row_norm(t, mod.weight, None, mod.eps, "rms")
        return mod(t)

    def lin(mod, t):
        # bf16 projections on the package's GEMM; other dtypes keep the module's own
        return gemm.module_linear(mod, t) if fused and t.dtype == torch.bfloat16 else mod(t)

    def cross_attend(xc):
        b_eff = xc.size(0)
        q = norm(lin(self.q, xc), self.norm_q).view(b_eff, -1, n, d)
        if crossattn_cache is not None and crossattn_cache["is_init"]:
            k, v = crossattn_cache["k"], crossattn_cache["v"]
        else:
            k = norm(lin(self.k, context), self.norm_k).view(b_eff, -1, n, d)
            v = lin(self.v, context).view(b_eff, -1, n, d)
            if crossattn_cache is not None:
                crossattn_cache["is_init"] = True
                crossattn_cache["k"], crossattn_cache["v"] = k, v
        o = attention(q, k, v, k_lens=context_lens)
        return lin(self.o, o.flatten(2))

    def chunk_and_attend(xp):
        Lp = xp.size(1)
        assert Lp % num_chunks == 0, f"{Lp} tokens are not divisible by {num_chunks} context chunks"
        tpc = Lp // num_chunks
        out = cross_attend(xp.reshape(b_orig, num_chunks, tpc, C).reshape(b_ctx, tpc, C))
        return out.view(b_orig, num_chunks, tpc, C).reshape(b_orig, Lp, C)

    if not is_teacher_forcing:
        return chunk_and_attend(x)
    assert L1 % 2 == 0
    half = L1 // 2
    return torch.cat([chunk_and_attend(x[:, :half]), chunk_and_attend(x[:, half:])], dim=1)


def install(model):
    """Per block: norm2 / norm3 -> RowLayerNorm, ffn -> GeluFFN, cross_attn.forward ->
    cross_attn_forward.  Returns the number of blocks changed."""
    blocks = model.blocks if hasattr(model, "blocks") else model
    n = 0
    for blk in blocks:
        for name in ("norm2", "norm3"):
            m = getattr(blk, name, None)
            if isinstance(m, nn.LayerNorm) and not isinstance(m, RowLayerNorm):
                setattr(blk, name, RowLayerNorm(m))
        f = getattr(blk, "ffn", None)
        if isinstance(f, nn.Sequential) and len(f) == 3 and isinstance(f[1], nn.GELU):
            blk.ffn = GeluFFN(f)
        ca = getattr(blk, "cross_attn", None)
        if ca is not None:
            if not hasattr(ca, "_rw_reference_forward"):
                ca._rw_reference_forward = ca.forward
            ca.forward = types.MethodType(cross_attn_forward, ca)
        n += 1
    return n
