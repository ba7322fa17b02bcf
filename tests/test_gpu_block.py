"""The DiT block's cross_attn_ffn with this package's drop-ins installed
(reworld_b200.block: norm2 / norm3 on rw_row_norm, the FFN's first GEMM with the
GELU in its epilogue, the cross-attention's norms on rw_row_norm and its
attention on the chunk-attention kernel) against the reference block's outputs
(bf16 fixture made from the reference's own modules on CPU)."""
import numpy as np
import pytest
import torch
import torch.nn as nn

import inputs as gi
from oracle import block as ob
from oracle.numerics import bits_to_torch_bf16, torch_bf16_to_bits

pytestmark = pytest.mark.gpu


def _ulps(a, b):
    def od(t):
        x = torch_bf16_to_bits(t).astype(np.int32) & 0xFFFF
        return np.where(x & 0x8000, -(x & 0x7FFF), x)
    return np.abs(od(a) - od(b))


class _RMS(nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.eps, self.weight = eps, nn.Parameter(torch.ones(dim))


class _CrossAttn(nn.Module):
    """Parameter container with the attribute names of MultiShotT2VCrossAttention."""

    def __init__(self, dim, heads, eps=1e-6):
        super().__init__()
        self.num_heads, self.head_dim = heads, dim // heads
        self.q, self.k, self.v, self.o = (nn.Linear(dim, dim) for _ in range(4))
        self.norm_q, self.norm_k = _RMS(dim, eps), _RMS(dim, eps)


class _Block(nn.Module):
    def __init__(self, dim, heads, ffn_dim, eps=1e-6):
        super().__init__()
        self.norm3 = nn.LayerNorm(dim, eps, elementwise_affine=True)
        self.cross_attn = _CrossAttn(dim, heads, eps)
        self.norm2 = nn.LayerNorm(dim, eps, elementwise_affine=False)
        self.ffn = nn.Sequential(nn.Linear(dim, ffn_dim), nn.GELU(approximate="tanh"), nn.Linear(ffn_dim, dim))


def _close(got, ref, tol=2e-2):
    d = (got.float().cpu() - ref.float()).abs()
    scale = max(1.0, ref.float().abs().max().item())
    assert d.max().item() < tol * scale and d.mean().item() < tol / 10 * scale, (d.max().item(), d.mean().item())


def test_cross_attn_ffn_matches_reference_fixture(cuda, golden):
    from reworld_b200 import block as rb
    g = golden["block"]
    blk = _Block(gi.BLOCK_DIM, gi.BLOCK_HEADS, gi.BLOCK_FFN)
    vals = gi.block_params({n: tuple(p.shape) for n, p in blk.named_parameters()})
    with torch.no_grad():
        for n, p in blk.named_parameters():
            p.copy_(vals[n])
    blk = blk.to(device=cuda, dtype=torch.bfloat16)
    assert rb.install([blk]) == 1
    assert isinstance(blk.norm2, rb.RowLayerNorm) and isinstance(blk.ffn, rb.GeluFFN)
    x, context, e_mod = (t.to(cuda) for t in gi.block_inputs())
    F, fs = gi.BLOCK_FRAMES, gi.BLOCK_FS
    e = e_mod.chunk(6, dim=2)
    lens = torch.tensor([gi.BLOCK_CTX], device=cuda)
    cache = {"is_init": False}
    with torch.no_grad():
        n3 = blk.norm3(x)
        ca = blk.cross_attn(n3, context, lens, crossattn_cache=cache)
        x1 = x + ca
        n2 = blk.norm2(x1)
        y = blk.ffn((n2.unflatten(dim=1, sizes=(F, fs)) * (1 + e[4]) + e[3]).flatten(1, 2))
        out = x1 + (y.unflatten(dim=1, sizes=(F, fs)) * e[5]).flatten(1, 2)
        # the cached text K/V path gives the same result
        ca2 = blk.cross_attn(n3, context, lens, crossattn_cache=cache)
    torch.cuda.synchronize()
    ref = {k: bits_to_torch_bf16(g[k]).view(-1) for k in ("norm3", "cross_attn", "x1", "norm2", "ffn", "out")}
    # the LayerNorm kernel: fp32 statistics, one rounding -> within a bf16 unit of torch's
    u = _ulps(n3.cpu(), ref["norm3"].view(n3.shape))
    assert u.max() <= 1 and (u == 0).mean() > 0.97, (u.max(), (u == 0).mean())
    _close(ca, ref["cross_attn"].view(ca.shape))
    assert torch.equal(ca2, ca) and cache["is_init"]
    _close(n2, ref["norm2"].view(n2.shape))
    _close(y, ref["ffn"].view(y.shape))
    _close(out, ref["out"].view(out.shape))


@pytest.mark.parametrize("mode", ["rms", "layer", "layer_affine"])
def test_row_norm_full_width_vs_oracle(cuda, mode):
    """rw_row_norm at the 5B width (3072) on strided rows, against the oracle's torch-CPU norms."""
    from reworld_b200.block import row_norm
    gen = torch.Generator().manual_seed(44)
    rows, C = 300, 3072
    big = (torch.randn(rows, C + 256, generator=gen) * 3).to(torch.bfloat16)
    x = big[:, 128:128 + C]
    w = (1 + 0.05 * torch.randn(C, generator=gen)).to(torch.bfloat16)
    b = (0.05 * torch.randn(C, generator=gen)).to(torch.bfloat16)
    if mode == "rms":
        got = row_norm(big.to(cuda)[:, 128:128 + C], w.to(cuda), None, 1e-6, "rms")
        ref = ob.rms_norm(x, w, 1e-6)
        lim = 2                       # a unit before the weight product can widen to two after it
    elif mode == "layer":
        got = row_norm(big.to(cuda)[:, 128:128 + C], None, None, 1e-6, "layer")
        ref = ob.layer_norm(x, None, None, 1e-6)
        lim = 1
    else:
        got = row_norm(big.to(cuda)[:, 128:128 + C], w.to(cuda), b.to(cuda), 1e-6, "layer")
        ref = ob.layer_norm(x, w, b, 1e-6)
        lim = 2                       # n * w + b can cancel: the small result's units are fine
    torch.cuda.synchronize()
    u = _ulps(got.cpu(), ref)
    assert u.max() <= lim and (u == 0).mean() > 0.97, (u.max(), (u == 0).mean())
