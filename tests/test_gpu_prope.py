"""PRoPE SE3 transform (rw_se3_block_apply) on the GPU against the oracle's
restatement of _se3_block_apply (wan_5b/modules/action_model.py:84-114) and the
reference formula evaluated by torch.  Each output is one fp32 sum of 4 exact
products rounded to bf16; only the order of that sum may differ from the
library's, so outputs agree within one bf16 unit, > 99 % of them exactly."""
import math

import numpy as np
import pytest
import torch

from oracle import self_attn as osa
from oracle.numerics import torch_bf16_to_bits

pytestmark = pytest.mark.gpu


def _ordered(bits):
    b = np.asarray(bits).astype(np.int32) & 0xFFFF
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def _ulps(a, b):
    return np.abs(_ordered(torch_bf16_to_bits(a)) - _ordered(torch_bf16_to_bits(b)))


def _poses(B, T, gen):
    """Camera-to-world SE3 matrices [B, T, 4, 4] from random yaw/pitch and translations."""
    yaw = torch.randn(B, T, generator=gen) * 0.6
    pitch = torch.randn(B, T, generator=gen) * 0.3
    cy, sy, cp, sp = yaw.cos(), yaw.sin(), pitch.cos(), pitch.sin()
    P = torch.zeros(B, T, 4, 4)
    P[..., 0, 0], P[..., 0, 1], P[..., 0, 2] = cy, sy * sp, sy * cp
    P[..., 1, 1], P[..., 1, 2] = cp, -sp
    P[..., 2, 0], P[..., 2, 1], P[..., 2, 2] = -sy, cy * sp, cy * cp
    P[..., :3, 3] = torch.randn(B, T, 3, generator=gen) * 2.0
    P[..., 3, 3] = 1.0
    return P


def _raw(x, out, mats, fs):
    from reworld_b200 import _native
    from reworld_b200._native import c_vp
    B, L, H, D = x.shape
    code = _native.lib().rw_se3_block_apply(c_vp(x.data_ptr()), c_vp(out.data_ptr()), c_vp(mats.data_ptr()),
                                            B, L, H, D, fs, *x.stride()[:3], *out.stride()[:3],
                                            _native.stream_ptr(x.device))
    _native.check(code, "rw_se3_block_apply")


@pytest.mark.parametrize("mode", ["P", "P_inv"])
def test_se3_kernel_matches_oracle(cuda, mode):
    """Same matrices on both sides: the kernel against the oracle's torch-CPU restatement."""
    gen = torch.Generator().manual_seed(5 if mode == "P" else 6)
    B, H, fs, nf = 2, 4, 20, 3
    L = nf * fs
    big = (torch.randn(B, L, H + 2, 128, generator=gen) * 1.5).to(torch.bfloat16)
    x = big[:, :, 1:H + 1]                                     # strided view
    ctx = _poses(B, nf + 2, gen)                                # more contexts than frames: the last nf are used
    want = osa._se3(x, ctx, mode, fs)                           # [B, L, H, D] bf16 (CPU)
    c = ctx[:, -nf:].to(torch.bfloat16)
    mats = (osa._inv_se3(c) if mode == "P_inv" else c).float().contiguous()
    xd = big.to(cuda)[:, :, 1:H + 1]
    out = torch.empty(B, L, H, 128, dtype=torch.bfloat16, device=cuda)
    _raw(xd, out, mats.to(cuda), fs)
    torch.cuda.synchronize()
    u = _ulps(out.cpu(), want.contiguous())
    assert u.max() <= 1 and (u == 0).mean() > 0.99, (u.max(), (u == 0).mean())


def test_se3_public_function_and_full_chunk(cuda):
    """se3_block_apply (matrices formed on the GPU, as the reference's GPU run forms
    them) against the reference formula on the GPU at the 704x1280 chunk shape."""
    from reworld_b200.self_attn import _se3_torch, se3_block_apply
    gen = torch.Generator().manual_seed(9)
    B, H, fs, nf = 1, 24, 880, 3
    L = nf * fs
    x = (torch.randn(B, L, H, 128, generator=gen)).to(torch.bfloat16).to(cuda)
    ctx = _poses(B, 15, gen).to(cuda)
    for mode in ("P", "P_inv"):
        got = se3_block_apply(x, ctx, mode, fs)
        want = _se3_torch(x, ctx, mode, fs)
        torch.cuda.synchronize()
        u = _ulps(got.cpu(), want.contiguous().cpu())
        assert u.max() <= 1 and (u == 0).mean() > 0.99, (mode, u.max(), (u == 0).mean())
    # into a column block of a wider buffer (the [y | P y] layout of the output GEMM)
    yy = torch.zeros(B, L, 2 * H * 128, dtype=torch.bfloat16, device=cuda)
    se3_block_apply(x, ctx, "P", fs, out=yy[..., H * 128:].view(B, L, H, 128))
    torch.cuda.synchronize()
    assert not yy[..., :H * 128].any()
    assert torch.equal(yy[..., H * 128:].view(B, L, H, 128), se3_block_apply(x, ctx, "P", fs))


def test_se3_rejects_partial_frames(cuda):
    from reworld_b200.self_attn import se3_block_apply
    x = torch.zeros(1, 50, 2, 128, dtype=torch.bfloat16, device=cuda)
    ctx = torch.eye(4, device=cuda).expand(1, 3, 4, 4)
    with pytest.raises(ValueError):
        se3_block_apply(x, ctx, "P", 20)
    with pytest.raises(ValueError):
        se3_block_apply(x.float(), ctx, "P", 25)


def test_se3_kernel_two_batches(cuda):
    """B = 2, each batch with its own frames' matrices, against the oracle."""
    gen = torch.Generator().manual_seed(17)
    B, H, fs, nf = 2, 3, 20, 3
    L = nf * fs
    x = (torch.randn(B, L, H, 128, generator=gen) * 1.5).to(torch.bfloat16)
    ctx = _poses(B, nf, gen)
    want = osa._se3(x, ctx, "P", fs)
    mats = ctx.to(torch.bfloat16).float().contiguous()
    out = torch.empty(B, L, H, 128, dtype=torch.bfloat16, device=cuda)
    _raw(x.to(cuda), out, mats.to(cuda), fs)
    torch.cuda.synchronize()
    u = _ulps(out.cpu(), want.contiguous())
    assert u.max() <= 1 and (u == 0).mean() > 0.99, (u.max(), (u == 0).mean())
