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


@pytest.mark.parametrize("B,Lq,Lk,H,fs,with_rope", [
    (1, 2640, 7920, 24, 880, True),   # the 704x1280 chunk: whole units plus merged key-split tail units
    (1, 512, 1024, 37, 128, False),   # 74 whole units (one per pair), no merge
    (2, 200, 640, 37, 40, False),     # 200 rows of 256 per unit: padded rows clipped by the store
])
def test_attention_writes_p_y_like_the_se3_kernel(cuda, B, Lq, Lk, H, fs, with_rope):
    """rw_attn_fwd_prope: the attention output y is bit-identical to rw_attn_fwd's
    and the P y it writes beside y bit-identical to rw_se3_block_apply on that y,
    through both output paths (the kernel's epilogue and the merge of key-split
    units), twice in a row into [y | P y] rows as the self-attention drop-in uses."""
    from reworld_b200 import RopeArgs, build_freqs, chunk_attention, device_table
    from reworld_b200 import _native as nat
    g = torch.Generator(device=cuda).manual_seed(Lq + H)
    q = torch.randn(B, Lq, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    frames = Lq // fs
    ctx = _poses(B, frames, torch.Generator().manual_seed(7)).to(torch.bfloat16)
    mats = ctx.float().contiguous().to(cuda)
    rope = None
    if with_rope:
        rope = RopeArgs(device_table(build_freqs(128, 12 / 22, 20 / 40), cuda), (3, 22, 40), 9)
    y_ref = chunk_attention(q, k, v, rope=rope)
    py_ref = torch.empty_like(y_ref)
    lib = nat.lib()
    code = lib.rw_se3_block_apply(nat.c_vp(y_ref.data_ptr()), nat.c_vp(py_ref.data_ptr()), nat.c_vp(mats.data_ptr()),
                                  B, Lq, H, 128, fs, *y_ref.stride()[:3], *py_ref.stride()[:3], nat.stream_ptr(cuda))
    nat.check(code, "rw_se3_block_apply")
    C = H * 128
    for call in range(2):
        yy = torch.full((B, Lq, 2 * C), float("nan"), dtype=torch.bfloat16, device=cuda)
        y = yy[..., :C].view(B, Lq, H, 128)
        py = yy[..., C:].view(B, Lq, H, 128)
        chunk_attention(q, k, v, rope=rope, out=y, se3=(mats, fs, py))
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref), call
        assert torch.equal(py, py_ref), call
    nat.check_status(cuda)


def test_attention_prope_rejects_bad_frames(cuda):
    from reworld_b200 import chunk_attention
    q = torch.zeros(1, 100, 2, 128, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(1, 256, 2, 128, dtype=torch.bfloat16, device=cuda)
    po = torch.empty_like(q)
    with pytest.raises(ValueError):       # 100 tokens are not whole frames of 30
        chunk_attention(q, k, k, se3=(torch.zeros(1, 3, 4, 4, device=cuda), 30, po))
    with pytest.raises(ValueError):       # fp16 matrices
        chunk_attention(q, k, k, se3=(torch.zeros(1, 5, 4, 4, dtype=torch.float16, device=cuda), 20, po))
