"""rw_qkv_norm_rope_store (q/k RMSNorm + RoPE of k + cache write in one launch)
on the GPU against the reference's WanRMSNorm outputs (bf16 fixture) and the
oracle's RoPE.  The norm's fp32 sum runs in another order than torch's, which
can move a value across a bf16 rounding boundary: outputs differ from the
reference by at most one bf16 unit before the weight multiply (two after it) in
under 1% of the elements; the cache write of v and the RoPE of the normed k are
bit-exact."""
import numpy as np
import pytest
import torch

import inputs as gi
from oracle import rope as orope
from oracle import self_attn as osa
from oracle.numerics import bits_to_torch_bf16, f32_to_bf16_bits, torch_bf16_to_bits

pytestmark = pytest.mark.gpu


def _ordered(bits):
    """bf16 bit patterns -> integers ordered like the values (+0 and -0 equal)."""
    b = np.asarray(bits).astype(np.int32) & 0xFFFF
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def _ulps(a, b):
    return np.abs(_ordered(torch_bf16_to_bits(a)) - _ordered(torch_bf16_to_bits(b)))


def _rows(q, k, v):
    """q, k, v [B, L, C] laid out as column slices of one [B, L, 3C] projection."""
    C = q.shape[-1]
    qkv = torch.cat([q, k, v], dim=-1)
    return qkv, qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]


def _status_clean():
    from reworld_b200 import _native
    _native.check_status()


def test_norm_matches_reference_fixture(cuda, golden):
    from reworld_b200 import qkv_norm_rope_store
    g = golden["rmsnorm"]
    x, wq, wk = gi.rmsnorm_case()
    assert abs(gi.checksum(x, wq, wk) - float(g["checksum"])) < 1e-6, "input generator drifted"
    B, L, C = x.shape
    H = C // 128
    v = torch.randn(B, L, C, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    _, qr, kr, vr = _rows(x.to(cuda), x.to(cuda), v.to(cuda))
    sentinel = torch.randn(B, L + 8, H, 128, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
    ck, cv = sentinel.clone().to(cuda), sentinel.clone().to(cuda)
    q_out = qkv_norm_rope_store(qr, kr, vr, wq.to(cuda), wk.to(cuda), ck, cv, 3, gi.RMSNORM_EPS)
    torch.cuda.synchronize()
    ref_q = bits_to_torch_bf16(g["norm_q"]).view(B, L, H, 128)
    ref_k = bits_to_torch_bf16(g["norm_k"]).view(B, L, H, 128)
    for got, ref in ((q_out.cpu(), ref_q), (ck[:, 3:3 + L].cpu(), ref_k)):
        u = _ulps(got, ref)
        assert u.max() <= 1, u.max()
        assert (u == 0).mean() > 0.99, (u == 0).mean()
    # the all-zero row stays zero
    assert not q_out[0, 5].any() and not ck[0, 3 + 5].any()
    assert torch.equal(cv[:, 3:3 + L].cpu(), v.view(B, L, H, 128))
    for c in (ck, cv):
        assert torch.equal(c[:, :3].cpu(), sentinel[:, :3]) and torch.equal(c[:, 3 + L:].cpu(), sentinel[:, 3 + L:])
    _status_clean()


@pytest.mark.parametrize("H,with_delta,grid,extra", [(2, False, (3, 4, 5), 4), (2, True, (3, 4, 5), 4),
                                                     (24, True, (3, 4, 5), 4), (24, True, (3, 22, 40), 8)])
def test_rope_of_normed_k_bit_exact(cuda, H, with_delta, grid, extra):
    """The k rows written with RoPE equal the oracle's RoPE(+PM-RoPE) of the k rows
    the same kernel writes without RoPE; q_out is the same either way.  The
    3x22x40 grid (2 x 2648 tokens) gives every CTA many tokens, so the staging
    ring wraps around several times."""
    from reworld_b200 import RopeArgs, device_table, qkv_norm_rope_store
    gen = torch.Generator().manual_seed(40 + H + grid[1])
    f, h, w = grid
    B, L = 2, f * h * w + extra                   # tokens past the grid stay unroped
    C = H * 128
    q, k, v = ((torch.randn(B, L, C, generator=gen) * 2).to(torch.bfloat16) for _ in range(3))
    wq, wk = ((1 + 0.05 * torch.randn(C, generator=gen)).to(torch.bfloat16) for _ in range(2))
    delta = torch.randn(B, f, 64, generator=gen) * 0.4 if with_delta else None
    freqs = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    _, qr, kr, vr = _rows(q.to(cuda), k.to(cuda), v.to(cuda))
    cap = L + 16
    ck0 = torch.zeros(B, cap, H, 128, dtype=torch.bfloat16, device=cuda)
    cv0 = torch.zeros_like(ck0)
    q0 = qkv_norm_rope_store(qr, kr, vr, wq.to(cuda), wk.to(cuda), ck0, cv0, 10, 1e-6)
    ck1, cv1 = torch.zeros_like(ck0), torch.zeros_like(ck0)
    rope = RopeArgs(device_table(freqs, cuda), (f, h, w), 9, delta=delta.to(cuda) if with_delta else None)
    q1 = qkv_norm_rope_store(qr, kr, vr, wq.to(cuda), wk.to(cuda), ck1, cv1, 10, 1e-6, rope=rope)
    torch.cuda.synchronize()
    assert torch.equal(q0, q1)
    assert torch.equal(cv0, cv1) and torch.equal(cv1[:, 10:10 + L].cpu(), v.view(B, L, H, 128))
    nk = ck0[:, 10:10 + L].float().cpu().numpy()
    want = orope.causal_rope_apply(nk, [(f, h, w)] * B, freqs, start_frame=9)
    if with_delta:
        # the phase factor torch.polar formed on the GPU (as in the reference's
        # GPU run); it may differ from the CPU's in the last bit of cos / sin
        cs = rope.delta_cs.cpu()                                   # [B, f, 64, 2]
        cr_cpu, ci_cpu = orope.delta_cos_sin(delta.numpy())
        assert np.abs(cs[..., 0].numpy() - cr_cpu).max() <= 2 ** -23
        assert np.abs(cs[..., 1].numpy() - ci_cpu).max() <= 2 ** -23
        tok = cs.unsqueeze(2).expand(-1, -1, h * w, -1, -1).reshape(B, f * h * w, 1, 64, 2)
        tok = torch.cat([tok, torch.zeros(B, L - f * h * w, 1, 64, 2)], dim=1).numpy()
        want = orope.pm_rope_apply_cs(want, tok[..., 0], tok[..., 1])
        want[:, f * h * w:] = nk[:, f * h * w:]
    assert np.array_equal(torch_bf16_to_bits(ck1[:, 10:10 + L]), f32_to_bf16_bits(want))
    assert not ck1[:, :10].any() and not ck1[:, 10 + L:].any()
    # the normed rows themselves against the oracle's norm (fp32 sum order: one bf16
    # unit before the weight multiply, up to two after it)
    for got, x, wt in ((q0, q, wq), (ck0[:, 10:10 + L], k, wk)):
        u = _ulps(got.cpu(), osa.rms_norm(x, wt, 1e-6).view(B, L, H, 128))
        assert u.max() <= 2 and (u == 0).mean() > 0.99, (u.max(), (u == 0).mean())
    _status_clean()


def test_full_chunk_size_against_torch_formula(cuda):
    """The 5B model's chunk (2640 tokens x 24 heads x 128) with the cache written
    at an offset, against the reference formula evaluated by torch on the GPU."""
    from reworld_b200 import qkv_norm_rope_store
    gen = torch.Generator(device=cuda).manual_seed(3)
    B, L, H = 1, 2640, 24
    C = H * 128
    qkv = (torch.randn(B, L, 3 * C, generator=gen, device=cuda) * 1.5).to(torch.bfloat16)
    wq, wk = ((1 + 0.05 * torch.randn(C, generator=gen, device=cuda)).to(torch.bfloat16) for _ in range(2))
    cap = 4 * L
    ck = torch.zeros(B, cap, H, 128, dtype=torch.bfloat16, device=cuda)
    cv = torch.zeros_like(ck)
    q_out = qkv_norm_rope_store(qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:], wq, wk, ck, cv, 2 * L, 1e-6)

    def ref(x, wt):
        # 1 / sqrt rounds like the reference's CPU rsqrt (torch's GPU rsqrt is approximate)
        xf = x.float()
        return (xf * (1.0 / torch.sqrt(xf.pow(2).mean(dim=-1, keepdim=True) + 1e-6))).type_as(x) * wt

    torch.cuda.synchronize()
    for got, x, wt in ((q_out, qkv[..., :C], wq), (ck[:, 2 * L:3 * L], qkv[..., C:2 * C], wk)):
        u = _ulps(got.cpu(), ref(x, wt).view(B, L, H, 128).cpu())
        # the fp32 sum order can move x * r across a bf16 rounding boundary (one unit),
        # which the weight multiply and its rounding can widen to two units
        assert u.max() <= 2 and (u == 0).mean() > 0.99, (u.max(), (u == 0).mean())
    assert torch.equal(cv[:, 2 * L:3 * L], qkv[..., 2 * C:].reshape(B, L, H, 128))
    assert not ck[:, :2 * L].any() and not ck[:, 3 * L:].any()
    _status_clean()


def test_rejects_mismatched_shapes(cuda):
    from reworld_b200 import qkv_norm_rope_store
    x = torch.zeros(1, 8, 256, dtype=torch.bfloat16, device=cuda)
    w = torch.ones(256, dtype=torch.bfloat16, device=cuda)
    ck = torch.zeros(1, 16, 2, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError):
        qkv_norm_rope_store(x, x, x, w, w, ck, ck.clone(), 12, 1e-6)          # write past the capacity
    with pytest.raises(ValueError):
        qkv_norm_rope_store(x, x, x, w.float(), w, ck, ck.clone(), 0, 1e-6)   # fp32 norm weight
    with pytest.raises(ValueError):
        qkv_norm_rope_store(x, x, x[..., :128], w, w, ck, ck.clone(), 0, 1e-6)


def test_width_of_the_14b_model(cuda):
    """40 heads (C = 5120: 7 token slots per CTA instead of 10), B = 2, against the
    oracle's norm; v rows exact."""
    from reworld_b200 import qkv_norm_rope_store
    gen = torch.Generator().manual_seed(91)
    B, L, H = 2, 300, 40
    C = H * 128
    q, k, v = ((torch.randn(B, L, C, generator=gen) * 2).to(torch.bfloat16) for _ in range(3))
    wq, wk = ((1 + 0.05 * torch.randn(C, generator=gen)).to(torch.bfloat16) for _ in range(2))
    _, qr, kr, vr = _rows(q.to(cuda), k.to(cuda), v.to(cuda))
    ck = torch.zeros(B, L + 4, H, 128, dtype=torch.bfloat16, device=cuda)
    cv = torch.zeros_like(ck)
    q_out = qkv_norm_rope_store(qr, kr, vr, wq.to(cuda), wk.to(cuda), ck, cv, 4, 1e-6)
    torch.cuda.synchronize()
    for got, x, wt in ((q_out, q, wq), (ck[:, 4:], k, wk)):
        u = _ulps(got.cpu(), osa.rms_norm(x, wt, 1e-6).view(B, L, H, 128))
        assert u.max() <= 2 and (u == 0).mean() > 0.99, (u.max(), (u == 0).mean())
    assert torch.equal(cv[:, 4:].cpu(), v.view(B, L, H, 128))
    _status_clean()
