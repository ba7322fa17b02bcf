"""Host-side logic of the drop-ins that needs no GPU: the stacked-weight
bookkeeping of the self-attention, the SE3 frame matrices, the block's module
swaps (and that they refuse CPU tensors)."""
import pytest
import torch
import torch.nn as nn

import inputs as gi
from oracle import self_attn as osa


class _Lin3(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.q, self.k, self.v = (nn.Linear(dim, dim) for _ in range(3))
        self.o, self.prope_proj = nn.Linear(dim, dim), nn.Linear(dim, dim)


def test_stacked_qkv_views_keep_values_and_follow_replacement():
    from reworld_b200.self_attn import _stacked_out, _stacked_qkv
    torch.manual_seed(0)
    m = _Lin3(64)
    before = {n: p.detach().clone() for n, p in m.named_parameters()}
    W, b = _stacked_qkv(m)
    assert W.shape == (192, 64) and b.shape == (192,)
    for i, lin in enumerate((m.q, m.k, m.v)):
        assert lin.weight.data_ptr() == W[64 * i].data_ptr()          # a view, no second copy
    for n, p in m.named_parameters():
        assert torch.equal(p, before[n]), n
    x = torch.randn(3, 64)
    assert torch.equal(nn.functional.linear(x, W, b)[:, 64:128], m.k(x))
    # in-place updates reach the stacked buffer; a replaced parameter triggers a rebuild
    with torch.no_grad():
        m.v.weight.add_(1.0)
    assert torch.equal(_stacked_qkv(m)[0][128:], m.v.weight)
    m.k.weight.data = torch.zeros(64, 64)
    W2, _ = _stacked_qkv(m)
    assert not W2[64:128].any() and m.k.weight.data_ptr() == W2[64].data_ptr()
    Wo, bo = _stacked_out(m)
    assert Wo.shape == (64, 128) and torch.equal(bo, m.o.bias + m.prope_proj.bias)
    y = torch.randn(3, 128)
    ref = m.o(y[:, :64]) + m.prope_proj(y[:, 64:])
    assert torch.allclose(nn.functional.linear(y, Wo, bo), ref, atol=1e-5)


@pytest.mark.parametrize("mode", ["P", "P_inv"])
def test_se3_mats_match_oracle(mode):
    from reworld_b200.self_attn import se3_mats
    torch.manual_seed(1)
    ctx = torch.eye(4).repeat(1, 5, 1, 1)
    ctx[..., :3, :3] = torch.linalg.qr(torch.randn(1, 5, 3, 3))[0]
    ctx[..., :3, 3] = torch.randn(1, 5, 3)
    got = se3_mats(ctx, mode, 3, torch.bfloat16)
    c = ctx[:, -3:].to(torch.bfloat16)
    want = (osa._inv_se3(c) if mode == "P_inv" else c).float()
    assert got.dtype == torch.float32 and got.is_contiguous() and torch.equal(got, want)


def test_block_install_swaps_modules_and_refuses_cpu_tensors():
    from reworld_b200 import block as rb

    class Blk(nn.Module):
        def __init__(self):
            super().__init__()
            self.norm3 = nn.LayerNorm(gi.BLOCK_DIM, 1e-6, elementwise_affine=True)
            self.norm2 = nn.LayerNorm(gi.BLOCK_DIM, 1e-6, elementwise_affine=False)
            self.ffn = nn.Sequential(nn.Linear(gi.BLOCK_DIM, 32), nn.GELU(approximate="tanh"),
                                     nn.Linear(32, gi.BLOCK_DIM))
            self.cross_attn = nn.Module()
            self.cross_attn.forward = lambda *a, **k: None

    blk = Blk()
    ln3 = blk.norm3
    assert rb.install([blk]) == 1
    assert isinstance(blk.norm3, rb.RowLayerNorm) and blk.norm3.inner is ln3
    assert isinstance(blk.norm2, rb.RowLayerNorm) and isinstance(blk.ffn, rb.GeluFFN)
    assert hasattr(blk.cross_attn, "_rw_reference_forward")
    rb.install([blk])                                   # idempotent: no double wrapping
    assert isinstance(blk.norm2.inner, nn.LayerNorm) and not isinstance(blk.norm2.inner, rb.RowLayerNorm)
    x = torch.randn(1, 4, gi.BLOCK_DIM)
    with pytest.raises(ValueError):
        blk.norm2(x)
    with pytest.raises(ValueError):
        blk.ffn(x)
    with pytest.raises(ValueError):
        rb.row_norm(x.bfloat16())


def test_host_pool_capped_by_ram_and_halved_on_failed_pinning(monkeypatch):
    """The tiered bank's pinned pool follows the reference's sizing: at most half of
    the free RAM, halved while pinning fails (the bank's K is lowered to fit)."""
    import warnings as _w
    from reworld_b200 import landmark as lm
    real_empty = torch.empty
    calls = []

    def fake_empty(*shape, pin_memory=False, **kw):
        dims = shape[0] if len(shape) == 1 and isinstance(shape[0], tuple) else shape
        n = dims[0] if len(dims) else 0
        calls.append(n)
        if pin_memory and n > 3:
            raise RuntimeError("cannot pin that much")
        return real_empty(*shape, **kw)

    monkeypatch.setattr(lm, "_available_ram", lambda: None)
    monkeypatch.setattr(lm.torch, "empty", fake_empty)
    with _w.catch_warnings(record=True) as rec:
        _w.simplefilter("always")
        pool = lm.host_pool(16, (2, 4, 8), torch.bfloat16)
    assert pool.shape == (2, 2, 4, 8) and [c for c in calls if c] == [16, 8, 4, 2]
    assert any("retry with" in str(r.message) for r in rec)
    # free-RAM cap: half of what is available
    member = 2 * 4 * 8 * 2
    monkeypatch.setattr(lm, "_available_ram", lambda: 2 * 3 * member + 1)
    with _w.catch_warnings(record=True) as rec:
        _w.simplefilter("always")
        pool = lm.host_pool(16, (2, 4, 8), torch.bfloat16)
    assert pool.shape[0] == 3 and any("capped by free RAM" in str(r.message) for r in rec)


def test_host_pool_falls_back_to_pageable_memory(monkeypatch):
    """No pinned slot at all: one pageable slot, as the reference's last resort
    (landmark_cache_v2.py:187-200); a pool too small for the retrieved landmarks
    is refused by the bank."""
    import warnings as _w
    from reworld_b200 import landmark as lm
    real_empty = torch.empty
    calls = []

    def fake_empty(*shape, pin_memory=False, **kw):
        dims = shape[0] if len(shape) == 1 and isinstance(shape[0], tuple) else shape
        calls.append((dims[0] if len(dims) else 0, pin_memory))
        if pin_memory:
            raise RuntimeError("cannot pin")
        return real_empty(*shape, **kw)

    monkeypatch.setattr(lm, "_available_ram", lambda: None)
    monkeypatch.setattr(lm.torch, "empty", fake_empty)
    with _w.catch_warnings(record=True) as rec:
        _w.simplefilter("always")
        pool = lm.host_pool(8, (2, 4, 8), torch.bfloat16)
    assert pool.shape == (1, 2, 4, 8) and not pool.is_pinned()
    assert [c for c in calls if c[0]] == [(8, True), (4, True), (2, True), (1, True), (1, False)]
    assert any("pageable" in str(r.message) for r in rec)
