"""Drop-in CausalWanPropSelfAttention forward (inference branch, KV cache) on the
GPU against the reference's outputs (bf16 fixtures) and the oracle."""
import numpy as np
import pytest
import torch
import torch.nn as nn

import inputs as gi
from oracle import rope as orope
from oracle import self_attn as osa

pytestmark = pytest.mark.gpu


class _RMSNorm(nn.Module):
    """Same arithmetic as the reference's WanRMSNorm (wan_5b/modules/model.py:73-89)."""

    def __init__(self, dim, eps):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)).type_as(x) * self.weight


class _PropSelfAttn(nn.Module):
    """Parameter container with the attribute names of CausalWanPropSelfAttention."""

    def __init__(self, dim, heads, eps=1e-6):
        super().__init__()
        self.num_heads, self.head_dim = heads, dim // heads
        self.local_attn_size, self.sink_size, self.max_attention_size = -1, 0, None
        self.q, self.k, self.v, self.o = (nn.Linear(dim, dim) for _ in range(4))
        self.norm_q, self.norm_k = _RMSNorm(dim, eps), _RMSNorm(dim, eps)
        self.pose_mlp = nn.Sequential(nn.Linear(12, 256), nn.SiLU(), nn.Linear(256, self.head_dim // 2))
        self.value_proj, self.prope_proj = nn.Linear(dim, dim), nn.Linear(dim, dim)


def _build(dtype, device):
    mod = _PropSelfAttn(gi.SELF_ATTN_DIM, gi.SELF_ATTN_HEADS)
    shapes = {n: tuple(p.shape) for n, p in mod.named_parameters()}
    vals, g = gi.self_attn_params(shapes)
    with torch.no_grad():
        for n, p in mod.named_parameters():
            p.copy_(vals[n])
    return mod.to(dtype=dtype, device=device), vals, g


@pytest.mark.parametrize("tag,dtype,with_ctx", [t for t in gi.SELF_ATTN_TAGS if t[1] == torch.bfloat16])
def test_forward_matches_reference_fixture(cuda, golden, tag, dtype, with_ctx):
    from reworld_b200.self_attn import install
    g = golden["self_attn"]
    mod, vals, gen = _build(dtype, cuda)
    install([type("Blk", (), {"self_attn": mod})()])
    k0, v0, x, ctx = gi.self_attn_inputs(gen, dtype, with_ctx)
    f, h, w = gi.SELF_ATTN_GRID
    ct = f * h * w
    n0 = gi.SELF_ATTN_CACHED * ct
    cap = (gi.SELF_ATTN_CACHED + 2) * ct
    H = gi.SELF_ATTN_HEADS
    cache = {"k": torch.zeros(1, cap, H, 128, dtype=dtype, device=cuda),
             "v": torch.zeros(1, cap, H, 128, dtype=dtype, device=cuda),
             "global_end_index": torch.tensor([n0], device=cuda), "local_end_index": torch.tensor([n0], device=cuda)}
    cache["k"][:, :n0], cache["v"][:, :n0] = k0.to(cuda), v0.to(cuda)
    freqs = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    with torch.no_grad():
        y = mod.forward(x.to(cuda), torch.tensor([ct]), torch.tensor([[f, h, w]]), freqs, None, kv_cache=cache,
                        current_start=n0, prope_context=ctx.to(cuda) if ctx is not None else None)
    torch.cuda.synchronize()
    # the bf16 module ran the stacked q|k|v GEMM and the fused norm/RoPE/store kernel;
    # its parameters are views of the stacked buffer and keep their values
    assert mod.q.weight.data_ptr() == mod._rw_wqkv.data_ptr()
    assert torch.equal(mod.v.weight.cpu(), vals["v.weight"].to(dtype))
    # cache bookkeeping exactly as the reference
    assert [int(cache["global_end_index"]), int(cache["local_end_index"])] == list(g[f"{tag}_ends"])
    assert torch.equal(cache["k"][:, :n0].cpu(), k0) and not cache["k"][:, n0 + ct:].any()
    # new K rows: RoPE in the store kernel; bit-exact without the PM-RoPE phase
    knew = cache["k"][:, n0:n0 + ct].float().cpu().numpy()
    kref = g[f"{tag}_knew"]
    if with_ctx:
        # the phase comes from a bf16 pose MLP evaluated on the GPU vs the CPU reference
        assert np.abs(knew - kref).max() < 0.05 * max(1.0, np.abs(kref).max())
    else:
        # projections run in cuBLAS bf16 on the GPU vs CPU in the reference: compare with tolerance
        assert np.abs(knew - kref).max() < 0.05 * max(1.0, np.abs(kref).max())
    yref = g[f"{tag}_y"]
    err = np.abs(y.float().cpu().numpy() - yref)
    assert err.max() < 2e-2 and err.mean() < 2e-3, (err.max(), err.mean())


def test_forward_attention_core_bit_level_vs_oracle(cuda):
    """Same bf16 q/k/v fed to both sides (no projections): the roped cache rows
    are bit-exact and the attention output is within the attention tolerance."""
    from reworld_b200 import RopeArgs, chunk_attention, device_table, rope_kv_store
    from oracle.attention import attention_f64
    g = torch.Generator().manual_seed(31)
    f, h, w, H = 3, 11, 20, 4
    ct = f * h * w
    n0 = 3 * ct
    q = torch.randn(1, ct, H, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, ct, H, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, ct, H, 128, generator=g).to(torch.bfloat16)
    cache_k = torch.randn(1, 5 * ct, H, 128, generator=g).to(torch.bfloat16)
    cache_v = torch.randn(1, 5 * ct, H, 128, generator=g).to(torch.bfloat16)
    freqs = orope.build_freqs(128, 12 / 22, 20 / 40)
    qr = orope.causal_rope_apply(q.float().numpy(), [(f, h, w)], freqs, start_frame=n0 // (h * w))
    kr = orope.causal_rope_apply(k.float().numpy(), [(f, h, w)], freqs, start_frame=n0 // (h * w))
    ck, cv = cache_k.to(cuda), cache_v.to(cuda)
    rope = RopeArgs(device_table(freqs, cuda), (f, h, w), n0 // (h * w))
    rope_kv_store(k.to(cuda), v.to(cuda), ck, cv, n0, rope=rope)
    out = chunk_attention(q.to(cuda), ck[:, :n0 + ct], cv[:, :n0 + ct], rope=rope)
    torch.cuda.synchronize()
    assert np.array_equal(ck[:, n0:n0 + ct].float().cpu().numpy(), kr)
    kk = np.concatenate([cache_k[:, :n0].float().numpy(), kr], axis=1)
    vv = np.concatenate([cache_v[:, :n0].float().numpy(), v.float().numpy()], axis=1)
    ref = attention_f64(qr, kk, vv)
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() < 2e-2 and err.mean() < 2e-3


def test_forward_rejects_fp32_cache(cuda):
    from reworld_b200.self_attn import install
    mod, _, _ = _build(torch.float32, cuda)
    install([type("Blk", (), {"self_attn": mod})()])
    cache = {"k": torch.zeros(1, 300, 2, 128, device=cuda), "v": torch.zeros(1, 300, 2, 128, device=cuda),
             "global_end_index": torch.tensor([0]), "local_end_index": torch.tensor([0])}
    with pytest.raises(NotImplementedError):
        mod.forward(torch.zeros(1, 60, 256, device=cuda), torch.tensor([60]), torch.tensor([[3, 4, 5]]),
                    orope.build_freqs(128), None, kv_cache=cache, current_start=0)


def test_fp32_module_with_bf16_cache_matches_oracle(cuda):
    """A module kept in fp32 (the 352x640 CPU configuration's dtype) on the GPU:
    torch's fp32 projections and norms, q/k/v cast to bf16 for the cache store
    (RoPE in rw_rope_kv_store) and the attention kernel, the output back in fp32
    through the fp32 o projection.  Against the oracle's fp32 forward on the same
    bf16-valued cache, within the attention tolerance; the cache bookkeeping is
    the reference's."""
    from reworld_b200.self_attn import install
    mod, vals, gen = _build(torch.float32, cuda)
    install([type("Blk", (), {"self_attn": mod})()])
    k0, v0, x, _ = gi.self_attn_inputs(gen, torch.float32, False)
    f, h, w = gi.SELF_ATTN_GRID
    ct = f * h * w
    n0 = gi.SELF_ATTN_CACHED * ct
    cap = (gi.SELF_ATTN_CACHED + 2) * ct
    H = gi.SELF_ATTN_HEADS
    k0b, v0b = k0.to(torch.bfloat16), v0.to(torch.bfloat16)
    cache = {"k": torch.zeros(1, cap, H, 128, dtype=torch.bfloat16, device=cuda),
             "v": torch.zeros(1, cap, H, 128, dtype=torch.bfloat16, device=cuda),
             "global_end_index": torch.tensor([n0], device=cuda), "local_end_index": torch.tensor([n0], device=cuda)}
    cache["k"][:, :n0], cache["v"][:, :n0] = k0b.to(cuda), v0b.to(cuda)
    freqs = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    with torch.no_grad():
        y = mod.forward(x.to(cuda), torch.tensor([ct]), torch.tensor([[f, h, w]]), freqs, None, kv_cache=cache,
                        current_start=n0)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32
    assert [int(cache["global_end_index"]), int(cache["local_end_index"])] == [n0 + ct, n0 + ct]
    W = {n: t.float() for n, t in vals.items()}
    kc = {"k": torch.zeros(1, cap, H, 128), "v": torch.zeros(1, cap, H, 128),
          "global_end_index": torch.tensor([n0]), "local_end_index": torch.tensor([n0])}
    kc["k"][:, :n0], kc["v"][:, :n0] = k0b.float(), v0b.float()
    y_ref, _ = osa.prop_self_attn_forward(W, x, (f, h, w), freqs, kc, n0, num_heads=H)
    err = (y.cpu() - y_ref).abs()
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3, (err.max().item(), err.mean().item())
