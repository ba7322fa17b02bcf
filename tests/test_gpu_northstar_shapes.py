"""Parity at the shapes of the 704x1280 workloads themselves (not only reduced
sizes): the full 30-layer x 24-head landmark gather with a 30-entry bank, the
chunk attention at the stress configuration (batch 4, 63360 / 66000 keys, 24
and 3 heads), the installed self-attention forward at the 5B width (3072
channels, 24 heads), and the chunk pose on device tensors."""
import numpy as np
import pytest
import torch

import inputs as gi
from oracle import landmark as olm
from oracle import rope as orope
from oracle import self_attn as osa
from oracle.numerics import torch_bf16_to_bits

pytestmark = pytest.mark.gpu

CT, LAYERS, H, D = 2640, 30, 24, 128


def _tag(c, layer, kv):
    """A 16-bit pattern per (chunk, layer, K or V) that marks the source of every byte."""
    return int((c * 7919 + layer * 104729 + kv * 1299709 + 12345) & 0x7FFF) | 0x0101


def test_full_size_gather_bytes_against_oracle_layout(cuda):
    """The bank update of the 704x1280 rollout at full size: 30 layers x [2640, 24,
    128] bf16 K and V per chunk, sink 1 + recent 5 + a 30-entry bank with top-6
    pose retrieval (budget 12 through budget_split), on a walk that revisits
    every 8 chunks.  Every chunk's bytes are the pattern base ^ tag(chunk, layer,
    K/V); after each chunk every layer's assembled cache [0, tot) must hold, in
    the oracle's layout order (sink | recent old->new | bank[R]), exactly the
    bytes of the chunks it names (longctx/inference/landmark_cache_v2.py:618-682)."""
    from reworld_b200.landmark import LandmarkBankStack
    from reworld_b200.poses import random_walk
    st = LandmarkBankStack.from_budget(CT, LAYERS, H, D, budget_chunks=12, n_sink=1, recent_w=5, landmark_k=30,
                                       device=cuda)
    sp = st.split
    assert (sp.n_sink, sp.recent_w, sp.n_landmark, sp.K) == (1, 5, 6, 30)
    orc = olm.OracleBank(sp.n_sink, sp.recent_w, sp.K, sp.n_landmark, "b")
    cap = (sp.budget + 1) * CT
    caches_k = [torch.zeros(1, cap, H, D, dtype=torch.bfloat16, device=cuda) for _ in range(LAYERS)]
    caches_v = [torch.zeros_like(c) for c in caches_k]
    g = torch.Generator(device=cuda).manual_seed(3)
    base = [torch.randint(-32768, 32767, (CT, H, D), generator=g, device=cuda, dtype=torch.int16)
            for _ in range(2)]
    poses = random_walk(48, seed=11, revisit_every=8)
    tot = 0
    bad = torch.zeros((), dtype=torch.int64, device=cuda)
    checked = 0
    for c in range(len(poses)):
        for layer in range(LAYERS):
            for kv, cache in ((0, caches_k[layer]), (1, caches_v[layer])):
                cache[0, tot:tot + CT].view(torch.int16).copy_(base[kv] ^ _tag(c, layer, kv))
        R = st.add_chunk_from([ck[0, tot:tot + CT] for ck in caches_k], [cv[0, tot:tot + CT] for cv in caches_v],
                              poses[c], poses[c])
        R_o = orc.add_chunk(poses[c], poses[c])
        assert R == R_o, (c, R, R_o)
        assert [m.born for m in st.bank] == orc.bank_borns()
        tot = st.write_into_caches(caches_k, caches_v, R)
        layout = orc.layout(R_o)
        assert tot == len(layout) * CT
        for i, born in enumerate(layout):
            for layer in range(LAYERS):
                for kv, cache in ((0, caches_k[layer]), (1, caches_v[layer])):
                    got = cache[0, i * CT:(i + 1) * CT].view(torch.int16)
                    bad += (got != (base[kv] ^ _tag(born, layer, kv))).sum()
        checked += 1
        if c % 8 == 7:
            assert int(bad) == 0, f"byte mismatches after chunk {c}"
    assert int(bad) == 0 and checked == len(poses)
    assert len(st.bank) == sp.K                     # the bank filled and evicted at full size
    assert any(e[0] == "evict" for e in st.events)


def _attn_ref_heads(q, k, v, heads, b):
    """fp32 softmax(q k^T / sqrt(128)) v on the GPU for the given heads of batch b."""
    out = []
    with torch.no_grad():
        for h in heads:
            qh = q[b, :, h].float()
            kh = k[b, :, h].float()
            vh = v[b, :, h].float()
            s = (qh @ kh.T) * (1.0 / np.sqrt(D))
            out.append(torch.softmax(s, dim=-1) @ vh)
    return out


@pytest.mark.parametrize("Lk", [63360, 66000])
@pytest.mark.parametrize("heads", [24, 3])
def test_attention_at_stress_shapes(cuda, Lk, heads):
    """Batch 4 (four rollouts), 2640 queries over 63360 (the literal 24-chunk
    budget) and 66000 keys (the budget plus the chunk), 24 heads and the 3 heads
    one rank holds at 8 GPUs; several heads of every batch element against an fp32
    reference, within max-abs 2e-2 and mean-abs 2e-3."""
    from reworld_b200 import chunk_attention
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=cuda).manual_seed(Lk + heads)
    B = 4
    q = torch.randn(B, CT, heads, D, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, Lk, heads, D, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, Lk, heads, D, generator=g, device=cuda).to(torch.bfloat16)
    out = chunk_attention(q, k, v)
    torch.cuda.synchronize()
    check = [0, heads - 1] if heads > 3 else list(range(heads))
    for b in range(B):
        refs = _attn_ref_heads(q, k, v, check, b)
        for h, ref in zip(check, refs):
            err = (out[b, :, h].float() - ref).abs()
            assert err.max().item() < 2e-2 and err.mean().item() < 2e-3, (b, h, err.max().item())
    # every head of every batch element: a convex combination of the values, row by row
    vmin = v.float().amin(dim=1, keepdim=True)
    vmax = v.float().amax(dim=1, keepdim=True)
    o = out.float()
    assert torch.isfinite(o).all()
    assert bool(((o >= vmin - 1e-2) & (o <= vmax + 1e-2)).all())


class _RMSNorm(torch.nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)).type_as(x) * self.weight


class _PropSelfAttn5B(torch.nn.Module):
    """Parameter container with the attribute names of CausalWanPropSelfAttention
    at the Wan2.2-TI2V-5B width."""

    def __init__(self, dim=3072, heads=24, eps=1e-6):
        super().__init__()
        self.num_heads, self.head_dim = heads, dim // heads
        self.local_attn_size, self.sink_size, self.max_attention_size = -1, 0, None
        self.q, self.k, self.v, self.o = (torch.nn.Linear(dim, dim) for _ in range(4))
        self.norm_q, self.norm_k = _RMSNorm(dim, eps), _RMSNorm(dim, eps)
        self.pose_mlp = torch.nn.Sequential(torch.nn.Linear(12, 256), torch.nn.SiLU(),
                                            torch.nn.Linear(256, self.head_dim // 2))
        self.value_proj, self.prope_proj = torch.nn.Linear(dim, dim), torch.nn.Linear(dim, dim)


def _ulps(a, b):
    def ordered(t):
        x = np.asarray(torch_bf16_to_bits(t)).astype(np.int32) & 0xFFFF
        return np.where(x & 0x8000, -(x & 0x7FFF), x)
    return np.abs(ordered(a) - ordered(b))


@pytest.mark.parametrize("norm_w,with_ctx", [("normal", False), ("ones", False), ("ones", True)])
def test_installed_forward_at_5b_width(cuda, norm_w, with_ctx):
    """The installed drop-in forward with 3072 channels and 24 heads on one
    660-token chunk (the 352x640 grid 3 x 11 x 20) over 1 sink + 2 recent cached
    chunks, bf16, weights N(0, 0.02) (RMSNorm weights N(0, 0.02) as written, or
    ones), against the oracle of the reference forward on the CPU.  The new K rows
    equal the oracle's RMSNorm + RoPE of the same bf16 projection rows (one bf16
    unit of the norm's fp32 summation order at most, in under 1 % of elements);
    the output is within the attention tolerance."""
    from reworld_b200.self_attn import install
    C = H * D
    f, h, w = 3, 11, 20
    ct = f * h * w
    n0 = 3 * ct
    cap = 4 * ct
    gen = torch.Generator().manual_seed(17 + (norm_w == "ones") + 2 * with_ctx)
    mod = _PropSelfAttn5B()
    W = {}
    with torch.no_grad():
        for n, p in mod.named_parameters():
            if n.startswith("norm_") and norm_w == "ones":
                val = torch.ones(p.shape)
            else:
                val = torch.randn(p.shape, generator=gen) * 0.02
            W[n] = val.to(torch.bfloat16)
            p.copy_(val)
    mod = mod.to(device=cuda, dtype=torch.bfloat16)
    install([type("Blk", (), {"self_attn": mod})()])
    x = torch.randn(1, ct, C, generator=gen).to(torch.bfloat16)
    k0 = torch.randn(1, n0, H, D, generator=gen).to(torch.bfloat16)
    v0 = torch.randn(1, n0, H, D, generator=gen).to(torch.bfloat16)
    ctx = None
    if with_ctx:
        from reworld_b200.poses import random_walk
        ctx = torch.from_numpy(np.stack(random_walk(6, seed=2)))[None].to(torch.bfloat16)
    freqs = orope.build_freqs(128, 12 / 22, 20 / 40)
    cache = {"k": torch.zeros(1, cap, H, D, dtype=torch.bfloat16, device=cuda),
             "v": torch.zeros(1, cap, H, D, dtype=torch.bfloat16, device=cuda),
             "global_end_index": torch.tensor([n0], device=cuda), "local_end_index": torch.tensor([n0], device=cuda)}
    cache["k"][:, :n0], cache["v"][:, :n0] = k0.to(cuda), v0.to(cuda)
    with torch.no_grad():
        y = mod.forward(x.to(cuda), torch.tensor([ct]), torch.tensor([[f, h, w]]), freqs, None, kv_cache=cache,
                        current_start=n0, prope_context=ctx.to(cuda) if ctx is not None else None)
        # the same bf16 projection rows the module fed its norm/RoPE/store kernel
        k_rows = torch.nn.functional.linear(x.to(cuda), mod.k.weight, mod.k.bias).cpu()
    torch.cuda.synchronize()
    assert [int(cache["global_end_index"]), int(cache["local_end_index"])] == [n0 + ct, n0 + ct]
    assert torch.equal(cache["k"][:, :n0].cpu(), k0) and torch.equal(cache["v"][:, :n0].cpu(), v0)
    knew = cache["k"][:, n0:n0 + ct].cpu()
    if not with_ctx:
        kn = osa.rms_norm(k_rows, W["norm_k.weight"], 1e-6).view(1, ct, H, D)
        kr = orope.causal_rope_apply(kn.float().numpy(), [(f, h, w)], freqs, start_frame=n0 // (h * w))
        want = torch.from_numpy(kr).to(torch.bfloat16)
        u = _ulps(knew, want)
        assert (u == 0).mean() > 0.99, (u == 0).mean()
        # a one-unit difference of the normed k before the rotation moves the rotated pair by
        # at most one unit of the pair's magnitude (the rotation keeps |pair|)
        a = knew.float().view(1, ct, H, D // 2, 2)
        b = want.float().view(1, ct, H, D // 2, 2)
        mag = b.norm(dim=-1, keepdim=True)
        assert bool(((a - b).abs() <= mag * 2.0 ** -6 + 1e-30).all()), (a - b).abs().max()
    kc = {"k": torch.zeros(1, cap, H, D, dtype=torch.bfloat16), "v": torch.zeros(1, cap, H, D, dtype=torch.bfloat16),
          "global_end_index": torch.tensor([n0]), "local_end_index": torch.tensor([n0])}
    kc["k"][:, :n0], kc["v"][:, :n0] = k0, v0
    y_ref, kc_ref = osa.prop_self_attn_forward(W, x, (f, h, w), freqs, kc, n0, prope_context=ctx, num_heads=H)
    if with_ctx:
        # the PM-RoPE phase comes from the pose MLP evaluated on the GPU vs the CPU
        assert (knew.float() - kc_ref["k"][:, n0:n0 + ct].float()).abs().max() < 0.05
    err = (y.float().cpu() - y_ref.float()).abs()
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3, (err.max().item(), err.mean().item())


def test_chunk_pose_of_device_context_matches_reference(cuda):
    """The reference computes the chunk pose from the model's prope_context on the
    GPU (compressed.py:355-377); the package's chunk_pose on a device tensor gives
    the fixture's bits."""
    import os
    from reworld_b200.landmark import chunk_pose
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "pipeline.npz"))
    for i, (T, fpc, dt) in enumerate(gi.POSE_CASES):
        ctx = torch.from_numpy(gold[f"pose{i}_ctx"]).to(getattr(torch, dt)).to(cuda)
        got = chunk_pose(ctx, fpc)
        assert np.array_equal(got.view(np.uint32), gold[f"pose{i}_out"].view(np.uint32)), i
