"""The oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the reference run on CPU)."""
import numpy as np
import pytest
import torch

import inputs as gi
from oracle import attention as oatt
from oracle import landmark as olm
from oracle import rope as orope
from oracle import self_attn as osa
from oracle.numerics import bits_to_torch_bf16, f32_to_bf16_bits, bf16_bits_to_f32, torch_bf16_to_bits


def test_bf16_rounding_matches_torch():
    x = torch.randn(100000, dtype=torch.float32) * 3
    x[:5] = torch.tensor([0.0, -0.0, float("inf"), -float("inf"), 1e-40])
    assert np.array_equal(f32_to_bf16_bits(x.numpy()), torch_bf16_to_bits(x.to(torch.bfloat16)))
    d = torch.randn(100000, dtype=torch.float64) * 5
    assert np.array_equal(f32_to_bf16_bits(d.numpy().astype(np.float32)), torch_bf16_to_bits(d.to(torch.bfloat16)))


@pytest.mark.parametrize("i", range(len(gi.ATTN_CASES)))
def test_attention_oracle_matches_reference(golden, i):
    g = golden["attention"]
    q, k, v = gi.attention_case(i)
    assert abs(gi.checksum(q, k, v) - float(g[f"c{i}_checksum"])) < 1e-6, "input generator drifted"
    ref = bf16_bits_to_f32(g[f"c{i}_o"]).reshape(q.shape)
    # the reference's CPU path itself (SDPA branch) reproduces the fixture bit for bit
    o = oatt.reference_attention_cpu(q, k, v)
    assert np.array_equal(torch_bf16_to_bits(o), g[f"c{i}_o"].reshape(q.shape))
    # the float64 restatement agrees within bf16 output rounding
    o64 = oatt.attention_f64(q.float().numpy(), k.float().numpy(), v.float().numpy())
    err = np.abs(o64 - ref)
    assert err.max() < 1e-2 and err.mean() < 1e-3


@pytest.mark.parametrize("tag", ["q", "k"])
def test_rmsnorm_oracle_matches_reference(golden, tag):
    """The oracle's WanRMSNorm restatement reproduces the reference's bf16 bits
    (zero row, tiny and large rows included)."""
    g = golden["rmsnorm"]
    x, wq, wk = gi.rmsnorm_case()
    assert abs(gi.checksum(x, wq, wk) - float(g["checksum"])) < 1e-6, "input generator drifted"
    y = osa.rms_norm(x, wq if tag == "q" else wk, gi.RMSNORM_EPS)
    assert y.dtype == torch.bfloat16
    assert np.array_equal(torch_bf16_to_bits(y), g[f"norm_{tag}"].reshape(x.shape))


def _block_params_bf16():
    import torch.nn as nn
    dim, H, ffn = gi.BLOCK_DIM, gi.BLOCK_HEADS, gi.BLOCK_FFN
    shapes = {"norm3.weight": (dim,), "norm3.bias": (dim,), "ffn.0.weight": (ffn, dim), "ffn.0.bias": (ffn,),
              "ffn.2.weight": (dim, ffn), "ffn.2.bias": (dim,)}
    for nm in ("q", "k", "v", "o"):
        shapes[f"cross_attn.{nm}.weight"], shapes[f"cross_attn.{nm}.bias"] = (dim, dim), (dim,)
    shapes["cross_attn.norm_q.weight"] = shapes["cross_attn.norm_k.weight"] = (dim,)
    vals = gi.block_params(shapes)
    return {k: v.to(torch.bfloat16) for k, v in vals.items()}, vals


def test_block_oracle_matches_reference(golden):
    """The oracle's cross_attn_ffn reproduces every stage of the reference block's bits."""
    from oracle import block as ob
    g = golden["block"]
    W, vals = _block_params_bf16()
    x, context, e = gi.block_inputs()
    assert abs(gi.checksum(*[vals[n] for n in sorted(vals)], x, context, e) - float(g["checksum"])) < 1e-6
    st = ob.cross_attn_ffn(W, x, context, e, gi.BLOCK_HEADS, gi.BLOCK_FRAMES)
    for name in ("norm3", "cross_attn", "x1", "norm2", "ffn", "out"):
        assert np.array_equal(torch_bf16_to_bits(st[name]), g[name].reshape(st[name].shape)), name


def test_rope_table_matches_reference(golden):
    g = golden["rope"]
    fr = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    assert np.array_equal(torch.view_as_real(fr[:48]).numpy(), g["freqs_head"])


@pytest.mark.parametrize("sf", [0, 7, 33])
def test_causal_rope_bit_exact(golden, sf):
    g = golden["rope"]
    x, grid, delta = gi.rope_case()
    assert abs(gi.checksum(x, delta) - float(g["checksum"])) < 1e-6
    fr = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    y = orope.causal_rope_apply(x.float().numpy(), [grid], fr, start_frame=sf)
    assert np.array_equal(f32_to_bf16_bits(y), g[f"rope_sf{sf}"].reshape(y.shape))


def test_pm_rope_delta_bit_exact(golden):
    g = golden["rope"]
    x, grid, delta = gi.rope_case()
    fr = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    y = orope.causal_rope_apply(x.float().numpy(), [grid], fr, start_frame=7)
    yd = orope.pm_rope_delta_apply(y, delta.numpy())
    assert np.array_equal(f32_to_bf16_bits(yd), g["rope_delta_sf7"].reshape(yd.shape))


def _self_attn_params():
    dim, H = gi.SELF_ATTN_DIM, gi.SELF_ATTN_HEADS
    shapes = {"q.weight": (dim, dim), "q.bias": (dim,), "k.weight": (dim, dim), "k.bias": (dim,),
              "v.weight": (dim, dim), "v.bias": (dim,), "o.weight": (dim, dim), "o.bias": (dim,),
              "norm_q.weight": (dim,), "norm_k.weight": (dim,),
              "pose_mlp.0.weight": (256, 12), "pose_mlp.0.bias": (256,),
              "pose_mlp.2.weight": (64, 256), "pose_mlp.2.bias": (64,),
              "value_proj.weight": (dim, dim), "value_proj.bias": (dim,),
              "prope_proj.weight": (dim, dim), "prope_proj.bias": (dim,)}
    return gi.self_attn_params(shapes)


@pytest.mark.parametrize("tag,dtype,with_ctx", gi.SELF_ATTN_TAGS)
def test_self_attn_oracle_matches_reference(golden, tag, dtype, with_ctx):
    g = golden["self_attn"]
    vals, gen = _self_attn_params()
    k0, v0, x, ctx = gi.self_attn_inputs(gen, dtype, with_ctx)
    assert abs(gi.checksum(*[vals[n] for n in sorted(vals)], k0, v0, x, *([ctx] if ctx is not None else []))
               - float(g[f"{tag}_checksum"])) < 1e-6
    W = {n: t.to(dtype) for n, t in vals.items()}
    f, h, w = gi.SELF_ATTN_GRID
    ct = f * h * w
    n0 = gi.SELF_ATTN_CACHED * ct
    cap = (gi.SELF_ATTN_CACHED + 2) * ct
    cache = {"k": torch.zeros(1, cap, 2, 128, dtype=dtype), "v": torch.zeros(1, cap, 2, 128, dtype=dtype),
             "global_end_index": torch.tensor([n0]), "local_end_index": torch.tensor([n0])}
    cache["k"][:, :n0], cache["v"][:, :n0] = k0, v0
    fr = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    y, kc = osa.prop_self_attn_forward(W, x, (f, h, w), fr, cache, n0, prope_context=ctx)
    np.testing.assert_array_equal(kc["k"][:, n0:n0 + ct].float().numpy(), g[f"{tag}_knew"])
    np.testing.assert_array_equal(kc["v"][:, n0:n0 + ct].float().numpy(), g[f"{tag}_vnew"])
    assert [int(kc["global_end_index"]), int(kc["local_end_index"])] == list(g[f"{tag}_ends"])
    np.testing.assert_allclose(y.float().numpy(), g[f"{tag}_y"], rtol=0, atol=1e-5)


@pytest.mark.parametrize("name", gi.landmark_runs_names())
def test_landmark_oracle_matches_reference(golden, name):
    g = golden["landmark"]
    poses, ct, H, D, ns, rw, K, rk, mode = gi.landmark_runs()[name]
    assert abs(float(np.sum(np.stack(poses).astype(np.float64))) - float(g[f"{name}_pose_checksum"])) < 1e-9
    ob = olm.OracleBank(ns, rw, K, rk, mode)
    N = len(poses) - 1
    Rg, Bg = g[f"{name}_R"], g[f"{name}_bank"]
    layouts = []
    for c in range(N):
        R = ob.add_chunk(poses[c], poses[c + 1])
        assert R == [int(x) for x in Rg[c] if x >= 0], f"retrieval differs at chunk {c}"
        assert ob.bank_borns() == [int(x) for x in Bg[c] if x >= 0], f"bank differs at chunk {c}"
        assert len(ob.layout(R)) * ct == int(g[f"{name}_tot"][c])
        layouts.append(ob.layout(R))
    ev = [(0 if e[0] == "add" else 1, e[1]) for e in ob.events]
    assert ev == [tuple(int(x) for x in e) for e in g[f"{name}_events"]]
    # reconstruct the cache bytes of the last chunks from the layout and the chunk K/V
    tail = g[f"{name}_cache_tail"]
    for t, c in enumerate(range(N - 3, N)):
        lay = layouts[c]
        cap = tail.shape[3]          # tail: [3, k/v, B=1, cap, H, D]
        kb = np.zeros((cap, H, D), np.uint16)
        vb = np.zeros((cap, H, D), np.uint16)
        for i, born in enumerate(lay):
            k, v = gi.landmark_kv(name, born, ct, H, D)
            kb[i * ct:(i + 1) * ct] = torch_bf16_to_bits(k)
            vb[i * ct:(i + 1) * ct] = torch_bf16_to_bits(v)
        assert np.array_equal(kb, tail[t, 0, 0])
        assert np.array_equal(vb, tail[t, 1, 0])


def test_budget_split_matches_pipeline_rule():
    assert olm.budget_split(12, 1, 5, 30) == (1, 5, 6, 30)
    assert olm.budget_split(24, 1, 7, 120) == (1, 7, 16, 120)
    assert olm.budget_split(4, 1, 5, 2) == (1, 2, 1, 2)


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_oracle_matches_reference(golden, world):
    from oracle import ulysses as ou
    g = golden["ulysses"]
    shards = [gi.ulysses_shard(r, world).numpy() for r in range(world)]
    ys = ou.seq_to_head(shards)
    zs = ou.head_to_seq(ys)
    for r in range(world):
        np.testing.assert_array_equal(ys[r], g[f"p{world}_r{r}_y"])
        np.testing.assert_array_equal(zs[r], g[f"p{world}_r{r}_z"])
