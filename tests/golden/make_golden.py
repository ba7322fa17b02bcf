"""Generates the golden fixtures in this directory by running the REFERENCE itself
(ReWorld, read from the reference checkout) on CPU.

Usage:  python tests/golden/make_golden.py [--reference PATH]

The reference is imported without its heavy package __init__ files: diffusers
(absent here) is stubbed with the two symbols the modules import, the wan /
wan_5b packages are registered as empty packages, and the flash-attention flags
of wan_5b/modules/attention.py are switched off so attention() takes its torch
SDPA branch (:164-179), the reference's CPU path.

Inputs are drawn from seeded torch generators by inputs.py (shared with the
tests); each fixture keeps a checksum of its inputs and the reference's outputs:
  attention.npz     reference attention() on bf16 q/k/v (several shapes)
  rope.npz          reference rope table rows, causal_rope_apply and
                    pm_rope_delta_apply on a bf16 chunk
  self_attn.npz     CausalWanPropSelfAttention.forward (inference branch) with a
                    KV cache, reduced width (2 heads x 128), fp32 and bf16,
                    with and without prope_context: output, new cache rows
  landmark.npz      LandmarkCacheV2 runs: retrieved index lists, bank contents,
                    events and write_into_cache bytes of the last chunks
  rmsnorm.npz       WanRMSNorm (the q/k norms) on bf16 rows of the 5B width
  block.npz         the DiT block's cross_attn_ffn (norm3, MultiShotT2VCrossAttention,
                    norm2 + modulation, FFN, gated residuals) at reduced width, bf16
  ulysses.npz       wan_5b/distributed/util.all_to_all (seq->head and back)
                    over gloo process groups of 2 and 4 ranks (gloo lacks
                    all_to_all; it is emulated by its definition with all_gather)
  pipeline.npz      the compressed pipeline's budget split (_init_compression_state)
                    and chunk pose (_compute_chunk_pose), both compiled from the
                    pipeline's source file and run on stub objects (importing the
                    pipeline module would pull in the whole model stack)
"""
import argparse
import functools
import math
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def setup_reference(ref):
    sys.path.insert(0, ref)
    diffusers = types.ModuleType("diffusers")
    cu = types.ModuleType("diffusers.configuration_utils")

    class ConfigMixin:
        pass

    cu.ConfigMixin = ConfigMixin
    cu.register_to_config = lambda f: f
    mu = types.ModuleType("diffusers.models.modeling_utils")
    mu.ModelMixin = torch.nn.Module
    dm = types.ModuleType("diffusers.models")
    sys.modules.update({"diffusers": diffusers, "diffusers.configuration_utils": cu,
                        "diffusers.models": dm, "diffusers.models.modeling_utils": mu})
    for pkg in ("wan", "wan.modules", "wan_5b", "wan_5b.modules", "wan_5b.distributed"):
        m = types.ModuleType(pkg)
        m.__path__ = [os.path.join(ref, *pkg.split("."))]
        sys.modules[pkg] = m
    import wan_5b.modules.attention as att
    att.FLASH_ATTN_2_AVAILABLE = False
    att.FLASH_ATTN_3_AVAILABLE = False
    return att


def bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))   # repo root: reworld_b200.poses
sys.path.insert(0, HERE)
import inputs as gi   # noqa: E402


def gen_attention(att):
    out = {"n_cases": np.array(len(gi.ATTN_CASES))}
    for i in range(len(gi.ATTN_CASES)):
        q, k, v = gi.attention_case(i)
        o = att.attention(q, k, v)
        out[f"c{i}_checksum"] = np.array(gi.checksum(q, k, v))
        out[f"c{i}_o"] = bits(o)
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)


def gen_rope():
    from wan_5b.modules.model import rope_params
    from wan_5b.modules.causal_model import causal_rope_apply
    from wan_5b.modules.action_model import pm_rope_delta_apply
    d = gi.HEAD_DIM
    freqs = torch.cat([rope_params(1024, d - 4 * (d // 6)),
                       rope_params(1024, 2 * (d // 6), pos_scale=gi.ROPE_SCALE_H),
                       rope_params(1024, 2 * (d // 6), pos_scale=gi.ROPE_SCALE_W)], dim=1)
    x, (f, h, w), delta = gi.rope_case()
    grid = torch.tensor([[f, h, w]])
    outs = {}
    for sf in (0, 7, 33):
        outs[f"rope_sf{sf}"] = bits(causal_rope_apply(x, grid, freqs, start_frame=sf).type_as(x))
    yd = pm_rope_delta_apply(causal_rope_apply(x, grid, freqs, start_frame=7).type_as(x), delta)
    np.savez_compressed(os.path.join(HERE, "rope.npz"), freqs_head=torch.view_as_real(freqs[:48]).numpy(),
                        checksum=np.array(gi.checksum(x, delta)), rope_delta_sf7=bits(yd), **outs)


def gen_rmsnorm():
    from wan_5b.modules.model import WanRMSNorm
    x, wq, wk = gi.rmsnorm_case()
    out = {"checksum": np.array(gi.checksum(x, wq, wk))}
    for tag, w in (("q", wq), ("k", wk)):
        norm = WanRMSNorm(gi.RMSNORM_DIM, eps=gi.RMSNORM_EPS)
        with torch.no_grad():
            norm.weight.copy_(w.float())
        norm = norm.to(torch.bfloat16)
        with torch.no_grad():
            out[f"norm_{tag}"] = bits(norm(x))
    np.savez_compressed(os.path.join(HERE, "rmsnorm.npz"), **out)


def gen_block(att):
    import torch.nn as nn
    import wan_5b.modules.causal_model as cm
    from wan_5b.modules.model import WanLayerNorm
    cm.flash_attention = att.attention   # CPU: the reference's SDPA branch (no flash-attention wheel)
    dim, H, ffn_dim = gi.BLOCK_DIM, gi.BLOCK_HEADS, gi.BLOCK_FFN
    mods = nn.ModuleDict({
        "norm3": WanLayerNorm(dim, 1e-6, elementwise_affine=True),
        "cross_attn": cm.MultiShotT2VCrossAttention(dim, H, (-1, -1), True, 1e-6),
        "norm2": WanLayerNorm(dim, 1e-6),
        "ffn": nn.Sequential(nn.Linear(dim, ffn_dim), nn.GELU(approximate="tanh"), nn.Linear(ffn_dim, dim)),
    })
    shapes = {n: tuple(p.shape) for n, p in mods.named_parameters()}
    vals = gi.block_params(shapes)
    with torch.no_grad():
        for n, p in mods.named_parameters():
            p.copy_(vals[n])
    mods = mods.to(torch.bfloat16)
    x, context, e_mod = gi.block_inputs()
    F, fs = gi.BLOCK_FRAMES, gi.BLOCK_FS
    lens = torch.tensor([gi.BLOCK_CTX])
    e = e_mod.chunk(6, dim=2)
    with torch.no_grad():
        # the block's cross_attn_ffn (action_model.py:547-556), with the reference's modules
        n3 = mods["norm3"](x)
        ca = mods["cross_attn"](n3, context, lens)
        x1 = x + ca
        n2 = mods["norm2"](x1)
        y = mods["ffn"]((n2.unflatten(dim=1, sizes=(F, fs)) * (1 + e[4]) + e[3]).flatten(1, 2))
        x2 = x1 + (y.unflatten(dim=1, sizes=(F, fs)) * e[5]).flatten(1, 2)
    out = {"checksum": np.array(gi.checksum(*[vals[n] for n in sorted(vals)], x, context, e_mod))}
    for name, t in (("norm3", n3), ("cross_attn", ca), ("x1", x1), ("norm2", n2), ("ffn", y), ("out", x2)):
        out[name] = bits(t)
    np.savez_compressed(os.path.join(HERE, "block.npz"), **out)


def gen_self_attn(att):
    import wan_5b.modules.action_model as am
    from wan_5b.modules.model import rope_params
    dim, H, d = gi.SELF_ATTN_DIM, gi.SELF_ATTN_HEADS, gi.HEAD_DIM
    f, h, w = gi.SELF_ATTN_GRID
    ct = f * h * w
    n0 = gi.SELF_ATTN_CACHED * ct
    out = {}
    for tag, dtype, with_ctx in gi.SELF_ATTN_TAGS:
        am.attention = functools.partial(att.attention, dtype=torch.float32) if dtype == torch.float32 \
            else att.attention
        mod = am.CausalWanPropSelfAttention(dim, H, -1, 0, True, 1e-6)
        shapes = {n: tuple(p.shape) for n, p in mod.named_parameters()}
        vals, g = gi.self_attn_params(shapes)
        with torch.no_grad():
            for n, p in mod.named_parameters():
                p.copy_(vals[n])
        mod = mod.to(dtype)
        freqs = torch.cat([rope_params(1024, d - 4 * (d // 6)),
                           rope_params(1024, 2 * (d // 6), pos_scale=gi.ROPE_SCALE_H),
                           rope_params(1024, 2 * (d // 6), pos_scale=gi.ROPE_SCALE_W)], dim=1)
        k0, v0, x, ctx = gi.self_attn_inputs(g, dtype, with_ctx)
        cap = (gi.SELF_ATTN_CACHED + 2) * ct
        cache = {"k": torch.zeros(1, cap, H, d, dtype=dtype), "v": torch.zeros(1, cap, H, d, dtype=dtype),
                 "global_end_index": torch.tensor([n0]), "local_end_index": torch.tensor([n0])}
        cache["k"][:, :n0] = k0
        cache["v"][:, :n0] = v0
        with torch.no_grad():
            y = mod(x, torch.tensor([ct]), torch.tensor([[f, h, w]]), freqs, None, kv_cache=cache,
                    current_start=n0, prope_context=ctx)
        out[f"{tag}_checksum"] = np.array(gi.checksum(*[vals[n] for n in sorted(vals)], k0, v0, x,
                                                      *([ctx] if ctx is not None else [])))
        out[f"{tag}_y"] = y.float().numpy()
        out[f"{tag}_knew"] = cache["k"][:, n0:n0 + ct].float().numpy()
        out[f"{tag}_vnew"] = cache["v"][:, n0:n0 + ct].float().numpy()
        out[f"{tag}_untouched"] = np.array(bool(torch.equal(cache["k"][:, :n0], k0) and
                                                torch.equal(cache["k"][:, n0 + ct:], torch.zeros_like(cache["k"][:, n0 + ct:]))))
        out[f"{tag}_ends"] = np.array([int(cache["global_end_index"].item()), int(cache["local_end_index"].item())])
    np.savez_compressed(os.path.join(HERE, "self_attn.npz"), **out)


def gen_landmark():
    from longctx.inference.landmark_cache_v2 import LandmarkCacheV2
    out = {}
    for name, (poses, ct, H, D, ns, rw, K, rk, mode) in gi.landmark_runs().items():
        lm = LandmarkCacheV2(ct, n_sink=ns, recent_w=rw, K=K, retrieve_k=rk, mode=mode)
        N = len(poses) - 1
        Rs, bank_borns, tots, cache_bytes = [], [], [], []
        cap = (ns + rw + (K if mode == "a" else rk)) * ct + 4
        for c in range(N):
            k, v = gi.landmark_kv(name, c, ct, H, D)
            R = lm.add_chunk(k, v, poses[c], poses[c + 1])
            Rs.append(R)
            bank_borns.append([e.born for e in lm.bank])
            kc = {"k": torch.zeros(1, cap, H, D, dtype=torch.bfloat16),
                  "v": torch.zeros(1, cap, H, D, dtype=torch.bfloat16)}
            tots.append(lm.write_into_cache(kc, R))
            cache_bytes.append(np.stack([bits(kc["k"]), bits(kc["v"])]))
        maxr = max(1, max(len(r) for r in Rs))
        Ra = np.full((N, maxr), -1, dtype=np.int32)
        for i, r in enumerate(Rs):
            Ra[i, :len(r)] = r
        maxb = max(1, max(len(b) for b in bank_borns))
        Ba = np.full((N, maxb), -1, dtype=np.int32)
        for i, b in enumerate(bank_borns):
            Ba[i, :len(b)] = b
        out[f"{name}_R"] = Ra
        out[f"{name}_bank"] = Ba
        out[f"{name}_events"] = np.array([[0 if e[0] == "add" else 1, e[1]] for e in lm.events],
                                         dtype=np.int32).reshape(-1, 2)
        out[f"{name}_tot"] = np.array(tots)
        # cache bytes of the last 3 chunks (the full sequence is reproducible from the layout)
        out[f"{name}_cache_tail"] = np.stack(cache_bytes[-3:])
        out[f"{name}_pose_checksum"] = np.array(float(np.sum(np.stack(poses).astype(np.float64))))
    np.savez_compressed(os.path.join(HERE, "landmark.npz"), **out)


def _gloo_all_to_all(output_list, input_list, group=None, **kw):
    """dist.all_to_all for the gloo backend (which lacks it), by its definition:
    output_list[j] on rank i receives input_list[i] of rank j."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    me = dist.get_rank(group)
    for j in range(world):
        gathered = [torch.empty_like(input_list[j]) for _ in range(world)]
        dist.all_gather(gathered, input_list[j].contiguous(), group=group)
        if j == me:
            for src in range(world):
                output_list[src].copy_(gathered[src])


def _a2a_worker(rank, world, port, ref, path_out):
    import torch.distributed as dist
    setup_reference(ref)
    dist.all_to_all = _gloo_all_to_all
    from wan_5b.distributed.util import all_to_all
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x = gi.ulysses_shard(rank, world)                            # sequence shard, all heads
    y = all_to_all(x, scatter_dim=2, gather_dim=1)               # full sequence, H/P heads
    z = all_to_all(y, scatter_dim=1, gather_dim=2)               # back to the sequence shard
    np.savez(f"{path_out}.{rank}.npz", y=y.numpy(), z=z.numpy())
    dist.destroy_process_group()


def gen_ulysses(ref):
    import tempfile
    import torch.multiprocessing as mp
    out = {}
    for world, port in ((2, 29611), (4, 29612)):
        tmp = tempfile.mkdtemp()
        base = os.path.join(tmp, "a2a")
        mp.spawn(_a2a_worker, args=(world, port, ref, base), nprocs=world, join=True)
        for r in range(world):
            d = np.load(f"{base}.{r}.npz")
            out[f"p{world}_r{r}_y"] = d["y"]
            out[f"p{world}_r{r}_z"] = d["z"]
    np.savez_compressed(os.path.join(HERE, "ulysses.npz"), **out)


def _compressed_methods(ref):
    """_init_compression_state and _compute_chunk_pose of
    CausalDiffusionInferenceCompressedPipeline, compiled from
    pipeline/causal_diffusion_inference_compressed.py as plain functions."""
    import ast
    path = os.path.join(ref, "pipeline", "causal_diffusion_inference_compressed.py")
    tree = ast.parse(open(path).read(), path)
    cls = next(n for n in tree.body
               if isinstance(n, ast.ClassDef) and n.name == "CausalDiffusionInferenceCompressedPipeline")
    fns = [n for n in cls.body
           if isinstance(n, ast.FunctionDef) and n.name in ("_init_compression_state", "_compute_chunk_pose")]
    ns = {"np": np, "torch": torch}
    exec(compile(ast.Module(body=fns, type_ignores=[]), path, "exec"), ns)
    return ns["_init_compression_state"], ns["_compute_chunk_pose"]


def gen_pipeline(ref):
    import types as _t
    import longctx.inference.landmark_cache as lc_mod
    init_state, chunk_pose = _compressed_methods(ref)

    made = []

    class Recorder:
        def __init__(self, **kw):
            made.append(kw)

    saved = lc_mod.LandmarkCache
    lc_mod.LandmarkCache = Recorder
    rows = []
    try:
        for policy, budget, n_sink, recent_w, landmark_k, cap_chunks in gi.BUDGET_CASES:
            ct = 8
            cfg = _t.SimpleNamespace(enabled=True, policy=policy, budget_chunks=budget, n_sink=n_sink,
                                     recent_w=recent_w, landmark_k=landmark_k, landmark_eps=0.5, retrieve_k=6)
            kv = [{"k": torch.empty(1, cap_chunks * ct, 1, 1)}] if cap_chunks else None
            self_ = _t.SimpleNamespace(kvc_cfg=cfg, kv_cache_pos=kv, num_transformer_blocks=1)
            made.clear()
            init_state(self_, ct, 1, 1)
            kw = made[0]
            rows.append([gi.POLICIES.index(policy), budget, n_sink, recent_w, landmark_k, cap_chunks, ct,
                         kw["n_sink"], kw["recent_w"], kw["K"], kw["retrieve_k"], 1 if kw["mode"] == "b" else 0,
                         1 if kw["diverse"] else 0])
    finally:
        lc_mod.LandmarkCache = saved
    out = {"budget": np.array(rows, dtype=np.int64)}
    from reworld_b200.poses import random_walk
    for i, (T, fpc, dt) in enumerate(gi.POSE_CASES):
        ctx = torch.from_numpy(np.stack(random_walk(T, seed=40 + i, step_t=0.7, step_deg=12.0)))[None]
        ctx = ctx.to(getattr(torch, dt))
        out[f"pose{i}_ctx"] = ctx.float().numpy() if dt == "bfloat16" else ctx.numpy()
        out[f"pose{i}_out"] = chunk_pose(None, ctx, fpc)
    np.savez_compressed(os.path.join(HERE, "pipeline.npz"), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("REWORLD_REFERENCE"),
                    required=not os.environ.get("REWORLD_REFERENCE"),
                    help="path of the reference checkout (or set REWORLD_REFERENCE)")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    att = setup_reference(a.reference)
    todo = a.only.split(",") if a.only else ["attention", "rope", "rmsnorm", "block", "self_attn", "landmark", "ulysses",
                                             "pipeline"]
    if "attention" in todo:
        gen_attention(att)
    if "rope" in todo:
        gen_rope()
    if "rmsnorm" in todo:
        gen_rmsnorm()
    if "block" in todo:
        gen_block(att)
    if "self_attn" in todo:
        gen_self_attn(att)
    if "landmark" in todo:
        gen_landmark()
    if "ulysses" in todo:
        gen_ulysses(a.reference)
    if "pipeline" in todo:
        gen_pipeline(a.reference)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
