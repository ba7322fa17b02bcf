"""Seeded inputs of the golden fixtures, shared by make_golden.py (which feeds
them to the reference) and the tests (which feed them to the oracle and the
CUDA path).  Everything is drawn from torch CPU generators with fixed seeds;
each fixture stores a checksum of its inputs so a change of the generator
stream is caught instead of producing a silent mismatch.
"""
import numpy as np
import torch

ATTN_CASES = [(1, 64, 192, 2), (2, 96, 130, 1), (1, 128, 384, 2), (1, 50, 257, 3)]

SELF_ATTN_DIM, SELF_ATTN_HEADS, HEAD_DIM = 256, 2, 128
SELF_ATTN_GRID = (3, 4, 5)
SELF_ATTN_CACHED = 3                       # cached chunks before the new one
SELF_ATTN_TAGS = (("f32", torch.float32, False), ("f32_ctx", torch.float32, True),
                  ("bf16", torch.bfloat16, False), ("bf16_ctx", torch.bfloat16, True))
ROPE_SCALE_H, ROPE_SCALE_W = 12 / 22, 20 / 40   # spatial position interpolation of the 720p config


def checksum(*tensors):
    h = 0.0
    for t in tensors:
        a = t.detach().float().cpu().numpy().ravel().astype(np.float64)
        h += float(np.sum(a * np.cos(np.arange(a.size) * 0.001)))
    return h


RMSNORM_DIM, RMSNORM_EPS = 3072, 1e-6      # the 5B model's width (24 heads x 128) and its norms' eps


def rmsnorm_case():
    """bf16 rows [2, 12, 3072] for the q/k RMSNorm: Gaussian rows with per-row
    scales from 1e-3 to 1e2, one all-zero row and one row holding a single large
    entry; norm weights ~ 1 + N(0, 0.05) rounded to bf16 (one for q, one for k)."""
    g = torch.Generator().manual_seed(23)
    B, L, C = 2, 12, RMSNORM_DIM
    scale = torch.logspace(-3, 2, B * L).reshape(B, L, 1)
    x = torch.randn(B, L, C, generator=g) * scale
    x[0, 5] = 0.0
    x[1, 7] = 0.0
    x[1, 7, 100] = 50.0
    x = x.to(torch.bfloat16)
    wq = (1.0 + torch.randn(C, generator=g) * 0.05).to(torch.bfloat16)
    wk = (1.0 + torch.randn(C, generator=g) * 0.05).to(torch.bfloat16)
    return x, wq, wk


BLOCK_DIM, BLOCK_HEADS, BLOCK_FFN = 256, 2, 512   # reduced width of the DiT block's cross-attn + FFN
BLOCK_FRAMES, BLOCK_FS, BLOCK_CTX = 2, 20, 16      # frames x tokens per frame; text tokens


def block_params(param_shapes):
    """Parameter values in sorted-name order (weights N(0, 0.05), norm weights 1 + N(0, 0.05))."""
    g = torch.Generator().manual_seed(31)
    vals = {}
    for name, shape in sorted(param_shapes.items()):
        if name.endswith("norm_q.weight") or name.endswith("norm_k.weight") or name == "norm3.weight":
            vals[name] = 1.0 + torch.randn(shape, generator=g) * 0.05
        else:
            vals[name] = torch.randn(shape, generator=g) * 0.05
    return vals


def block_inputs():
    """x [1, F*fs, dim], context [1, ctx, dim] and the block's modulation e [1, F, 6, dim], bf16."""
    g = torch.Generator().manual_seed(32)
    L = BLOCK_FRAMES * BLOCK_FS
    x = torch.randn(1, L, BLOCK_DIM, generator=g).to(torch.bfloat16)
    context = torch.randn(1, BLOCK_CTX, BLOCK_DIM, generator=g).to(torch.bfloat16)
    e = (torch.randn(1, BLOCK_FRAMES, 6, BLOCK_DIM, generator=g) * 0.1).to(torch.bfloat16)
    return x, context, e


def attention_case(i):
    B, Lq, Lk, H = ATTN_CASES[i]
    g = torch.Generator().manual_seed(100 + i)
    q = torch.randn(B, Lq, H, HEAD_DIM, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Lk, H, HEAD_DIM, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Lk, H, HEAD_DIM, generator=g).to(torch.bfloat16)
    return q, k, v


def rope_case():
    """x [1, L, 3, 128] bf16 (grid 3x4x5 plus 4 tokens past the grid) and delta [1, L, 1, 64]."""
    g = torch.Generator().manual_seed(7)
    f, h, w = 3, 4, 5
    L = f * h * w + 4
    x = (torch.randn(1, L, 3, HEAD_DIM, generator=g) * 2.0).to(torch.bfloat16)
    delta = torch.randn(1, L, 1, HEAD_DIM // 2, generator=g) * 0.5
    return x, (f, h, w), delta


def self_attn_params(param_shapes):
    """Parameter values in sorted-name order, drawn from one generator (norm weights ~ 1 + N(0, 0.02))."""
    g = torch.Generator().manual_seed(12)
    vals = {}
    for name, shape in sorted(param_shapes.items()):
        vals[name] = torch.randn(shape, generator=g) * 0.02
    for nm in ("norm_q.weight", "norm_k.weight"):
        vals[nm] = 1.0 + torch.randn(param_shapes[nm], generator=g) * 0.02
    return vals, g


def self_attn_inputs(g, dtype, with_ctx):
    """Cache contents, new-chunk activations and (optionally) the PRoPE context, drawn after the params."""
    dim, H, d = SELF_ATTN_DIM, SELF_ATTN_HEADS, HEAD_DIM
    f, h, w = SELF_ATTN_GRID
    ct = f * h * w
    n = SELF_ATTN_CACHED * ct
    k0 = torch.randn(1, n, H, d, generator=g).to(dtype)
    v0 = torch.randn(1, n, H, d, generator=g).to(dtype)
    x = torch.randn(1, ct, dim, generator=g).to(dtype)
    ctx = None
    if with_ctx:
        T = SELF_ATTN_CACHED * f + f
        ang = torch.randn(T, generator=g) * 0.3
        c, s = torch.cos(ang), torch.sin(ang)
        P = torch.zeros(1, T, 4, 4)
        P[0, :, 0, 0], P[0, :, 0, 2], P[0, :, 2, 0], P[0, :, 2, 2] = c, s, -s, c
        P[0, :, 1, 1] = 1.0
        P[0, :, 3, 3] = 1.0
        P[0, :, :3, 3] = torch.randn(T, 3, generator=g) * 0.5
        ctx = P.to(dtype)
    return k0, v0, x, ctx


def landmark_runs():
    """name -> (poses, ct, H, D, n_sink, recent_w, K, retrieve_k, mode)."""
    from reworld_b200.poses import random_walk, yaw_walk
    return {
        "walk_cfg2": (random_walk(64, seed=0), 2, 1, 8, 1, 5, 30, 6, "b"),
        "revisit_cfg4": (random_walk(40, seed=1, revisit_every=8), 2, 1, 8, 1, 5, 30, 6, "b"),
        "yaw_always_full": (yaw_walk(201, seed=1, step_t=0.25, step_yaw_deg=30.0), 2, 1, 8, 1, 5, 30, 6, "b"),
        "stress_cfg5": (random_walk(160, seed=5), 2, 1, 8, 1, 7, 120, 16, "b"),
        "small_k": (yaw_walk(40, seed=3, step_t=0.2, step_yaw_deg=40.0), 3, 2, 8, 1, 3, 8, 3, "b"),
        "mode_a": (yaw_walk(30, seed=4), 2, 1, 8, 1, 3, 6, 6, "a"),
    }


def landmark_kv(name, c, ct, H, D):
    """K and V of chunk c of run `name` (bf16 [ct, H, D])."""
    g = torch.Generator().manual_seed(10_000 * (sorted(landmark_runs_names()).index(name) + 1) + c)
    k = torch.randn(ct, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(ct, H, D, generator=g).to(torch.bfloat16)
    return k, v


def landmark_runs_names():
    return ["walk_cfg2", "revisit_cfg4", "yaw_always_full", "stress_cfg5", "small_k", "mode_a"]


ULYSSES_SHAPE = (1, 12, 8, 16)   # B, L, H, D


def ulysses_shard(rank, world):
    B, L, H, D = ULYSSES_SHAPE
    g = torch.Generator().manual_seed(1000 + rank)
    return torch.randn(B, L // world, H, D, generator=g)


# compressed pipeline (pipeline.npz): budget-split cases
# (policy, budget_chunks, n_sink, recent_w, landmark_k, cache chunks or 0 = no cache given)
BUDGET_CASES = [
    ("v15b", 12, 1, 5, 30, 0), ("v15b", 24, 1, 7, 120, 0), ("v15b", 24, 1, 7, 10, 0), ("v15b", 3, 1, 5, 30, 0),
    ("v15b", 2, 1, 5, 30, 0), ("v15b", 1, 1, 5, 30, 0), ("v15c", 12, 2, 5, 30, 0), ("consol", 12, 1, 5, 30, 0),
    ("consol_div", 20, 4, 7, 30, 0), ("v15a", 20, 4, 7, 30, 0), ("v15b", 20, 1, 5, 30, 13),
    ("v15b", 12, 1, 5, 30, 40), ("consol", 30, 1, 5, 8, 9), ("v15b", 9, 0, 4, 6, 0),
]
POLICIES = ["consol", "consol_div", "v15a", "v15b", "v15c"]
# chunk-pose cases: (frames seen T, frames per chunk, prope_context dtype)
POSE_CASES = [(3, 3, "float32"), (7, 3, "float32"), (12, 4, "float32"), (5, 1, "float32"), (9, 3, "bfloat16"),
              (6, 3, "float64")]
