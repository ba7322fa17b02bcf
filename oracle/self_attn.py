"""Oracle of CausalWanPropSelfAttention.forward, inference branch (TEST
INFRASTRUCTURE, see oracle/__init__.py).

Restates wan_5b/modules/action_model.py:148-319 with a KV cache (no sliding
window, the shipped configuration's inference_local_attn_size = -1): q/k/v
Linear + RMSNorm over all heads (wan_5b/modules/model.py:73-89), the PRoPE
phase delta = pose_mlp(vec R, t) and V-side P^-1 residual when prope_context is
given, RoPE(+delta) on q and the new k at the chunk's start frame, cache write,
attention over cache[:, :local_end] (reference CPU SDPA path), o projection
(+ P residual).  torch on CPU; the RoPE comes from oracle.rope.
"""
import math

import numpy as np
import torch

from .attention import reference_attention_cpu
from .numerics import bits_to_torch_bf16, f32_to_bf16_bits
from .rope import causal_rope_apply, pm_rope_delta_apply


def rms_norm(x, w, eps):
    """WanRMSNorm.forward (wan_5b/modules/model.py:82-89): fp32 mean of squares,
    rsqrt, .type_as(x), times the weight."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return y.type_as(x) * w


def _lin(x, w, b):
    return torch.nn.functional.linear(x, w, b)


def _inv_se3(T):
    R = T[..., :3, :3]
    t = T[..., :3, 3:]
    Ri = R.transpose(-1, -2)
    out = T.clone()
    out[..., :3, :3] = Ri
    out[..., :3, 3:] = -Ri @ t
    out[..., 3, :3] = 0
    out[..., 3, 3] = 1
    return out


def _se3(x, ctx_all, mode, fs):
    B, L, H, D = x.shape
    nf = L // fs
    ctx = ctx_all[:, -nf:].to(x.dtype)
    if mode == "P_inv":
        ctx = _inv_se3(ctx)
    xv = x.permute(0, 2, 1, 3).reshape(B, H, nf, fs, D // 4, 4)
    y = torch.matmul(ctx.unsqueeze(1).unsqueeze(3).unsqueeze(4), xv.unsqueeze(-1)).squeeze(-1)
    return y.reshape(B, H, L, D).permute(0, 2, 1, 3)


def _to_dtype_vals(arr, dtype):
    """float32 array of values already representable in `dtype` -> torch tensor of dtype."""
    t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32))
    return t.to(dtype)


def prop_self_attn_forward(W, x, grid, freqs, kv_cache, current_start, prope_context=None, num_heads=2,
                           eps=1e-6):
    """W: dict of parameters (state_dict names, tensors of the module dtype).
    Returns (out, new kv_cache dict).  dtype follows x (fp32 or bf16)."""
    dtype = x.dtype
    b, s = x.shape[:2]
    n = num_heads
    d = x.shape[-1] // n
    q = rms_norm(_lin(x, W["q.weight"], W["q.bias"]), W["norm_q.weight"], eps).view(b, s, n, d)
    k = rms_norm(_lin(x, W["k.weight"], W["k.bias"]), W["norm_k.weight"], eps).view(b, s, n, d)
    v = _lin(x, W["v.weight"], W["v.bias"]).view(b, s, n, d)
    f, h, w = grid
    fs = h * w
    delta = None
    if prope_context is not None:
        c_all = torch.cat([prope_context[..., :3, :3].flatten(-2), prope_context[..., :3, 3]], dim=-1)
        T = s // fs
        c = c_all[:, -T:]
        hdn = torch.nn.functional.silu(_lin(c, W["pose_mlp.0.weight"], W["pose_mlp.0.bias"]))
        dl = _lin(hdn, W["pose_mlp.2.weight"], W["pose_mlp.2.bias"])          # [B, T, d/2]
        delta = dl.unsqueeze(2).expand(-1, -1, fs, -1).reshape(b, T * fs, d // 2).unsqueeze(2)
        v_p = _se3(v, prope_context, "P_inv", fs)
        v = (v.flatten(2) + _lin(v_p.flatten(2), W["value_proj.weight"], W["value_proj.bias"])).view(b, s, n, d)
    start_f = current_start // fs
    g = [(max(1, s // fs), h, w)]

    def rope(t):
        if dtype == torch.bfloat16:
            y = causal_rope_apply(t.float().numpy(), g, freqs, start_frame=start_f)
            if delta is not None:
                y = pm_rope_delta_apply(y, delta.float().numpy())
            return bits_to_torch_bf16(f32_to_bf16_bits(y)).view(t.shape)
        # fp32: the fp64 product is cast to fp32 (type_as), delta in fp32
        y = _rope_f32(t, g, freqs, start_f)
        if delta is not None:
            yc = torch.view_as_complex(y.reshape(*y.shape[:-1], d // 2, 2))
            rot = torch.polar(torch.ones_like(delta.float()), delta.float())
            y = torch.view_as_real(yc * rot).flatten(-2)
        return y

    q_f, k_f = rope(q), rope(k)
    ge = int(kv_cache["global_end_index"].item())
    le = int(kv_cache["local_end_index"].item())
    cur_end = current_start + s
    local_end = le + cur_end - ge
    local_start = local_end - s
    kc = {kk: vv.clone() for kk, vv in kv_cache.items()}
    kc["k"][:, local_start:local_end] = k_f
    kc["v"][:, local_start:local_end] = v
    o = reference_attention_cpu(q_f, kc["k"][:, :local_end], kc["v"][:, :local_end], dtype=dtype)
    kc["global_end_index"].fill_(cur_end)
    kc["local_end_index"].fill_(local_end)
    out = _lin(o.flatten(2), W["o.weight"], W["o.bias"])
    if prope_context is not None:
        x_p = _se3(o, prope_context, "P", fs)
        out = out + _lin(x_p.flatten(2), W["prope_proj.weight"], W["prope_proj.bias"])
    return out, kc


def _rope_f32(t, grid, freqs, start_f):
    """causal_rope_apply for fp32 activations: complex128 product cast back to fp32."""
    n, c = t.size(2), t.size(3) // 2
    fr = freqs.split([c - 2 * (c // 3), c // 3, c // 3], dim=1)
    f, h, w = grid[0]
    seq = f * h * w
    xi = torch.view_as_complex(t[0, :seq].to(torch.float64).reshape(seq, n, -1, 2))
    fi = torch.cat([fr[0][start_f:start_f + f].view(f, 1, 1, -1).expand(f, h, w, -1),
                    fr[1][:h].view(1, h, 1, -1).expand(f, h, w, -1),
                    fr[2][:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1).reshape(seq, 1, -1)
    y = torch.view_as_real(xi * fi).flatten(2)
    y = torch.cat([y, t[0, seq:].to(torch.float64)])
    return y.unsqueeze(0).type_as(t)
