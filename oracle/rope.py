"""3-D RoPE oracle (TEST INFRASTRUCTURE, see oracle/__init__.py).

rope_params / build_freqs follow wan_5b/modules/model.py:29-39 and
wan_5b/modules/causal_model.py:790-807 (temporal table unscaled, h/w tables with
the spatial position-interpolation scale), computed with torch on CPU exactly as
the reference does.  causal_rope_apply follows causal_model.py:156-184 and
pm_rope_delta_apply follows wan_5b/modules/action_model.py:40-51, restated in
numpy with explicit real arithmetic (separately rounded products and sums) and
the reference's bf16 casts (fp64 -> fp32 -> bf16).
"""
import numpy as np
import torch

from .numerics import round_bf16


def rope_params(max_seq_len, dim, theta=10000, pos_scale=1.0):
    """model.py:29-39: polar(1, (pos * pos_scale) outer theta^(-2i/dim)), complex128."""
    freqs = torch.outer(
        torch.arange(max_seq_len).to(torch.float64) * float(pos_scale),
        1.0 / torch.pow(theta, torch.arange(0, dim, 2).to(torch.float64).div(dim)))
    return torch.polar(torch.ones_like(freqs), freqs)


def build_freqs(head_dim=128, scale_h=1.0, scale_w=1.0, max_pos=1024):
    """causal_model.py:802-807: cat of temporal (unscaled), height and width tables, [max_pos, D/2]."""
    d = head_dim
    return torch.cat([
        rope_params(max_pos, d - 4 * (d // 6)),
        rope_params(max_pos, 2 * (d // 6), pos_scale=scale_h),
        rope_params(max_pos, 2 * (d // 6), pos_scale=scale_w),
    ], dim=1)


def rope_split(head_dim=128):
    c = head_dim // 2
    return (c - 2 * (c // 3), c // 3, c // 3)


def causal_rope_apply(x, grid_sizes, freqs, start_frame=0):
    """causal_model.py:156-184.  x: float array [B, L, n, d] holding bf16 values;
    grid_sizes: [(f, h, w)] per sample; freqs: complex128 [max_pos, d/2]
    (numpy or torch).  Returns fp32 array of bf16 values."""
    x = np.asarray(x, dtype=np.float32)
    fr = freqs.numpy() if isinstance(freqs, torch.Tensor) else np.asarray(freqs)
    B, L, n, d = x.shape
    c = d // 2
    st, sh, sw = rope_split(d)
    f_t, f_h, f_w = fr[:, :st], fr[:, st:st + sh], fr[:, st + sh:]
    out = x.copy()
    for i, (f, h, w) in enumerate(grid_sizes):
        seq = f * h * w
        xi = x[i, :seq].astype(np.float64).reshape(seq, n, c, 2)
        fi = np.concatenate([
            np.broadcast_to(f_t[start_frame:start_frame + f].reshape(f, 1, 1, -1), (f, h, w, st)),
            np.broadcast_to(f_h[:h].reshape(1, h, 1, -1), (f, h, w, sh)),
            np.broadcast_to(f_w[:w].reshape(1, 1, w, -1), (f, h, w, sw)),
        ], axis=-1).reshape(seq, 1, c)
        ar, ai = xi[..., 0], xi[..., 1]
        cr, ci = fi.real, fi.imag
        yr = ar * cr - ai * ci
        yi = ar * ci + ai * cr
        y = np.stack([yr, yi], axis=-1).reshape(seq, n, d)
        out[i, :seq] = round_bf16(y)
    return out


def pm_rope_delta_apply(x, delta):
    """action_model.py:40-51.  x: [B, L, n, d] bf16 values; delta: [B, L, 1, d/2]
    fp32 phases.  cos/sin come from torch.polar in fp32 like the reference."""
    cr, ci = delta_cos_sin(delta)
    return pm_rope_apply_cs(x, cr, ci)


def pm_rope_apply_cs(x, cr, ci):
    """pm_rope_delta_apply with the phase factor given as its fp32 (cos, sin)
    parts [B, L, 1, d/2] (e.g. the factor torch.polar formed on the GPU, where
    the reference runs it)."""
    x = np.asarray(x, dtype=np.float32)
    cr = np.asarray(cr, dtype=np.float32)
    ci = np.asarray(ci, dtype=np.float32)
    B, L, n, d = x.shape
    xc = x.reshape(B, L, n, d // 2, 2)
    ar, ai = xc[..., 0], xc[..., 1]
    zr = ar * cr - ai * ci
    zi = ar * ci + ai * cr
    return round_bf16(np.stack([zr, zi], axis=-1).reshape(B, L, n, d))


def delta_cos_sin(delta):
    """(cos, sin) of the PM-RoPE phases as torch.polar computes them in fp32."""
    dt = torch.as_tensor(np.asarray(delta, dtype=np.float32))
    rot = torch.polar(torch.ones_like(dt), dt)
    return rot.real.numpy().astype(np.float32), rot.imag.numpy().astype(np.float32)
