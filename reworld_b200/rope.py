"""3-D RoPE tables and kernel arguments.

The model's frequency table is the reference's `freqs` buffer
(wan_5b/modules/causal_model.py:790-807: temporal table unscaled, height/width
tables with the spatial position-interpolation scales, built by rope_params,
wan_5b/modules/model.py:29-39), a complex128 [1024, head_dim/2] tensor.  The
kernels read it as (real, imag) float64 pairs; `RopeArgs` carries the per-call
position (start frame, token grid) and the optional PM-RoPE phase.
"""
import ctypes

import torch

from ._native import RwRope


def rope_params(max_seq_len, dim, theta=10000, pos_scale=1.0):
    """complex128 [max_seq_len, dim/2]: polar(1, pos * pos_scale * theta^(-2i/dim))."""
    freqs = torch.outer(
        torch.arange(max_seq_len).to(torch.float64) * float(pos_scale),
        1.0 / torch.pow(theta, torch.arange(0, dim, 2).to(torch.float64).div(dim)))
    return torch.polar(torch.ones_like(freqs), freqs)


def build_freqs(head_dim=128, scale_h=1.0, scale_w=1.0, max_pos=1024):
    """The model's table: temporal (head_dim - 4*(head_dim//6)), height and width sections."""
    d = head_dim
    return torch.cat([rope_params(max_pos, d - 4 * (d // 6)),
                      rope_params(max_pos, 2 * (d // 6), pos_scale=scale_h),
                      rope_params(max_pos, 2 * (d // 6), pos_scale=scale_w)], dim=1)


def rope_split(head_dim=128):
    c = head_dim // 2
    return (c - 2 * (c // 3), c // 3, c // 3)


_table_cache = {}


def device_table(freqs, device):
    """float64 (real, imag) view of a complex128 freqs table on `device` (cached per tensor)."""
    key = (id(freqs), freqs.data_ptr(), str(device))
    t = _table_cache.get(key)
    if t is None or t[0] is not freqs:
        tab = torch.view_as_real(freqs.to(torch.complex128)).to(device).contiguous()
        _table_cache[key] = (freqs, tab)
        return tab
    return t[1]


class RopeArgs:
    """Arguments of one RoPE application: token grid (f, h, w) of the chunk, the
    temporal start frame and the optional PM-RoPE phase delta [B, f, head_dim/2]
    (per frame, fp32).  `table` is the device float64 view of the freqs table."""

    def __init__(self, table, grid, start_frame, head_dim=128, delta=None):
        if table.dtype != torch.float64 or table.dim() != 3 or table.shape[-1] != 2:
            raise ValueError("table must be the float64 (real, imag) view of the freqs table")
        self.table = table
        self.grid = tuple(int(x) for x in grid)
        self.start_frame = int(start_frame)
        self.head_dim = head_dim
        self.delta_cs = None
        if delta is not None:
            d = delta.to(device=table.device, dtype=torch.float32)
            rot = torch.polar(torch.ones_like(d), d)          # the reference's fp32 phase factor
            self.delta_cs = torch.view_as_real(rot).contiguous()
        f, h, w = self.grid
        if self.start_frame + f > table.shape[0] or h > table.shape[0] or w > table.shape[0]:
            raise ValueError("RoPE positions exceed the frequency table")

    def struct(self):
        c_t, c_h, c_w = rope_split(self.head_dim)
        f, h, w = self.grid
        return RwRope(ctypes.c_void_p(self.table.data_ptr()), self.table.shape[0], self.start_frame, f, h, w,
                      c_t, c_h, c_w,
                      ctypes.c_void_p(self.delta_cs.data_ptr()) if self.delta_cs is not None else None)
