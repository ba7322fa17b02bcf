"""Rounding helpers (TEST INFRASTRUCTURE, see oracle/__init__.py)."""
import numpy as np


def f32_to_bf16_bits(x):
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns
    (the conversion torch's .to(bfloat16) performs on CPU)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b):
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x):
    """fp32/fp64 values rounded to bf16, returned as fp32.  fp64 inputs are
    rounded to fp32 first (torch's double -> bfloat16 cast goes through float)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x).astype(np.float32)))


def torch_bf16_to_bits(t):
    import torch
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def bits_to_torch_bf16(b):
    import torch
    return torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)
