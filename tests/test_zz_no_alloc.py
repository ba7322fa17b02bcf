"""rw_attn_fwd_noalloc: chunk attention for callers that cannot allocate device memory.

Some hosts cannot give this library a workspace: a runtime that owns all device
memory behind its own allocator, or a real-time streaming loop where a cudaMalloc
(which can synchronise the whole device) would stall frame delivery.  For them
rw_attn_fwd_noalloc keeps the key-split scratch in a fixed array inside the
library.  These tests call it through the C ABI and check it against the
regular entry point (caller-provided workspace) on two calls in a row, and that
the array covers the scratch of every shape on this GPU.

This file is named so that pytest collects it last.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _noalloc(lib, q, k, v, out, status, stream):
    B, Lq, H, D = q.shape
    return lib.rw_attn_fwd_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), B, Lq, k.shape[1], H, D,
        *q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3],
        1.0 / math.sqrt(D), None, ctypes.c_void_p(status.data_ptr()), stream)


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 2640, 34320, 24), (2, 300, 6000, 2)])
def test_noalloc_matches_regular_entry_point_on_two_calls(cuda, B, Lq, Lk, H):
    from reworld_b200 import _native, chunk_attention
    lib = _native.lib()
    need = lib.rw_attn_workspace_bytes(B, Lq, Lk, H)
    assert 0 < need <= 80 * 1024 * 1024          # this shape does use the scratch array
    st = _native.status_tensor(cuda)
    stream = _native.stream_ptr(cuda)
    for call in range(2):                          # the second call reuses the array's old contents
        g = torch.Generator(device=cuda).manual_seed(1000 * call + Lq + H)
        q = torch.randn(B, Lq, H, 128, generator=g, device=cuda).to(torch.bfloat16)
        k = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
        v = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
        ref = chunk_attention(q, k, v)             # regular entry point, caller workspace
        out = torch.full_like(q, float("nan"))
        assert _noalloc(lib, q, k, v, out, st, stream) == 0
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert err.max().item() < MAX_ABS and err.mean().item() < MEAN_ABS, (call, err.max().item())
    _native.check_status(cuda)


def test_noalloc_scratch_array_covers_every_shape(cuda):
    """The split needs 0 bytes or 2 slots of 133,120 bytes per resident pair,
    whatever the shape (at most 74 pairs on a B200: 19.7 MB), so on this GPU no
    shape reaches the RW_ERR_CAPACITY refusal; a sweep over batch, head and
    length counts (the 704x1280 chunk and the B = 4, 66000-key stress shape
    among them) checks that bound against the array's size."""
    from reworld_b200 import _native
    lib = _native.lib()
    cap = 80 * 1024 * 1024
    slot_pair = 2 * (128 * 256 + 2 * 256) * 4          # two partial slots of one pair
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    seen = set()
    for B in (1, 2, 4):
        for H in (1, 3, 6, 12, 24, 40, 64):
            for Lq, Lk in ((1, 1), (300, 1000), (660, 2640), (2640, 34320), (2640, 66000), (5280, 4096)):
                need = lib.rw_attn_workspace_bytes(B, Lq, Lk, H)
                assert need >= 0 and need % slot_pair == 0, (B, H, Lq, Lk, need)
                assert need <= (sms // 2) * slot_pair <= cap, (B, H, Lq, Lk, need)
                seen.add(need > 0)
    assert seen == {False, True}                       # the sweep has shapes with and without a split
    assert (sms // 2) * slot_pair < cap // 4           # a B200 uses under a quarter of the array
    assert b"capacity" in lib.rw_error_string(-5)      # RW_ERR_CAPACITY, the refusal's message
