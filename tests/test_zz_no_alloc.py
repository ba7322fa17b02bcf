"""rw_attn_fwd_noalloc: chunk attention for callers that cannot allocate device memory.

Some hosts cannot give this library a workspace: a runtime that owns all device
memory behind its own allocator, or a real-time streaming loop where a cudaMalloc
(which can synchronise the whole device) would stall frame delivery.  For them
rw_attn_fwd_noalloc keeps the key-split scratch in a fixed array inside the
library.  These tests call it through the C ABI and check it against the
regular entry point (caller-provided workspace) on two calls in a row, and that
shapes needing more scratch than the array holds are refused.

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


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 2640, 34320, 24), (2, 300, 1000, 2)])
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


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda):
    from reworld_b200 import _native
    lib = _native.lib()
    cap = 80 * 1024 * 1024
    shape = None
    for H in range(1, 65):                         # find a head count whose split exceeds the array
        if lib.rw_attn_workspace_bytes(1, 2048, 8192, H) > cap:
            shape = (1, 2048, 8192, H)
            break
    if shape is None:
        pytest.skip("no shape in the scan needs more scratch than the array on this GPU")
    B, Lq, Lk, H = shape
    q = torch.zeros(B, Lq, H, 128, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(B, Lk, H, 128, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros_like(q)
    st = _native.status_tensor(cuda)
    assert _noalloc(lib, q, k, k, out, st, _native.stream_ptr(cuda)) == -5    # RW_ERR_CAPACITY
    assert b"capacity" in lib.rw_error_string(-5)
