"""torch.nn.functional.linear on the package's tcgen05 GEMM (rw_gemm_bf16).

`linear(x, weight, bias=None, gelu=False, residual=None, out=None)` computes
x @ weight.T + bias (bf16 in and out, fp32 accumulation, one rounding),
optionally followed by the tanh GELU, or added to `residual` the way torch adds
two bf16 tensors.  It replaces the reference's nn.Linear calls on the cached
chunk's path: the q/k/v projections (wan_5b/modules/action_model.py:164-166),
value_proj and its residual (:203), o + prope_proj (:308-318) and the block's
FFN (:547-556).  Operands must be bf16 CUDA tensors whose rows are contiguous
(any row stride that is a multiple of 8 elements); K must be a multiple of 64
and N of 128.
"""
import torch

from . import _native
from ._native import c_vp

EPI_NONE, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESIDUAL = 0, 1, 2, 3

_workspaces = {}


def _workspace(device, nbytes):
    """Per-device workspace of the GEMM's shared last round: zeroed once when
    (re)allocated; every call leaves its flags at zero again.  Calls on one device
    are stream-ordered on the current stream, so they never overlap on it."""
    if nbytes <= 0:
        return None
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[idx] = ws
    return ws


def _rows(t, name):
    """[..., n] tensor -> (2-D view [rows, n], row stride) without copying."""
    if t.stride(-1) != 1:
        raise ValueError(f"{name}: the last dimension must be contiguous")
    if t.dim() == 1:
        return t.unsqueeze(0), t.shape[0]
    try:
        m = t.view(-1, t.shape[-1]) if t.dim() > 2 else t
    except RuntimeError:
        raise ValueError(f"{name}: leading dimensions must collapse into one row stride") from None
    return m, m.stride(0) if m.shape[0] > 1 else max(m.shape[1], 8)


def linear(x, weight, bias=None, gelu=False, residual=None, out=None):
    """x: bf16 [..., K]; weight: bf16 [N, K]; bias: bf16 [N] or None; residual:
    bf16 [..., N] (may be `out` itself).  Returns bf16 [..., N] (`out` if given)."""
    for t, n in ((x, "x"), (weight, "weight")):
        if not t.is_cuda or t.dtype != torch.bfloat16:
            raise ValueError(f"{n} must be a bf16 CUDA tensor")
    K = x.shape[-1]
    N, Kw = weight.shape
    if Kw != K:
        raise ValueError(f"x has {K} features, weight expects {Kw}")
    lead = x.shape[:-1]
    a, lda = _rows(x, "x")
    w, ldb = _rows(weight, "weight")
    M = a.shape[0]
    if out is None:
        out = torch.empty(*lead, N, dtype=torch.bfloat16, device=x.device)
    if out.shape != (*lead, N) or out.dtype != torch.bfloat16:
        raise ValueError("out must be bf16 [..., N]")
    c, ldc = _rows(out, "out")
    epi = EPI_NONE
    bptr = None
    if bias is not None:
        if bias.dtype != torch.bfloat16 or bias.shape != (N,) or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous bf16 [N] tensor")
        bptr = c_vp(bias.data_ptr())
        epi = EPI_BIAS
    elif gelu or residual is not None:
        bias = torch.zeros(N, dtype=torch.bfloat16, device=x.device)
        bptr = c_vp(bias.data_ptr())
    rptr, ldr = None, 0
    if gelu and residual is not None:
        raise ValueError("gelu and residual cannot be combined")
    if gelu:
        epi = EPI_BIAS_GELU
    if residual is not None:
        if residual.shape != (*lead, N) or residual.dtype != torch.bfloat16:
            raise ValueError("residual must be bf16 [..., N]")
        r, ldr = _rows(residual, "residual")
        rptr = c_vp(r.data_ptr())
        epi = EPI_BIAS_RESIDUAL
    lib = _native.lib()
    with torch.cuda.device(x.device):
        st = _native.status_tensor(x.device)
        ws = _workspace(x.device, lib.rw_gemm_workspace_bytes(M, N, K))
        code = lib.rw_gemm_bf16(c_vp(a.data_ptr()), lda, c_vp(w.data_ptr()), ldb, bptr, rptr, ldr,
                                c_vp(c.data_ptr()), ldc, M, N, K, epi,
                                c_vp(ws.data_ptr()) if ws is not None else None, ws.numel() if ws is not None else 0,
                                c_vp(st.data_ptr()), _native.stream_ptr(x.device))
    _native.check(code, "rw_gemm_bf16")
    return out


def supported(x, weight):
    """True when linear() can run this projection: bf16 CUDA operands, K a multiple
    of 64 and N of 128."""
    return (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and x.shape[-1] % 64 == 0 and weight.shape[0] % 128 == 0 and weight.shape[1] == x.shape[-1])


def module_linear(mod, x, **kw):
    """An nn.Linear `mod` applied to bf16 x on linear(); raises for shapes outside
    the kernel's domain (no silent library fallback)."""
    if mod.bias is not None and mod.bias.dtype != torch.bfloat16:
        raise NotImplementedError("the GEMM runs bf16 modules (bias dtype differs)")
    if not supported(x, mod.weight):
        raise NotImplementedError(f"linear {tuple(mod.weight.shape)} on {tuple(x.shape)}: the GEMM needs bf16, "
                                  "in_features % 64 == 0 and out_features % 128 == 0")
    return linear(x, mod.weight, mod.bias, **kw)
