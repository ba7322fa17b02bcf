"""ctypes binding of the package's CUDA library (include/reworld_b200.h).

The library is the only compute path: if it is missing or fails to load, the
import raises, there is no fallback.
"""
import ctypes
import os

import torch

from .build import lib_path

c_int = ctypes.c_int
c_ll = ctypes.c_longlong
c_float = ctypes.c_float
c_vp = ctypes.c_void_p

RW_OK = 0
RW_STATUS_BITS = {
    0x01: "TMA producer wait timed out",
    0x02: "MMA issuer wait timed out",
    0x04: "softmax/epilogue wait timed out",
    0x08: "bulk-copy wait timed out",
    0x10: "descriptor or slot index out of range",
    0x20: "cross-rank barrier wait timed out",
}


class RwRope(ctypes.Structure):
    _fields_ = [
        ("freqs", c_vp),
        ("max_pos", c_int),
        ("start_frame", c_int),
        ("grid_f", c_int),
        ("grid_h", c_int),
        ("grid_w", c_int),
        ("c_t", c_int),
        ("c_h", c_int),
        ("c_w", c_int),
        ("delta_cs", c_vp),
    ]


class RwSpSync(ctypes.Structure):
    """rw_sp_sync_t: cross-rank ordering carried by a sequence-parallel kernel."""
    _fields_ = [("sig_ptrs", c_vp), ("counter", c_vp), ("P", c_int), ("rank", c_int), ("wait_slot", c_int),
                ("wait_epoch", c_int), ("signal_slot", c_int), ("signal_epoch", c_int), ("timeout_ms", c_int),
                ("pad", c_int)]


class RwCopyDesc(ctypes.Structure):
    _fields_ = [("src", c_vp), ("dst", c_vp), ("nbytes", c_ll)]


# name -> (restype, argtypes)
_SIGNATURES = {
    "rw_attn_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int] + [c_ll] * 12
                    + [c_float, ctypes.POINTER(RwRope), c_vp, c_ll, c_vp, c_vp]),
    "rw_attn_fwd_prope": (c_int, [c_vp] * 6 + [c_int] * 6 + [c_ll] * 15
                          + [c_float, ctypes.POINTER(RwRope), c_vp, c_ll, c_vp, c_vp]),
    "rw_attn_workspace_bytes": (c_ll, [c_int, c_int, c_int, c_int]),
    "rw_attn_fwd_noalloc": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int] + [c_ll] * 12
                            + [c_float, ctypes.POINTER(RwRope), c_vp, c_vp]),
    "rw_rope_kv_store": (c_int, [c_vp] * 6 + [c_int] * 5 + [c_ll] * 18 + [ctypes.POINTER(RwRope), c_vp]),
    "rw_qkv_norm_rope_store": (c_int, [c_vp] * 8 + [c_int] * 5 + [c_float] * 2 + [c_ll] * 15
                               + [ctypes.POINTER(RwRope), c_vp, c_vp]),
    "rw_se3_block_apply": (c_int, [c_vp] * 3 + [c_int] * 5 + [c_ll] * 6 + [c_vp]),
    "rw_row_norm": (c_int, [c_vp] * 4 + [c_ll, c_int, c_ll, c_ll, c_float, c_int, c_vp]),
    "rw_copy_chunks": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "rw_bank_step": (c_int, [c_vp, c_int, c_int, c_int, c_vp, c_int, c_int, c_vp, c_int, c_int, c_vp, c_vp]),
    "rw_a2a_pack": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp]),
    "rw_a2a_unpack": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp]),
    "rw_sp_scatter_qkv": (c_int, [c_vp, c_vp, c_vp] + [c_ll] * 6 + [c_vp, c_vp, c_vp] + [c_int] * 7
                          + [ctypes.POINTER(RwRope), ctypes.POINTER(RwSpSync), c_vp, c_vp]),
    "rw_sp_wait": (c_int, [ctypes.POINTER(RwSpSync), c_vp, c_vp]),
    "rw_sp_scatter_out": (c_int, [c_vp, c_vp] + [c_int] * 5 + [c_vp]),
    "rw_sp_barrier": (c_int, [c_vp] + [c_int] * 5 + [c_vp, c_vp]),
    "rw_sp_attn_fwd": (c_int, [c_vp] * 3 + [c_int] * 4 + [c_ll] * 6 + [c_vp] + [c_int] * 3
                       + [c_float, ctypes.POINTER(RwRope), c_vp, c_ll, ctypes.POINTER(RwSpSync), c_vp, c_vp]),
    "rw_gemm_bf16": (c_int, [c_vp, c_ll, c_vp, c_ll, c_vp, c_vp, c_ll, c_vp, c_ll, c_int, c_int, c_int, c_int, c_vp,
                             c_ll, c_vp, c_vp]),
    "rw_gemm_workspace_bytes": (c_ll, [c_int, c_int, c_int]),
    "rw_error_string": (ctypes.c_char_p, [c_int]),
    "rw_abi_version": (c_int, []),
}

ABI_VERSION = 4
_lib = None


def exported_symbols():
    """Names of every C-ABI entry point declared in include/reworld_b200.h."""
    return sorted(_SIGNATURES)


def lib():
    """Loads the CUDA library once; raises ImportError when it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise ImportError(
            f"reworld_b200 CUDA library not built ({path} missing); run `python reworld_b200/build.py`")
    handle = ctypes.CDLL(path)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(handle, name, None)
        if fn is None:
            raise ImportError(f"{path} does not export {name}")
        fn.restype = res
        fn.argtypes = args
    if handle.rw_abi_version() != ABI_VERSION:
        raise ImportError(f"{path}: ABI version {handle.rw_abi_version()} != {ABI_VERSION}")
    _lib = handle
    return _lib


def check(code, what):
    if code != RW_OK:
        msg = lib().rw_error_string(code).decode()
        raise RuntimeError(f"{what} failed: {msg} (code {code})")


def stream_ptr(device=None):
    return c_vp(torch.cuda.current_stream(device).cuda_stream)


_status = {}


def status_tensor(device):
    """Per-device int32 status word the kernels atomically OR error bits into."""
    idx = device.index if isinstance(device, torch.device) else int(device)
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def check_status(device=None, reset=True):
    """Raises if any kernel on `device` reported an asynchronous failure."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    t = status_tensor(device)
    v = int(t[0].item())
    if reset and v:
        t.zero_()
    if v:
        reasons = [m for b, m in RW_STATUS_BITS.items() if v & b]
        raise RuntimeError(f"reworld_b200 kernel status 0x{v:x}: {'; '.join(reasons)}")
