"""The C-ABI library loads and exports every entry point of include/reworld_b200.h;
argument validation runs on the host (no kernel launch, no GPU needed)."""
import ctypes
import os
import re

import pytest

from reworld_b200 import _native
from reworld_b200.landmark import RwBankResult, RwBankState, RwPose

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    src = open(os.path.join(ROOT, "include", "reworld_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rw_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    declared = _header_functions()
    assert declared == _native.exported_symbols()
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.rw_abi_version() == _native.ABI_VERSION


def test_error_strings():
    lib = _native.lib()
    for code in (0, -1, -2, -3, -4, -5, -99):
        assert isinstance(lib.rw_error_string(code), bytes)


def test_struct_sizes_match_header():
    # rw_pose_t: 8 doubles; state/result sizes follow the header layout
    assert ctypes.sizeof(RwPose) == 64
    assert ctypes.sizeof(RwBankState) == 16 + 1024 * 64 + 3 * 1024 * 4
    assert ctypes.sizeof(RwBankResult) == 48 + 2 * 1024 * 4


def test_attn_rejects_bad_arguments_without_launching():
    lib = _native.lib()
    args = [None] * 4 + [1, 128, 128, 1, 128] + [0] * 12 + [0.1, None, None, 0, None, None]
    assert lib.rw_attn_fwd(*args) == -1                    # null pointers
    p = ctypes.c_void_p(16)
    st = [128 * 128, 128, 128] * 4
    assert lib.rw_attn_fwd(p, p, p, p, 1, 128, 128, 1, 64, *st, 0.1, None, None, 0, None, None) == -2   # head_dim 64
    assert lib.rw_attn_fwd(p, p, p, p, 1, 128, 0, 1, 128, *st, 0.1, None, None, 0, None, None) == -1    # Lk = 0
    assert lib.rw_attn_fwd(p, p, p, p, 1, 128, 128, 1, 128, *st, -1.0, None, None, 0, None, None) == -1  # scale <= 0
    odd = ctypes.c_void_p(18)
    assert lib.rw_attn_fwd(odd, p, p, p, 1, 128, 128, 1, 128, *st, 0.1, None, None, 0, None, None) == -1  # misaligned
    bad = [128 * 128, 130, 128] * 4
    assert lib.rw_attn_fwd(p, p, p, p, 1, 128, 128, 1, 128, *bad, 0.1, None, None, 0, None, None) == -1  # stride % 8


def test_other_entry_points_reject_bad_arguments():
    lib = _native.lib()
    assert lib.rw_copy_chunks(None, 0, None, None) == 0         # nothing to do
    assert lib.rw_copy_chunks(None, 3, None, None) == -1
    assert lib.rw_copy_chunks(None, -1, None, None) == -1
    assert lib.rw_bank_step(None, 30, 2, 0, None, 0, 0, None, 6, 1, None, None) == -1
    p = ctypes.c_void_p(64)
    assert lib.rw_bank_step(p, 2000, 2, 0, None, 0, 0, p, 6, 1, p, None) == -1   # K > capacity
    assert lib.rw_bank_step(p, 30, 2, 1, None, 0, 0, p, 6, 1, p, None) == -1     # admit without pose
    assert lib.rw_a2a_pack(p, p, 1, 8, 24, 128, 5, None) == -1                 # heads not divisible
    assert lib.rw_a2a_unpack(None, p, 1, 8, 24, 128, 2, None) == -1
    z = [0] * 18
    assert lib.rw_rope_kv_store(p, p, None, None, p, p, 1, 8, 2, 64, 0, *z, None, None) == -2
    assert lib.rw_rope_kv_store(p, p, p, None, p, p, 1, 8, 2, 128, 0, *z, None, None) == -1
    # rw_qkv_norm_rope_store: every rejection happens before a launch
    s15 = [3 * 256, 3 * 256] * 3 + [256, 256, 128] * 3
    ok8 = [p] * 8
    fn = lib.rw_qkv_norm_rope_store
    assert fn(*ok8, 1, 0, 2, 128, 0, 1e-6, 1e-6, *s15, None, None, None) == 0             # L = 0: nothing to do
    assert fn(*([None] + ok8[1:]), 1, 8, 2, 128, 0, 1e-6, 1e-6, *s15, None, None, None) == -1   # null pointer
    assert fn(*ok8, 1, 8, 2, 64, 0, 1e-6, 1e-6, *s15, None, None, None) == -2             # head_dim 64
    assert fn(*ok8, 1, 8, 289, 128, 0, 1e-6, 1e-6, *s15, None, None, None) == -2          # 6*H*D > 216 KB
    assert fn(*ok8, 1, 8, 2, 128, 0, -1.0, 1e-6, *s15, None, None, None) == -1            # eps < 0
    assert fn(*ok8, 1, 8, 2, 128, -1, 1e-6, 1e-6, *s15, None, None, None) == -1           # dst_start < 0
    assert fn(*([ctypes.c_void_p(18)] + ok8[1:]), 1, 8, 2, 128, 0, 1e-6, 1e-6, *s15, None, None, None) == -1
    assert fn(*ok8, 1, 8, 2, 128, 0, 1e-6, 1e-6, *(s15[:1] + [12] + s15[2:]), None, None, None) == -1  # row stride % 8
    # rw_se3_block_apply
    se = lib.rw_se3_block_apply
    s6 = [0, 256, 128, 0, 256, 128]
    assert se(p, p, p, 1, 0, 2, 128, 20, *s6, None) == 0                  # L = 0: nothing to do
    assert se(None, p, p, 1, 40, 2, 128, 20, *s6, None) == -1             # null pointer
    assert se(p, p, p, 1, 40, 2, 64, 20, *s6, None) == -2                 # head_dim 64
    assert se(p, p, p, 1, 50, 2, 128, 20, *s6, None) == -1                # partial frame
    assert se(p, p, ctypes.c_void_p(72), 1, 40, 2, 128, 20, *s6, None) == -1   # misaligned matrices
    assert se(p, p, p, 1, 40, 2, 128, 20, 0, 260, 128, 0, 256, 128, None) == -1  # stride % 8
    # rw_row_norm
    rn = lib.rw_row_norm
    assert rn(p, p, None, None, 0, 256, 256, 256, 1e-6, 1, None) == 0      # no rows
    assert rn(None, p, None, None, 4, 256, 256, 256, 1e-6, 1, None) == -1  # null x
    assert rn(p, p, None, None, 4, 256, 256, 256, 1e-6, 0, None) == -1     # rms needs a weight
    assert rn(p, p, None, p, 4, 256, 256, 256, 1e-6, 1, None) == -1        # bias without weight
    assert rn(p, p, None, None, 4, 250, 256, 256, 1e-6, 1, None) == -1     # C % 8
    assert rn(p, p, None, None, 4, 256, 200, 256, 1e-6, 1, None) == -1     # row stride < C
    assert rn(p, p, None, None, 4, 256, 256, 256, 1e-6, 7, None) == -1     # unknown mode


def test_import_fails_loudly_without_library(monkeypatch, tmp_path):
    import reworld_b200.build as b
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "lib_path", lambda: str(tmp_path / "missing.so"))
    with pytest.raises(ImportError):
        _native.lib()


def test_attn_workspace_plan():
    lib = _native.lib()
    # 704x1280 chunk over the 13-chunk cache: 264 query-pair units, a split tail
    n = lib.rw_attn_workspace_bytes(1, 2640, 34320, 24)
    assert n > 0 and n % (4 * (128 * 256 + 512)) == 0
    # short key ranges run whole: no workspace (text cross-attention, 512 keys)
    assert lib.rw_attn_workspace_bytes(1, 2640, 512, 24) == 0
    assert lib.rw_attn_workspace_bytes(0, 1, 1, 1) == 0


def test_ctypes_bindings_match_header_parameter_counts():
    """Every declaration in include/reworld_b200.h has as many parameters as the
    ctypes binding of the same name (a mismatch would shift every later argument)."""
    src = open(os.path.join(ROOT, "include", "reworld_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    decls = dict(re.findall(r"\b(rw_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", src))
    assert set(decls) == set(_native.exported_symbols())
    for name, params in decls.items():
        params = params.strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert n == len(_native._SIGNATURES[name][1]), (name, n, len(_native._SIGNATURES[name][1]))
