"""rw_gemm_bf16 (the tcgen05 GEMM behind the projections and the FFN) against an
fp32 reference of torch.nn.functional.linear on the same bf16 operands: the only
difference allowed is the final bf16 rounding (accumulation order moves a value
across a rounding boundary at most by one bf16 unit), at the workload's own
shapes (2640 tokens of the 704x1280 chunk) and at ragged small ones."""
import pytest
import torch

pytestmark = pytest.mark.gpu

# (M, N, K, epilogue): the q|k|v, value_proj (+ residual), o|prope_proj, FFN up (GELU)
# and FFN down shapes of one layer-chunk, then small and ragged cases
SHAPES = [
    (2640, 9216, 3072, "bias"), (2640, 3072, 3072, "residual"), (2640, 3072, 6144, "bias"),
    (2640, 14336, 3072, "gelu"), (2640, 3072, 14336, "bias"),
    (1, 128, 64, "none"), (7, 256, 64, "bias"), (300, 384, 192, "gelu"), (257, 640, 128, "residual"),
    (513, 128, 1024, "none"), (5000, 512, 256, "bias"), (660, 9216, 3072, "bias"),
    (3000, 2560, 448, "gelu"), (3000, 2560, 448, "residual"),
]


def _ref(x, w, b, epi, r):
    torch.backends.cuda.matmul.allow_tf32 = False
    y = x.float() @ w.float().T
    if b is not None:
        y = y + b.float()
    if epi == "gelu":
        y = torch.nn.functional.gelu(y, approximate="tanh")
    if epi == "residual":
        return (y.to(torch.bfloat16) + r).float(), y
    return y, y


def _ulp(v):
    """One bf16 unit at |v| (2^(e - 7) for v in [2^e, 2^(e+1)))."""
    a = v.abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


@pytest.mark.parametrize("M,N,K,epi", SHAPES)
def test_gemm_matches_fp32_reference(cuda, M, N, K, epi):
    from reworld_b200.gemm import linear
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    b = None if epi == "none" else (torch.randn(N, generator=g, device=cuda) * 0.5).to(torch.bfloat16)
    r = torch.randn(M, N, generator=g, device=cuda).to(torch.bfloat16) if epi == "residual" else None
    out = linear(x, w, b, gelu=epi == "gelu", residual=r)
    torch.cuda.synchronize()
    ref, lin = _ref(x, w, b, epi, r)
    o = out.float()
    assert torch.isfinite(o).all()
    # fp32 accumulation in another order: an absolute error far below the bf16 unit of
    # typical outputs, bounded by 2^-18 of sum |x w| (which matters only for results
    # near zero, where one bf16 unit is tiny)
    acc_err = 2.0 ** -18 * (x.float().abs() @ w.float().abs().T)
    if epi == "residual":
        # bf16(r + bf16(lin)): the inner rounding may differ by one unit of lin
        tol = _ulp(ref) + _ulp(lin) + acc_err
    else:
        tol = _ulp(ref) + acc_err
    bad = (o - ref).abs() > tol
    assert not bool(bad.any()), (int(bad.sum()), (o - ref).abs().max().item())
    if M >= 256 and epi != "gelu":
        # cuBLAS on the same operands: equal in the vast majority of elements (the GELU
        # form is not compared: torch rounds the Linear's output before the GELU, this
        # epilogue applies it to the fp32 accumulator)
        if epi == "residual":
            lib = r + torch.nn.functional.linear(x, w, b)
        else:
            lib = torch.nn.functional.linear(x, w, b)
        assert (out == lib).float().mean().item() > 0.9
    from reworld_b200 import _native
    _native.check_status(cuda)


def test_gemm_in_place_residual_on_strided_rows(cuda):
    """value_proj's residual written in place into the v columns of the stacked
    q|k|v projection rows (row stride 3C), as the self-attention drop-in does."""
    from reworld_b200.gemm import linear
    g = torch.Generator(device=cuda).manual_seed(5)
    M, C = 660, 3072
    qkv = torch.randn(M, 3 * C, generator=g, device=cuda).to(torch.bfloat16)
    vp = torch.randn(M, C, generator=g, device=cuda).to(torch.bfloat16)
    w = (torch.randn(C, C, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    b = (torch.randn(C, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    before = qkv.clone()
    v = qkv[:, 2 * C:]
    want = v + torch.nn.functional.linear(vp, w, b)
    linear(vp, w, b, residual=v, out=v)
    torch.cuda.synchronize()
    assert torch.equal(qkv[:, :2 * C], before[:, :2 * C])          # q and k columns untouched
    d = (qkv[:, 2 * C:].float() - want.float()).abs()
    acc_err = 2.0 ** -18 * (vp.float().abs() @ w.float().abs().T)
    assert (d <= _ulp(want.float()) * 2 + acc_err).all()
    assert (qkv[:, 2 * C:] == want).float().mean().item() > 0.9


def test_gemm_rejects_unsupported_shapes(cuda):
    from reworld_b200.gemm import linear
    x = torch.zeros(4, 96, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError):
        linear(x, torch.zeros(128, 96, dtype=torch.bfloat16, device=cuda))      # K not a multiple of 64
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError):
        linear(x, torch.zeros(100, 64, dtype=torch.bfloat16, device=cuda))      # N not a multiple of 128
    with pytest.raises(ValueError):
        linear(x.float(), torch.zeros(128, 64, device=cuda))


def _raw(lib, x, w, b, out, ws, epi=1):
    import ctypes
    from reworld_b200 import _native
    M, K = x.shape
    N = w.shape[0]
    st = _native.status_tensor(x.device)
    return lib.rw_gemm_bf16(ctypes.c_void_p(x.data_ptr()), K, ctypes.c_void_p(w.data_ptr()), K,
                            ctypes.c_void_p(b.data_ptr()), None, 0, ctypes.c_void_p(out.data_ptr()), N, M, N, K, epi,
                            ctypes.c_void_p(ws.data_ptr()) if ws is not None else None,
                            ws.numel() if ws is not None else 0, ctypes.c_void_p(st.data_ptr()),
                            _native.stream_ptr(x.device))


@pytest.mark.parametrize("M,N,K", [(2640, 3072, 3072), (2640, 9216, 3072), (3000, 2560, 448)])
def test_shared_last_round_matches_whole_tiles(cuda, M, N, K):
    """The last, partial round shared out among all CTA pairs by k-blocks (partial
    sums meeting in the workspace) against the same GEMM with every tile run whole
    (no workspace): equal up to fp32 summation order, on three calls in a row (the
    workspace's ready flags are reset by each call), flags zero afterwards."""
    from reworld_b200 import _native
    lib = _native.lib()
    need = lib.rw_gemm_workspace_bytes(M, N, K)
    assert need > 0                                   # these shapes leave a partial last round
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    for call in range(3):
        x = torch.randn(M, K, generator=g, device=cuda).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
        b = (torch.randn(N, generator=g, device=cuda) * 0.1).to(torch.bfloat16)
        whole = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
        shared = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda)
        assert _raw(lib, x, w, b, whole, None) == 0
        assert _raw(lib, x, w, b, shared, ws) == 0
        torch.cuda.synchronize()
        ref = x.float() @ w.float().T + b.float()
        acc_err = 2.0 ** -18 * (x.float().abs() @ w.float().abs().T)
        for out in (whole, shared):
            assert torch.isfinite(out.float()).all()
            assert bool(((out.float() - ref).abs() <= _ulp(ref) + acc_err).all()), call
        assert (whole == shared).float().mean().item() > 0.95
    flags = ws[-4096:].view(torch.int32)
    assert not flags.any()
    _native.check_status(cuda)
