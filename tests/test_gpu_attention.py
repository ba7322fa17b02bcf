"""Chunk-attention kernel (rw_attn_fwd) against the oracle and the reference's outputs.

Tolerance (bf16 output, fp32 accumulation): max-abs 2e-2 and mean-abs 2e-3 against
the reference's own attention on the same inputs."""
import math

import numpy as np
import pytest
import torch

import inputs as gi
from oracle import attention as oatt
from oracle import rope as orope
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _check(out, ref):
    err = (out.float().cpu().numpy() - np.asarray(ref, dtype=np.float64))
    a = np.abs(err)
    assert np.isfinite(out.float().cpu().numpy()).all()
    assert a.max() < MAX_ABS and a.mean() < MEAN_ABS, (a.max(), a.mean())


def _status_clean():
    from reworld_b200 import _native
    _native.check_status()


@pytest.mark.parametrize("i", range(len(gi.ATTN_CASES)))
def test_attention_matches_reference_fixture(cuda, golden, i):
    from reworld_b200 import attention
    q, k, v = gi.attention_case(i)
    ref = bf16_bits_to_f32(golden["attention"][f"c{i}_o"]).reshape(q.shape)
    out = attention(q.to(cuda), k.to(cuda), v.to(cuda))
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == q.shape
    _check(out, ref)
    _status_clean()


SHAPES = [  # B, Lq, Lk, H : tails of both tile sizes, one key, one query, pair tails
    (1, 1, 1, 1), (1, 5, 3, 2), (1, 128, 128, 1), (1, 129, 127, 1), (1, 255, 257, 2), (1, 256, 256, 1),
    (2, 300, 1000, 2), (3, 77, 513, 3), (1, 660, 2640, 4),
]


@pytest.mark.parametrize("B,Lq,Lk,H", SHAPES)
def test_attention_shapes_vs_oracle(cuda, B, Lq, Lk, H):
    from reworld_b200 import chunk_attention
    g = torch.Generator().manual_seed(B * 1000 + Lq + Lk + H)
    q = torch.randn(B, Lq, H, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Lk, H, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Lk, H, 128, generator=g).to(torch.bfloat16)
    ref = oatt.attention_f64(q.float().numpy(), k.float().numpy(), v.float().numpy())
    out = chunk_attention(q.to(cuda), k.to(cuda), v.to(cuda))
    torch.cuda.synchronize()
    _check(out, ref)
    _status_clean()


def test_attention_large_scores_rescale_path(cuda):
    """Scores with a large dynamic range exercise the in-place O rescale."""
    from reworld_b200 import chunk_attention
    g = torch.Generator().manual_seed(5)
    B, Lq, Lk, H = 1, 256, 1024, 2
    q = (torch.randn(B, Lq, H, 128, generator=g) * 3).to(torch.bfloat16)
    k = (torch.randn(B, Lk, H, 128, generator=g) * 3).to(torch.bfloat16)
    k[:, 900:] *= 2.0   # late keys raise the running maximum well past the rescale threshold
    v = torch.randn(B, Lk, H, 128, generator=g).to(torch.bfloat16)
    ref = oatt.attention_f64(q.float().numpy(), k.float().numpy(), v.float().numpy())
    out = chunk_attention(q.to(cuda), k.to(cuda), v.to(cuda))
    torch.cuda.synchronize()
    _check(out, ref)


def test_attention_on_cache_view_with_strides(cuda):
    """k/v as kv_cache[:, :local_end] views of a larger [B, cap, H, D] cache, B=2."""
    from reworld_b200 import chunk_attention
    g = torch.Generator().manual_seed(9)
    B, Lq, H, cap, le = 2, 200, 3, 1500, 1111
    cache_k = torch.randn(B, cap, H, 128, generator=g).to(torch.bfloat16)
    cache_v = torch.randn(B, cap, H, 128, generator=g).to(torch.bfloat16)
    q = torch.randn(B, Lq, H, 128, generator=g).to(torch.bfloat16)
    ref = oatt.attention_f64(q.float().numpy(), cache_k[:, :le].float().numpy(), cache_v[:, :le].float().numpy())
    ck, cv = cache_k.to(cuda), cache_v.to(cuda)
    out = chunk_attention(q.to(cuda), ck[:, :le], cv[:, :le])
    torch.cuda.synchronize()
    _check(out, ref)


def test_attention_in_kernel_rope_matches_oracle(cuda):
    """q given un-roped; the kernel applies the 3-D RoPE (+ PM-RoPE phase) itself."""
    from reworld_b200 import RopeArgs, chunk_attention, device_table
    g = torch.Generator().manual_seed(21)
    f, h, w, H = 3, 11, 20, 2
    Lq = f * h * w
    Lk = 4 * Lq
    q = torch.randn(1, Lq, H, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, Lk, H, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, Lk, H, 128, generator=g).to(torch.bfloat16)
    delta = torch.randn(1, f, 64, generator=g) * 0.3
    freqs = orope.build_freqs(128, 12 / 22, 20 / 40)
    for d_ in (None, delta):
        qr = orope.causal_rope_apply(q.float().numpy(), [(f, h, w)], freqs, start_frame=9)
        if d_ is not None:
            dtok = d_.unsqueeze(2).expand(-1, -1, h * w, -1).reshape(1, Lq, 1, 64).numpy()
            qr = orope.pm_rope_delta_apply(qr, dtok)
        ref = oatt.attention_f64(qr, k.float().numpy(), v.float().numpy())
        rope = RopeArgs(device_table(freqs, cuda), (f, h, w), 9, delta=d_.to(cuda) if d_ is not None else None)
        out = chunk_attention(q.to(cuda), k.to(cuda), v.to(cuda), rope=rope)
        torch.cuda.synchronize()
        _check(out, ref)
    _status_clean()


def test_attention_drop_in_signature(cuda):
    from reworld_b200 import attention
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 64, 2, 128, generator=g)
    k = torch.randn(2, 300, 2, 128, generator=g)
    v = torch.randn(2, 300, 2, 128, generator=g)
    # fp32 inputs: computed in bf16, returned in q's dtype (flash-attention branch semantics)
    out = attention(q.to(cuda), k.to(cuda), v.to(cuda))
    assert out.dtype == torch.float32
    qb, kb, vb = q.bfloat16().float(), k.bfloat16().float(), v.bfloat16().float()
    _check(out, oatt.attention_f64(qb.numpy(), kb.numpy(), vb.numpy()))
    # k_lens restricts keys per batch element
    out2 = attention(q.to(cuda).bfloat16(), k.to(cuda).bfloat16(), v.to(cuda).bfloat16(), k_lens=[300, 123])
    ref1 = oatt.attention_f64(qb[1:].numpy(), kb[1:, :123].numpy(), vb[1:, :123].numpy())
    _check(out2[1:], ref1)
    # softmax_scale and q_scale
    out3 = attention(q.to(cuda).bfloat16(), k.to(cuda).bfloat16(), v.to(cuda).bfloat16(), softmax_scale=0.05)
    _check(out3, oatt.attention_f64(qb.numpy(), kb.numpy(), vb.numpy(), softmax_scale=0.05))
    with pytest.raises(NotImplementedError):
        attention(q.to(cuda), k.to(cuda), v.to(cuda), causal=True)
    with pytest.raises(NotImplementedError):
        attention(q.to(cuda), k.to(cuda), v.to(cuda), dropout_p=0.1)
    with pytest.raises(ValueError):
        from reworld_b200 import chunk_attention
        chunk_attention(q, k, v)   # CPU tensors: no CPU fallback


def test_attention_full_size_heads_vs_fp32_reference(cuda):
    """704x1280 chunk (Lq 2640) over the 13-chunk cache (Lk 34320), 24 heads; a torch
    fp32 reference on the GPU checks 3 heads, and every head is checked for
    finiteness and for the size-independent property that rows are convex
    combinations of V (|o| <= max |v| per dim)."""
    from reworld_b200 import chunk_attention
    g = torch.Generator(device=cuda).manual_seed(1)
    Lq, Lk, H = 2640, 34320, 24
    q = torch.randn(1, Lq, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(1, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(1, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    out = chunk_attention(q, k, v)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    vmax = v.float().abs().amax(dim=1, keepdim=True)
    assert (out.float().abs() <= vmax + 1e-2).all()
    for h in (0, 11, 23):
        qh, kh, vh = q[0, :, h].float(), k[0, :, h].float(), v[0, :, h].float()
        ref = torch.softmax((qh @ kh.T) / math.sqrt(128), dim=-1) @ vh
        err = (out[0, :, h].float() - ref).abs()
        assert err.max().item() < MAX_ABS and err.mean().item() < MEAN_ABS
    _status_clean()


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 2640, 34320, 24), (1, 2640, 34320, 6), (1, 2640, 34320, 3),
                                         (1, 660, 5600, 40), (2, 300, 6000, 2)])
def test_attention_key_split_matches_unsplit(cuda, B, Lq, Lk, H):
    """Pairs sharing units (workspace given: equal shares of the key tiles, partial
    results merged) and one whole unit per pair (no workspace) compute the same
    attention; 3 and 6 heads are the per-rank shapes at 8 and 4 GPUs."""
    import ctypes
    from reworld_b200 import _native, chunk_attention
    g = torch.Generator(device=cuda).manual_seed(Lq + Lk)
    q = torch.randn(B, Lq, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    lib = _native.lib()
    assert lib.rw_attn_workspace_bytes(B, Lq, Lk, H) > 0      # these shapes do split
    split = chunk_attention(q, k, v)
    whole = torch.empty_like(q)
    st = _native.status_tensor(cuda)
    code = lib.rw_attn_fwd(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                           ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(whole.data_ptr()), B, Lq, Lk, H, 128,
                           *q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *whole.stride()[:3],
                           1.0 / math.sqrt(128), None, None, 0, ctypes.c_void_p(st.data_ptr()),
                           _native.stream_ptr(cuda))
    assert code == 0
    torch.cuda.synchronize()
    err = (split.float() - whole.float()).abs()
    assert err.max().item() < 1e-2 and err.mean().item() < 1e-4
    _status_clean()


def test_text_cross_attention_shape(cuda):
    """The DiT block's text cross-attention (wan_5b/modules/model.py:164-197 and the
    multi-shot form, causal_model.py:186-289): the chunk's 2640 queries over the
    cached 512 text keys, context_lens restricting the keys per batch element
    (flash_attention(q, k, v, k_lens=context_lens)), against an fp32 reference."""
    from reworld_b200 import attention
    g = torch.Generator(device=cuda).manual_seed(21)
    B, Lq, Lk, H = 2, 2640, 512, 24
    q = torch.randn(B, Lq, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    # ragged lengths (one launch per element), then one length for the batch (one launch)
    for lens in (torch.tensor([512, 77], device=cuda), torch.tensor([300, 300], device=cuda)):
        out = attention(q, k, v, k_lens=lens)
        torch.cuda.synchronize()
        for b, h in ((0, 0), (0, 17), (1, 5), (1, 23)):
            n = int(lens[b])
            qh, kh, vh = q[b, :, h].float(), k[b, :n, h].float(), v[b, :n, h].float()
            ref = torch.softmax((qh @ kh.T) / math.sqrt(128), dim=-1) @ vh
            err = (out[b, :, h].float() - ref).abs()
            assert err.max().item() < MAX_ABS and err.mean().item() < MEAN_ABS, (b, h, lens.tolist())
    _status_clean()
