"""Drop-in forward for the reference's CausalWanPropSelfAttention (inference branch).

`prop_self_attn_forward(self, x, seq_lens, grid_sizes, freqs, block_mask,
kv_cache=None, current_start=0, cache_start=None, prope_context=None)` has the
signature and semantics of wan_5b/modules/action_model.py:148-319 with a KV
cache: q/k/v projections + RMSNorm over all heads, PM-RoPE phase and V-side
P^-1 residual when prope_context is given, the chunk's RoPE at its start frame
(or kv_cache["rope_start_frame"]), the cache write at
[local_end - num_new, local_end), attention over kv_cache[:, :local_end], the
index updates of :304-305 and the o projection (+ P residual).

What runs on the B200 kernels for a bf16 module: the q/k/v projections as one
rw_gemm_bf16 GEMM over the stacked weights, the RMSNorm of q and k, the RoPE of k
and the cache write of k/v (one rw_qkv_norm_rope_store launch), the PRoPE SE3
transforms (rw_se3_block_apply) with value_proj and its residual as one GEMM
written in place, the attention with q's RoPE applied inside the kernel
(rw_attn_fwd), and o(y) + prope_proj(P y) as one GEMM over [y | P y].  A module
in another dtype keeps torch's projections and norm, casts q/k/v to bf16 and uses
rw_rope_kv_store and the attention kernel.  The KV cache must be bf16.

Install it per block the way the reference installs its sequence-parallel
forward (wan_5b/text2video.py:150-154): `install(model)`.
"""
import math
import sys
import types
import weakref

import torch

from . import _native
from . import gemm
from ._native import c_vp
from .attention import chunk_attention
from .kv_cache import qkv_norm_rope_store, rope_kv_store
from .rope import RopeArgs, device_table


def _invert_se3(T):
    R = T[..., :3, :3]
    t = T[..., :3, 3:]
    Ri = R.transpose(-1, -2)
    out = T.clone()
    out[..., :3, :3] = Ri
    out[..., :3, 3:] = -Ri @ t
    out[..., 3, :3] = 0
    out[..., 3, 3] = 1
    return out


def _ref_flag(module_obj, name):
    """A module-level switch of the reference model module that defines the
    attention class (action_model.py:65-67: _PROPE_LOG_T, _SE3_T_BOUND, set by
    CausalWanActionModel's constructor, :604-608); False when absent."""
    mod = sys.modules.get(type(module_obj).__module__)
    return bool(getattr(mod, name, False))


def _bound_t(ctx):
    """Row-wise translation bound t / (1 + |t|) of action_model.py:97-102."""
    t = ctx[..., :3, 3]
    ctx = ctx.clone()
    ctx[..., :3, 3] = t / (1.0 + t.norm(dim=-1, keepdim=True))
    return ctx


def se3_mats(prope_context, mode, n_frames, dtype, t_bound=False):
    """The frames' 4x4 matrices as _se3_block_apply forms them (action_model.py:
    96-104): the last n_frames contexts cast to the activation dtype, the
    translation bounded first when the reference's _SE3_T_BOUND switch is on,
    inverted in that dtype for 'P_inv'; returned as fp32 [B, n_frames, 4, 4]
    (same values) for the kernel."""
    ctx = prope_context[:, -n_frames:].to(dtype)
    if t_bound:
        ctx = _bound_t(ctx)
    if mode == "P_inv":
        ctx = _invert_se3(ctx)
    return ctx.float().contiguous()


# The frames' matrices depend only on the camera context, not on the layer: every
# layer of a forward reuses the ones the first layer formed.  id(context) -> (weak
# reference, version counter, {(mode, frames, dtype, bound, device): matrices}).
_MATS_CACHE = {}


def _cached_mats(prope_context, mode, n_frames, dtype, t_bound, device):
    ver = _version(prope_context)
    key = (mode, n_frames, dtype, bool(t_bound), str(device))
    ent = _MATS_CACHE.get(id(prope_context))
    if ver is None or ent is None or ent[0]() is not prope_context or ent[1] != ver:
        if ver is None:
            return se3_mats(prope_context, mode, n_frames, dtype, t_bound).to(device)
        k = id(prope_context)
        ent = (weakref.ref(prope_context, lambda _r, k=k: _MATS_CACHE.pop(k, None)), ver, {})
        _MATS_CACHE[k] = ent
    mats = ent[2].get(key)
    if mats is None:
        mats = se3_mats(prope_context, mode, n_frames, dtype, t_bound).to(device)
        ent[2][key] = mats
    return mats


def se3_block_apply(x, prope_context, mode, frame_seqlen, out=None, t_bound=False):
    """Block-diagonal 4x4 transform over head_dim per frame (action_model.py:84-114)
    with one rw_se3_block_apply launch.  x: bf16 [B, L, H, 128] on the GPU (any
    strides with a contiguous head dim); returns `out` (default: a new contiguous
    [B, L, H, 128] tensor).  t_bound: the reference's _SE3_T_BOUND switch."""
    B, L, H, D = x.shape
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError("se3_block_apply runs on bf16 CUDA tensors")
    if L % frame_seqlen != 0:
        raise ValueError(f"{L} tokens are not whole frames of {frame_seqlen}")
    mats = _cached_mats(prope_context, mode, L // frame_seqlen, x.dtype, t_bound, x.device)
    if out is None:
        out = torch.empty((B, L, H, D), dtype=torch.bfloat16, device=x.device)
    lib = _native.lib()
    with torch.cuda.device(x.device):
        code = lib.rw_se3_block_apply(c_vp(x.data_ptr()), c_vp(out.data_ptr()), c_vp(mats.data_ptr()), B, L, H, D,
                                      int(frame_seqlen), *x.stride()[:3], *out.stride()[:3],
                                      _native.stream_ptr(x.device))
    _native.check(code, "rw_se3_block_apply")
    return out


def _stacked_qkv(self):
    """The q/k/v projections' weights [3C, C] (and biases [3C]) in one buffer, so
    that one GEMM computes all three.  The module's own parameters are re-pointed
    to views of that buffer the first time (the values are unchanged and no
    second copy is kept); if they are later replaced, the buffer is rebuilt."""
    lins = (self.q, self.k, self.v)
    W = getattr(self, "_rw_wqkv", None)
    C = lins[0].weight.shape[0]
    if W is None or any(m.weight.data_ptr() != W[i * C].data_ptr() for i, m in enumerate(lins)):
        W = torch.cat([m.weight.detach() for m in lins])
        for i, m in enumerate(lins):
            m.weight.data = W[i * C:(i + 1) * C]
        self._rw_wqkv = W
    if all(m.bias is not None for m in lins):
        bias = getattr(self, "_rw_bqkv", None)
        if bias is None or any(m.bias.data_ptr() != bias[i * C].data_ptr() for i, m in enumerate(lins)):
            bias = torch.cat([m.bias.detach() for m in lins])
            for i, m in enumerate(lins):
                m.bias.data = bias[i * C:(i + 1) * C]
            self._rw_bqkv = bias
    else:
        bias = torch.cat([m.bias.detach() if m.bias is not None else W.new_zeros(C) for m in lins])
    return W, bias


def _stacked_out(self):
    """[W_o | W_prope] as one [C, 2C] weight (the module's o / prope_proj weights
    re-pointed to its column blocks, values unchanged) and b_o + b_prope, so that
    o(y) + prope_proj(P y) is one GEMM over [y | P y]."""
    W = getattr(self, "_rw_wout", None)
    C = self.o.weight.shape[0]
    if W is None or self.o.weight.data_ptr() != W.data_ptr() or \
            self.prope_proj.weight.data_ptr() != W[:, C:].data_ptr():
        W = torch.cat([self.o.weight.detach(), self.prope_proj.weight.detach()], dim=1)
        self.o.weight.data = W[:, :C]
        self.prope_proj.weight.data = W[:, C:]
        self._rw_wout = W
    bo, bp = self.o.bias, self.prope_proj.bias
    if bo is None and bp is None:
        return W, None
    # b_o + b_prope, formed again only when either bias tensor changed (in place or replaced)
    key = tuple((t.data_ptr(), _version(t)) if t is not None else None for t in (bo, bp))
    cached = getattr(self, "_rw_bout", None)
    if cached is None or cached[0] != key or None in (k[1] for k in key if k is not None):
        bias = (bo.detach() if bo is not None else 0) + (bp.detach() if bp is not None else 0)
        self._rw_bout = (key, bias)
        return W, bias
    return W, cached[1]


# Host mirrors of the kv_cache index tensors this module wrote last:
# id(tensor) -> (weak reference, version counter after the write, value).  A
# tensor's version counter advances with every in-place write, so a mirror is
# used only while nobody else (e.g. the pipeline's local_end_index.fill_ after
# the landmark assembly) has written the tensor since; otherwise the value is
# read from the device.  This saves two device synchronisations per layer.
_INDEX_MIRROR = {}


def _version(t):
    try:
        return t._version
    except RuntimeError:      # inference-mode tensors keep no version counter
        return None


def read_index(t):
    """int(t.item()) for a one-element index tensor, from the host mirror when
    this module wrote the tensor last."""
    ent = _INDEX_MIRROR.get(id(t))
    ver = _version(t)
    if ent is not None and ver is not None and ent[0]() is t and ent[1] == ver:
        return ent[2]
    return int(t.item())


def write_index(t, value):
    """t.fill_(value), remembering the value on the host."""
    t.fill_(value)
    ver = _version(t)
    if ver is None:
        return
    key = id(t)
    _INDEX_MIRROR[key] = (weakref.ref(t, lambda _r, k=key: _INDEX_MIRROR.pop(k, None)), ver, int(value))


def _fused_path(self, x):
    return x.dtype == torch.bfloat16 and all(
        t.dtype == torch.bfloat16 for t in (self.q.weight, self.k.weight, self.v.weight, self.norm_q.weight,
                                            self.norm_k.weight))


def _se3_torch(x, prope_context, mode, frame_seqlen, t_bound=False):
    """The transform with torch ops, for modules outside the bf16 kernels' domain."""
    B, L, H, D = x.shape
    nf = L // frame_seqlen
    ctx = prope_context[:, -nf:].to(x.dtype)
    if t_bound:
        ctx = _bound_t(ctx)
    if mode == "P_inv":
        ctx = _invert_se3(ctx)
    xv = x.permute(0, 2, 1, 3).reshape(B, H, nf, frame_seqlen, D // 4, 4)
    y = torch.matmul(ctx[:, None, :, None, None], xv.unsqueeze(-1)).squeeze(-1)
    return y.reshape(B, H, L, D).permute(0, 2, 1, 3)


def _cache_local_size(local_attn_size):
    if isinstance(local_attn_size, (list, tuple)):
        finite = [abs(sz) for sz in local_attn_size if sz != -1]
        return max(finite) if finite else -1
    return abs(local_attn_size) if local_attn_size != -1 else -1


def prop_self_attn_forward(self, x, seq_lens, grid_sizes, freqs, block_mask, kv_cache=None, current_start=0,
                           cache_start=None, prope_context=None):
    if kv_cache is None:
        # training / teacher-forcing branch: not part of the cached chunk path
        return self._rw_reference_forward(x, seq_lens, grid_sizes, freqs, block_mask, kv_cache=kv_cache,
                                          current_start=current_start, cache_start=cache_start,
                                          prope_context=prope_context)
    if kv_cache["k"].dtype != torch.bfloat16:
        raise NotImplementedError("the B200 chunk-attention path keeps the KV cache in bf16")
    b, s, n, d = *x.shape[:2], self.num_heads, self.head_dim
    fused = _fused_path(self, x)
    if fused:
        C = n * d
        qkv = gemm.linear(x, *_stacked_qkv(self))                       # [b, s, 3C]
        q_rows, k_rows, v_rows = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
        v = v_rows.view(b, s, n, d)
    else:
        q = self.norm_q(self.q(x)).view(b, s, n, d)
        k = self.norm_k(self.k(x)).view(b, s, n, d)
        v = self.v(x).view(b, s, n, d)
    g0 = [int(t) for t in grid_sizes[0].tolist()]
    frame_seqlen = g0[1] * g0[2]

    delta = None
    t_bound = _ref_flag(self, "_SE3_T_BOUND")
    if prope_context is not None:
        R_flat = prope_context[..., :3, :3].flatten(-2)
        t_vec = prope_context[..., :3, 3]
        if _ref_flag(self, "_PROPE_LOG_T"):
            t_vec = torch.sign(t_vec) * torch.log1p(t_vec.abs())
        c_all = torch.cat([R_flat, t_vec], dim=-1)
        T_half = s // frame_seqlen
        delta = self.pose_mlp(c_all[:, -T_half:])                  # [B, T, d/2] per-frame phase
        if fused:
            # v + value_proj(P^-1 v): one GEMM whose epilogue adds the residual (two
            # roundings, as the reference's bf16 add) in place into the v columns
            v_p = se3_block_apply(v, prope_context, "P_inv", frame_seqlen, t_bound=t_bound)
            gemm.module_linear(self.value_proj, v_p.flatten(2), residual=v_rows, out=v_rows)
        else:
            v_p = _se3_torch(v, prope_context, "P_inv", frame_seqlen, t_bound)
            v = (v.flatten(2) + self.value_proj(v_p.flatten(2))).view(b, s, n, d)

    num_new = s
    cur_end = current_start + num_new
    sink_tokens = self.sink_size * frame_seqlen
    cache_local = _cache_local_size(self.local_attn_size)
    self.max_attention_size = None if cache_local == -1 else int(cache_local) * int(frame_seqlen)
    kv_cache_size = kv_cache["k"].shape[1]
    g_start_f = current_start // frame_seqlen
    rsf = kv_cache.get("rope_start_frame") if isinstance(kv_cache, dict) else None
    if rsf is not None:
        g_start_f = read_index(rsf)
    grid = (max(1, num_new // frame_seqlen), g0[1], g0[2])

    global_end = read_index(kv_cache["global_end_index"])
    local_end_prev = read_index(kv_cache["local_end_index"])
    if cache_local != -1 and cur_end > global_end and num_new + local_end_prev > kv_cache_size:
        n_evict = num_new + local_end_prev - kv_cache_size
        n_roll = local_end_prev - n_evict - sink_tokens
        for key in ("k", "v"):
            kv_cache[key][:, sink_tokens:sink_tokens + n_roll] = \
                kv_cache[key][:, sink_tokens + n_evict:sink_tokens + n_evict + n_roll].clone()
        local_end = local_end_prev + cur_end - global_end - n_evict
    else:
        local_end = local_end_prev + cur_end - global_end
    local_start = local_end - num_new

    table = device_table(freqs, x.device)
    rope = RopeArgs(table, grid, g_start_f, head_dim=d, delta=delta)
    if fused:
        q = qkv_norm_rope_store(q_rows, k_rows, v_rows, self.norm_q.weight, self.norm_k.weight, kv_cache["k"],
                                kv_cache["v"], local_start, self.norm_q.eps, self.norm_k.eps, rope=rope)
    else:
        rope_kv_store(k, v, kv_cache["k"], kv_cache["v"], local_start, rope=rope)
    if self.max_attention_size is None:
        k_slice = kv_cache["k"][:, :local_end]
        v_slice = kv_cache["v"][:, :local_end]
    else:
        s0 = max(0, local_end - self.max_attention_size)
        k_slice = kv_cache["k"][:, s0:local_end]
        v_slice = kv_cache["v"][:, s0:local_end]
    if fused and prope_context is not None:
        # [y | P y] in one buffer, both halves written by the attention (P y from its bf16
        # output values, as _se3_block_apply forms it); one GEMM does o(y) + prope_proj(P y)
        # (action_model.py:307-318)
        C = n * d
        yy = torch.empty((b, s, 2 * C), dtype=torch.bfloat16, device=x.device)
        y = yy[..., :C].view(b, s, n, d)
        mats = _cached_mats(prope_context, "P", s // frame_seqlen, torch.bfloat16, t_bound, x.device)
        chunk_attention(q, k_slice, v_slice, rope=rope, out=y,
                        se3=(mats, frame_seqlen, yy[..., C:].view(b, s, n, d)))
        write_index(kv_cache["global_end_index"], cur_end)
        write_index(kv_cache["local_end_index"], local_end)
        return gemm.linear(yy, *_stacked_out(self))
    attn_out = chunk_attention(q, k_slice, v_slice, rope=rope).to(x.dtype)
    write_index(kv_cache["global_end_index"], cur_end)
    write_index(kv_cache["local_end_index"], local_end)

    if fused:
        return gemm.module_linear(self.o, attn_out.flatten(2))
    out = self.o(attn_out.flatten(2))
    if prope_context is not None:
        x_p = _se3_torch(attn_out, prope_context, "P", frame_seqlen, t_bound)
        out = out + self.prope_proj(x_p.flatten(2))
    return out


def install(model):
    """Replaces block.self_attn.forward of every block of a CausalWanActionModel
    (or any module with .blocks[i].self_attn) by prop_self_attn_forward."""
    blocks = model.blocks if hasattr(model, "blocks") else model
    n = 0
    for blk in blocks:
        sa = blk.self_attn
        if not hasattr(sa, "_rw_reference_forward"):
            sa._rw_reference_forward = sa.forward
        sa.forward = types.MethodType(prop_self_attn_forward, sa)
        n += 1
    return n


def patch_attention_symbol(module):
    """Rebinds `module.attention` (e.g. wan_5b.modules.action_model) to this
    package's attention(), the way the reference's compressed pipeline patches
    it (pipeline/causal_diffusion_inference_compressed.py:168-214)."""
    from .attention import attention
    prev = getattr(module, "attention", None)
    module.attention = attention
    return prev
