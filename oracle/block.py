"""Oracle of the DiT block's cross_attn_ffn (TEST INFRASTRUCTURE, see
oracle/__init__.py): wan_5b/modules/action_model.py:547-556 with norm3 / norm2
WanLayerNorm (wan_5b/modules/model.py:92-102), the text cross-attention of
MultiShotT2VCrossAttention (wan_5b/modules/causal_model.py:186-289, one context
chunk per video: WanCrossAttention, model.py:164-197) on the reference's CPU
attention path, and ffn Linear -> GELU(tanh) -> Linear (action_model.py:404-406).
torch on CPU; W holds the parameters by their module names."""
import torch
import torch.nn.functional as F

from .attention import reference_attention_cpu
from .self_attn import rms_norm


def layer_norm(x, w, b, eps):
    return F.layer_norm(x, (x.shape[-1],), w, b, eps).type_as(x)


def cross_attention(W, x, context, num_heads, eps=1e-6, prefix="cross_attn."):
    b, dim = x.shape[0], x.shape[-1]
    n, d = num_heads, dim // num_heads
    lin = lambda t, name: F.linear(t, W[prefix + name + ".weight"], W[prefix + name + ".bias"])
    q = rms_norm(lin(x, "q"), W[prefix + "norm_q.weight"], eps).view(b, -1, n, d)
    k = rms_norm(lin(context, "k"), W[prefix + "norm_k.weight"], eps).view(b, -1, n, d)
    v = lin(context, "v").view(b, -1, n, d)
    o = reference_attention_cpu(q, k, v)
    return lin(o.flatten(2), "o")


def cross_attn_ffn(W, x, context, e_mod, num_heads, frames, eps=1e-6):
    """Returns the stages (norm3, cross_attn, x1, norm2, ffn, out)."""
    fs = x.shape[1] // frames
    e = e_mod.chunk(6, dim=2)
    n3 = layer_norm(x, W["norm3.weight"], W["norm3.bias"], eps)
    ca = cross_attention(W, n3, context, num_heads, eps)
    x1 = x + ca
    n2 = layer_norm(x1, None, None, eps)
    h = (n2.unflatten(dim=1, sizes=(frames, fs)) * (1 + e[4]) + e[3]).flatten(1, 2)
    h = F.gelu(F.linear(h, W["ffn.0.weight"], W["ffn.0.bias"]), approximate="tanh")
    y = F.linear(h, W["ffn.2.weight"], W["ffn.2.bias"])
    out = x1 + (y.unflatten(dim=1, sizes=(frames, fs)) * e[5]).flatten(1, 2)
    return {"norm3": n3, "cross_attn": ca, "x1": x1, "norm2": n2, "ffn": y, "out": out}
