"""reworld_b200 — B200 (sm_100a) kernels for ReWorld's per-chunk causal self-attention.

The hot path of the Wan2.2-TI2V-5B streaming world model's cached chunk
attention, with the reference's plugin points as the API:
  attention / flash_attention   drop-in for wan_5b/modules/attention.py:133
  self_attn.install(model)      drop-in forward for CausalWanPropSelfAttention
  landmark.LandmarkCacheV2      drop-in for longctx/inference/landmark_cache_v2.py
  landmark.LandmarkBankStack    the same bank for all layers, one gather launch
  ulysses                       sequence-parallel (head-sharded) chunk attention
All compute runs in the package's CUDA library (reworld_b200/_lib); importing
the compute modules fails if it is missing.
"""
from . import _native

_native.lib()   # fail loudly at import when the CUDA library is absent

from .attention import attention, chunk_attention, flash_attention  # noqa: E402
from .kv_cache import qkv_norm_rope_store, rope_kv_store  # noqa: E402
from .rope import RopeArgs, build_freqs, device_table, rope_params  # noqa: E402

__all__ = ["attention", "flash_attention", "chunk_attention", "rope_kv_store", "qkv_norm_rope_store", "RopeArgs",
           "build_freqs", "rope_params", "device_table"]
