"""B200-native (sm_100a) Llama inference hot path.

Drop-in for the per-layer hot path of Llama_Pure_Compute: the operator module
(``ops``: rope_forward, rmsswiglu_forward, update_kv_cache), the attention entry
point (``flash_attention.flash_attention_v2``), ``RMSNorm``, the KV-cache manager
and the model / generator call sites, all running hand-written CUDA kernels
for sm_100a through the C-ABI library ``lib/liblpc_b200.so``.
"""
from .config import PRESETS, LlamaModelConfig, Precision
from .ops import (decode_attention, is_cuda_backend_available, rmsnorm_forward, rmsswiglu_forward,
                  rope_forward, rope_kv_append, update_kv_cache)

__version__ = "0.1.0"

__all__ = [
    "LlamaModelConfig",
    "Precision",
    "PRESETS",
    "rope_forward",
    "rmsswiglu_forward",
    "update_kv_cache",
    "is_cuda_backend_available",
    "rmsnorm_forward",
    "rope_kv_append",
    "decode_attention",
]
