"""Model configuration (shapes, eps, RoPE theta) for the Llama hot path.

Same fields, defaults, HF key mapping and presets as the reference's
``LlamaModelConfig`` (src/llama_pure_compute/config.py:27-179); only what the
hot path reads is kept (no C++ header generator).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from enum import Enum
from pathlib import Path
from typing import Any, Dict, Optional, Union


class Precision(str, Enum):
    FP32 = "fp32"
    FP16 = "fp16"
    BF16 = "bf16"
    INT8 = "int8"
    INT4 = "int4"

    def byte_size(self) -> float:
        return {"fp32": 4.0, "fp16": 2.0, "bf16": 2.0, "int8": 1.0, "int4": 0.5}[self.value]


@dataclass
class LlamaModelConfig:
    vocab_size: int = 32000
    dim: int = 4096
    inter_dim: int = 11008
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: Optional[int] = None
    head_dim: int = field(init=False)
    max_seq_len: int = 4096
    max_batch_size: int = 1
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    precision: Precision = Precision.FP16
    aligned_byte_boundary: int = 64

    def __post_init__(self) -> None:
        if self.num_kv_heads is None:
            self.num_kv_heads = self.num_heads
        if self.dim % self.num_heads != 0:
            raise ValueError(f"Dim ({self.dim}) must be divisible by num_heads ({self.num_heads})")
        self.head_dim = self.dim // self.num_heads
        if self.num_heads % self.num_kv_heads != 0:
            raise ValueError(
                f"num_heads ({self.num_heads}) must be multiple of num_kv_heads ({self.num_kv_heads})")
        if self.max_seq_len <= 0 or self.max_batch_size <= 0:
            raise ValueError("Sequence lengths and batch sizes must be strictly positive")

    @property
    def gqa_group_size(self) -> int:
        return self.num_heads // self.num_kv_heads

    @property
    def kv_cache_elements_per_token(self) -> int:
        return 2 * self.num_kv_heads * self.head_dim

    def estimate_kv_cache_memory_bytes(self) -> int:
        n = self.num_layers * self.max_batch_size * self.max_seq_len * self.kv_cache_elements_per_token
        return int(n * self.precision.byte_size())

    def num_parameters(self) -> int:
        D, I, H, Hkv, hd = self.dim, self.inter_dim, self.num_heads, self.num_kv_heads, self.head_dim
        per_layer = D * (H + 2 * Hkv) * hd + H * hd * D + 3 * D * I + 2 * D
        return self.num_layers * per_layer + 2 * self.vocab_size * D + D

    @classmethod
    def from_dict(cls, data: Dict[str, Any]) -> "LlamaModelConfig":
        valid = {f.name for f in cls.__dataclass_fields__.values() if f.init}
        kw = {k: v for k, v in data.items() if k in valid}
        if isinstance(kw.get("precision"), str):
            kw["precision"] = Precision(kw["precision"].lower())
        return cls(**kw)

    @classmethod
    def from_json(cls, json_path: Union[str, Path]) -> "LlamaModelConfig":
        path = Path(json_path)
        if not path.is_file():
            raise FileNotFoundError(f"Config file not found at: {path}")
        data = json.loads(path.read_text(encoding="utf-8"))
        mapping = {
            "hidden_size": "dim",
            "intermediate_size": "inter_dim",
            "num_hidden_layers": "num_layers",
            "num_attention_heads": "num_heads",
            "num_key_value_heads": "num_kv_heads",
        }
        return cls.from_dict({mapping.get(k, k): v for k, v in data.items()})


PRESETS: Dict[str, LlamaModelConfig] = {
    "llama-2-7b": LlamaModelConfig(vocab_size=32000, dim=4096, inter_dim=11008, num_layers=32,
                                   num_heads=32, num_kv_heads=32),
    "llama-3-8b": LlamaModelConfig(vocab_size=128256, dim=4096, inter_dim=14336, num_layers=32,
                                   num_heads=32, num_kv_heads=8, rope_theta=500000.0),
    "llama-2-70b": LlamaModelConfig(vocab_size=32000, dim=8192, inter_dim=28672, num_layers=80,
                                    num_heads=64, num_kv_heads=8),
}
