"""Per-layer static KV cache with ragged per-sequence lengths.

API of the reference ``KVCacheManager`` (src/llama_pure_compute/kv_manager.py:25-348):
same constructor arguments and validation, ``begin_request``/``reset``,
``update(layer_idx=, key_states=, value_states=, start_pos=)`` returning the
``[:B, :, :end, :]`` views, ``get`` and ``current_seq_len``.

B200 additions (same cache layout ``[max_batch, kv_heads, max_seq_len, head_dim]``
per layer, allocated once in HBM):
  * ``append_qkv`` -- the fused RoPE + append from the QKV projection output,
    at arbitrary per-sequence positions (ragged batches);
  * ``set_seq_lens`` -- per-sequence context lengths kept on the device
    (``seq_lens`` int32 [max_batch]), consumed by the ragged decode kernel
    without a host sync;
  * ``prepare_forward`` / ``attend`` -- the step interface the model calls
    (shared with ``ragged_cache.RaggedKVCache``).
"""
from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Optional, Tuple, Union

import torch

from .flash_attention import flash_attention_v2
from .ops import (decode_attention, decode_attention_workspace, qkv_rope_append, rope_kv_append,
                  update_kv_cache)

logger = logging.getLogger("llama_pure_compute_b200.kv_manager")

__all__ = ["KVCacheSpec", "KVCacheManager"]


@dataclass(frozen=True)
class KVCacheSpec:
    num_layers: int
    max_batch_size: int
    max_seq_len: int
    num_kv_heads: int
    head_dim: int
    dtype: torch.dtype
    device: torch.device


class KVCacheManager:
    def __init__(
        self,
        *,
        num_layers: int,
        max_batch_size: int,
        max_seq_len: int,
        n_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype = torch.float16,
        device: Union[str, torch.device] = "cuda",
    ) -> None:
        if num_layers <= 0:
            raise ValueError("num_layers must be positive")
        if max_batch_size <= 0:
            raise ValueError("max_batch_size must be positive")
        if max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if n_kv_heads <= 0 or head_dim <= 0:
            raise ValueError("n_kv_heads and head_dim must be positive")
        self.spec = KVCacheSpec(num_layers, max_batch_size, max_seq_len, n_kv_heads, head_dim,
                                dtype, torch.device(device))
        if self.spec.device.type != "cuda":
            raise RuntimeError("KVCacheManager lives in GPU memory: a CUDA device is required.")
        if not torch.cuda.is_available():
            raise RuntimeError("KVCacheManager requested CUDA but CUDA is unavailable.")
        self.device = self.spec.device
        shape = (max_batch_size, n_kv_heads, max_seq_len, head_dim)
        self.k_cache: list[torch.Tensor] = [torch.empty(shape, dtype=dtype, device=self.device)
                                            for _ in range(num_layers)]
        self.v_cache: list[torch.Tensor] = [torch.empty(shape, dtype=dtype, device=self.device)
                                            for _ in range(num_layers)]
        self.seq_lens = torch.zeros(max_batch_size, dtype=torch.int32, device=self.device)
        self.active_batch_size = 0
        logger.info("Allocated KV cache: layers=%d batch=%d seq=%d kv_heads=%d head_dim=%d "
                    "memory=%.2f GiB", num_layers, max_batch_size, max_seq_len, n_kv_heads,
                    head_dim, self.memory_footprint_bytes() / 2**30)

    # -- properties (kv_manager.py:135-157) ---------------------------------
    @property
    def max_batch_size(self) -> int:
        return self.spec.max_batch_size

    @property
    def max_seq_len(self) -> int:
        return self.spec.max_seq_len

    @property
    def num_layers(self) -> int:
        return self.spec.num_layers

    @property
    def n_kv_heads(self) -> int:
        return self.spec.num_kv_heads

    @property
    def head_dim(self) -> int:
        return self.spec.head_dim

    @property
    def dtype(self) -> torch.dtype:
        return self.spec.dtype

    def memory_footprint_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k_cache + self.v_cache)

    # -- request lifecycle (kv_manager.py:170-204) --------------------------
    def begin_request(self, batch_size: int) -> None:
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if batch_size > self.max_batch_size:
            raise ValueError(f"batch_size={batch_size} exceeds max_batch_size={self.max_batch_size}")
        self.active_batch_size = batch_size
        self.seq_lens[:batch_size].zero_()

    def reset(self) -> None:
        if self.active_batch_size:
            self.seq_lens[: self.active_batch_size].zero_()
        self.active_batch_size = 0

    def current_seq_len(self, batch_idx: int = 0) -> int:
        if batch_idx < 0 or batch_idx >= self.max_batch_size:
            raise IndexError("invalid batch index")
        return int(self.seq_lens[batch_idx].item())

    def _check_layer(self, layer_idx: int) -> None:
        if not 0 <= layer_idx < self.num_layers:
            raise IndexError(f"layer_idx={layer_idx} outside [0, {self.num_layers})")

    # -- reference update (kv_manager.py:206-317) ---------------------------
    @torch.no_grad()
    def update(
        self,
        *,
        layer_idx: int,
        key_states: torch.Tensor,
        value_states: torch.Tensor,
        start_pos: int,
    ) -> Tuple[torch.Tensor, torch.Tensor]:
        """Write [B, KV_HEADS, SEQ, D] states at positions [start_pos, start_pos+SEQ)
        of rows 0..B-1 and return the ``[:B, :, :end, :]`` cache views."""
        self._check_layer(layer_idx)
        if key_states.ndim != 4 or value_states.ndim != 4:
            raise ValueError("key_states and value_states must be [B, H, S, D]")
        if key_states.shape != value_states.shape:
            raise ValueError("K/V shapes must match")
        batch_size, kv_heads, seq_len, head_dim = key_states.shape
        if kv_heads != self.n_kv_heads:
            raise ValueError(f"expected {self.n_kv_heads} KV heads, got {kv_heads}")
        if head_dim != self.head_dim:
            raise ValueError(f"expected head_dim={self.head_dim}, got {head_dim}")
        if batch_size > self.max_batch_size:
            raise ValueError("batch size exceeds cache capacity")
        if start_pos < 0:
            raise ValueError("start_pos must be non-negative")
        end_pos = start_pos + seq_len
        if end_pos > self.max_seq_len:
            raise ValueError(f"KV cache overflow: end_pos={end_pos}, max_seq_len={self.max_seq_len}")
        k_src = key_states.permute(0, 2, 1, 3).contiguous().view(-1, self.n_kv_heads, self.head_dim)
        v_src = value_states.permute(0, 2, 1, 3).contiguous().view(-1, self.n_kv_heads, self.head_dim)
        dev = key_states.device
        slot_mapping = (torch.arange(batch_size, device=dev, dtype=torch.int64).unsqueeze(1)
                        * self.max_seq_len
                        + torch.arange(start_pos, end_pos, device=dev, dtype=torch.int64).unsqueeze(0)
                        ).reshape(-1)
        update_kv_cache(k_src, v_src, self.k_cache[layer_idx], self.v_cache[layer_idx], slot_mapping)
        self.seq_lens[:batch_size] = end_pos
        return (self.k_cache[layer_idx][:batch_size, :, :end_pos, :],
                self.v_cache[layer_idx][:batch_size, :, :end_pos, :])

    def get(self, *, layer_idx: int, batch_size: int, seq_len: int) -> Tuple[torch.Tensor, torch.Tensor]:
        if not 0 <= layer_idx < self.num_layers:
            raise IndexError("invalid layer index")
        if batch_size > self.max_batch_size:
            raise ValueError("batch size exceeds cache capacity")
        if seq_len > self.max_seq_len:
            raise ValueError("sequence length exceeds cache capacity")
        return (self.k_cache[layer_idx][:batch_size, :, :seq_len, :],
                self.v_cache[layer_idx][:batch_size, :, :seq_len, :])

    # -- ragged additions ---------------------------------------------------
    @torch.no_grad()
    def append_qkv(
        self,
        *,
        layer_idx: int,
        qkv: torch.Tensor,
        positions: torch.Tensor,
        cos_table: torch.Tensor,
        sin_table: torch.Tensor,
        num_heads: int,
    ) -> torch.Tensor:
        """RoPE + append for ``qkv`` [B, S, (H+2Hkv)*D] at per-token ``positions``
        [B, S] (row b of the batch is cache row b); returns rotated q [B, H, S, D].
        Does not touch ``seq_lens`` (see ``set_seq_lens``)."""
        self._check_layer(layer_idx)
        if qkv.shape[0] > self.max_batch_size:
            raise ValueError("batch size exceeds cache capacity")
        return rope_kv_append(qkv, positions, cos_table, sin_table, self.k_cache[layer_idx],
                              self.v_cache[layer_idx], num_heads, self.n_kv_heads)

    @torch.no_grad()
    def set_seq_lens(self, positions: torch.Tensor) -> torch.Tensor:
        """seq_lens[b] = positions[b, -1] + 1 (device op, no sync); returns the [:B] view."""
        b = positions.shape[0]
        if b > self.max_batch_size:
            raise ValueError("batch size exceeds cache capacity")
        self.seq_lens[:b].copy_(positions[:, -1] + 1)
        return self.seq_lens[:b]

    # -- model-facing step interface (KVCacheManager and RaggedKVCache) -------
    def decode_workspace(self, batch: int, num_heads: int) -> torch.Tensor:
        """Split-KV partials buffer of the decode kernel, kept across steps."""
        key = (batch, num_heads)
        ws = getattr(self, "_decode_ws", None)
        if ws is None or ws[0] != key:
            t = decode_attention_workspace(batch, num_heads, self.max_seq_len, self.head_dim,
                                           self.seq_lens.device)
            ws = (key, t)
            self._decode_ws = ws
        return ws[1]

    @torch.no_grad()
    def prepare_forward(self, positions: torch.Tensor, ctx, num_heads: int) -> None:
        """Per-forward state: a one-token step is a decode step (device
        seq_lens, no host sync); longer inputs are a prefill starting at
        positions[0, 0] for every row (one host read per forward, where the
        reference reads it in every layer, model.py:159-161)."""
        B, S = positions.shape
        if S == 1:
            ctx.decode = True
            ctx.seq_lens = self.set_seq_lens(positions)
            ctx.workspace = self.decode_workspace(B, num_heads)
        else:
            ctx.decode = False
            ctx.start_pos = int(positions[0, 0].item())
            self.seq_lens[:B] = ctx.start_pos + S

    def attend(self, *, layer_idx: int, positions: torch.Tensor, ctx, num_heads: int,
               scale: float, qkv: Optional[torch.Tensor] = None,
               x: Optional[torch.Tensor] = None, packed_qkv=None,
               norm_eps: float = 0.0) -> torch.Tensor:
        """RoPE + append of ``qkv`` [B, S, (H+2Hkv)*D] -- or, given the hidden
        states ``x`` and the "heads"-packed q/k/v weight, the projection with
        RoPE and the append fused in one kernel (``norm_eps > 0``: ``x`` is the
        raw residual stream and the input RMSNorm, folded into the packed
        weight, runs in the same kernel) -- then causal attention of the new
        queries over the cached context; returns [B, S, H*D]."""
        if packed_qkv is not None:
            B, S, _ = x.shape
            self._check_layer(layer_idx)
            if B > self.max_batch_size:
                raise ValueError("batch size exceeds cache capacity")
            q = qkv_rope_append(x, packed_qkv, positions, ctx.cos_table, ctx.sin_table,
                                self.k_cache[layer_idx], self.v_cache[layer_idx], num_heads,
                                self.n_kv_heads, norm_eps=norm_eps)
        else:
            B, S, _ = qkv.shape
            q = self.append_qkv(layer_idx=layer_idx, qkv=qkv, positions=positions,
                                cos_table=ctx.cos_table, sin_table=ctx.sin_table,
                                num_heads=num_heads)
        D = self.head_dim
        kc, vc = self.k_cache[layer_idx], self.v_cache[layer_idx]
        if ctx.decode:
            out = decode_attention(q.view(B, num_heads, D), kc, vc, ctx.seq_lens, scale,
                                   workspace=ctx.workspace)
            return out.view(B, 1, num_heads * D)
        end = ctx.start_pos + S
        out = flash_attention_v2(q, kc[:B, :, :end, :], vc[:B, :, :end, :], causal=True,
                                 sm_scale=scale)
        return out.transpose(1, 2).reshape(B, S, num_heads * D)
