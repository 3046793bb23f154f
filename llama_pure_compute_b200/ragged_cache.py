"""Ragged (variable-length) KV cache for mixed-length batches.

The reference cache (src/llama_pure_compute/kv_manager.py:90-121) gives every
sequence ``max_seq_len`` rows of a ``[max_batch, kv_heads, max_seq_len,
head_dim]`` tensor per layer, and one shared ``start_pos`` per batch.  With
prompts of 1k-8k tokens that layout wastes most of HBM: 64 sequences x 8448
rows x 512 KiB (the 7B shape's K+V per token over 32 layers) is 283 GB, while
the tokens actually held need about 165 GB.  This cache packs sequences back
to back instead:

  * per layer, K and V are ``[kv_heads, total_rows, head_dim]``; sequence i
    owns rows ``[base[i], base[i] + capacity[i])`` of every head (the
    paged/ragged layout of runtime/paged_cache.py:14-57, with one page per
    sequence sized at admission);
  * a forward runs on a *selection* of sequences (``select``): batch row b is
    sequence ``ids[b]``; prefill rows start at the same position, decode rows
    may be at different positions (ragged lengths, device ``seq_lens``);
  * the kernels are ``lpc_rope_kv_append_ragged``,
    ``lpc_decode_attention_ragged`` and, for prefill, ``lpc_flash_attention``
    on each sequence's rows (a strided view, no copy).

The step interface (``prepare_forward`` / ``attend``) is the one the model
calls on ``KVCacheManager``; ``LlamaForCausalLM`` takes either cache.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from .flash_attention import flash_attention_v2
from .ops import (decode_attention_ragged, decode_attention_workspace, qkv_rope_append,
                  rope_kv_append_ragged)

__all__ = ["RaggedKVCache"]


class RaggedKVCache:
    def __init__(self, *, num_layers: int, capacities: Sequence[int], n_kv_heads: int,
                 head_dim: int, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str = "cuda"):
        caps = [int(c) for c in capacities]
        if num_layers <= 0 or n_kv_heads <= 0 or head_dim <= 0:
            raise ValueError("num_layers, n_kv_heads and head_dim must be positive")
        if not caps or min(caps) <= 0:
            raise ValueError("every sequence needs a positive capacity")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("RaggedKVCache lives on a CUDA device")
        self.num_layers, self.n_kv_heads, self.head_dim = num_layers, n_kv_heads, head_dim
        self.dtype = dtype
        self.capacities: List[int] = caps
        bases, acc = [], 0
        for c in caps:
            bases.append(acc)
            acc += c
        self.bases: List[int] = bases
        self.total_rows = acc
        self.max_seq_len = max(caps)
        shape = (n_kv_heads, self.total_rows, head_dim)
        self.k_cache = [torch.empty(shape, dtype=dtype, device=self.device) for _ in range(num_layers)]
        self.v_cache = [torch.empty(shape, dtype=dtype, device=self.device) for _ in range(num_layers)]
        self.seq_base = torch.tensor(bases, dtype=torch.int64, device=self.device)
        self.seq_cap = torch.tensor(caps, dtype=torch.int32, device=self.device)
        self.seq_lens = torch.zeros(len(caps), dtype=torch.int32, device=self.device)
        self._ws = None
        self.select(range(len(caps)))

    @property
    def num_sequences(self) -> int:
        return len(self.capacities)

    def memory_footprint_bytes(self) -> int:
        per = self.n_kv_heads * self.total_rows * self.head_dim * torch.empty(0, dtype=self.dtype).element_size()
        return 2 * self.num_layers * per

    def select(self, ids: Sequence[int]) -> None:
        """Batch row b of the next forwards is sequence ids[b]."""
        ids = [int(i) for i in ids]
        if not ids or min(ids) < 0 or max(ids) >= self.num_sequences:
            raise ValueError("sequence ids outside the cache")
        self.active_ids = ids
        idx = torch.tensor(ids, dtype=torch.int64, device=self.device)
        self.active_base = self.seq_base[idx].contiguous()
        self.active_cap = self.seq_cap[idx].contiguous()
        self.active_lens = self.seq_lens[idx].contiguous()
        self._idx = idx

    # -- step interface used by the model ----------------------------------
    def decode_workspace(self, batch: int, num_heads: int) -> torch.Tensor:
        key = (batch, num_heads)
        if self._ws is None or self._ws[0] != key:
            self._ws = (key, decode_attention_workspace(batch, num_heads, self.max_seq_len,
                                                        self.head_dim, self.device))
        return self._ws[1]

    @torch.no_grad()
    def prepare_forward(self, positions: torch.Tensor, ctx, num_heads: int) -> None:
        B, S = positions.shape
        if B != len(self.active_ids):
            raise ValueError(f"batch of {B} rows but {len(self.active_ids)} selected sequences")
        if S == 1:
            ctx.decode = True
            self.active_lens.copy_(positions[:, -1] + 1)
            ctx.seq_lens = self.active_lens
            ctx.workspace = self.decode_workspace(B, num_heads)
        else:
            ctx.decode = False
            ctx.start_pos = int(positions[0, 0].item())
            end = ctx.start_pos + S
            for i in self.active_ids:
                if end > self.capacities[i]:
                    raise ValueError(f"sequence {i}: {end} positions exceed its capacity "
                                     f"{self.capacities[i]}")
            self.active_lens.fill_(end)
        self.seq_lens.index_copy_(0, self._idx, self.active_lens)

    def attend(self, *, layer_idx: int, positions: torch.Tensor, ctx, num_heads: int,
               scale: float, qkv: Optional[torch.Tensor] = None,
               x: Optional[torch.Tensor] = None, packed_qkv=None,
               norm_eps: float = 0.0) -> torch.Tensor:
        D = self.head_dim
        kc, vc = self.k_cache[layer_idx], self.v_cache[layer_idx]
        if packed_qkv is not None:
            B, S, _ = x.shape
            q = qkv_rope_append(x, packed_qkv, positions, ctx.cos_table, ctx.sin_table, kc, vc,
                                num_heads, self.n_kv_heads, seq_base=self.active_base,
                                seq_cap=self.active_cap, norm_eps=norm_eps)
        else:
            B, S, _ = qkv.shape
            q = rope_kv_append_ragged(qkv, positions, ctx.cos_table, ctx.sin_table, kc, vc,
                                      self.active_base, self.active_cap, num_heads,
                                      self.n_kv_heads)
        if ctx.decode:
            out = decode_attention_ragged(q.view(B, num_heads, D), kc, vc, ctx.seq_lens,
                                          self.active_base, self.active_cap, self.max_seq_len,
                                          scale, workspace=ctx.workspace)
            return out.view(B, 1, num_heads * D)
        end = ctx.start_pos + S
        outs = []
        for b, i in enumerate(self.active_ids):
            base = self.bases[i]
            k = kc[:, base:base + end, :].unsqueeze(0)  # [1, Hkv, end, D], rows stride D
            v = vc[:, base:base + end, :].unsqueeze(0)
            outs.append(flash_attention_v2(q[b:b + 1], k, v, causal=True, sm_scale=scale))
        out = torch.cat(outs, 0) if len(outs) > 1 else outs[0]
        return out.transpose(1, 2).reshape(B, S, num_heads * D)
