"""Attention entry point with the reference signature, on the sm_100a kernels.

``flash_attention_v2(q, k, v, causal=True, sm_scale=None)`` keeps the argument
checks and error types of src/llama_pure_compute/triton_kernels/
flash_attention.py:998-1098.  Dispatch:
  * q_len == 1           -> split-KV decode kernel (lpc_decode_attention),
    head_dim 32, 64 or 128;
  * otherwise            -> tcgen05 flash-attention kernel (lpc_flash_attention),
    causal or not, q_len <= kv_len with bottom-right alignment; head_dim 64
    and 128 natively, head_dim 32 by zero-padding q/k/v to 64 columns (the
    padded dims add nothing to q.k and give zero output columns, dropped).
K and V may be sequence slices of a preallocated ``[B, H, S_max, D]`` cache
(the views ``KVCacheManager.update`` returns): they are read in place through
their strides, without the reference's ``.contiguous()`` copy of the prefix
(flash_attention.py:1100-1102).  GQA (fewer K/V heads) is handled in-kernel.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .ops import decode_attention

__all__ = ["flash_attention_v2"]


def _strides(t: torch.Tensor):
    """(batch, head) strides in elements; size-1 dims get the packed value
    (torch reports arbitrary strides for them)."""
    b, h, s, d = t.shape
    hs = t.stride(1) if h > 1 else s * d
    bs = t.stride(0) if b > 1 else h * hs
    return bs, hs


def _kv_layout_ok(k: torch.Tensor, v: torch.Tensor) -> bool:
    D = k.shape[-1]
    kb, kh = _strides(k)
    return (_strides(v) == (kb, kh) and k.stride(-1) == 1 and (k.shape[2] == 1 or k.stride(-2) == D)
            and kh >= k.shape[2] * D and kb >= k.shape[1] * kh
            and k.storage_offset() % 8 == 0 and v.storage_offset() % 8 == 0)


def flash_attention_v2(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = True,
    sm_scale: Optional[float] = None,
) -> torch.Tensor:
    """softmax(q k^T * sm_scale [+ causal mask]) v with fp32 accumulation.

    q: [B, H, Q_LEN, D]; k, v: [B, H_kv, KV_LEN, D]; Q_LEN <= KV_LEN; queries
    are the last Q_LEN positions of the sequence (bottom-right causal mask,
    tests/test_attention_correctness.py:39-64).
    """
    if not q.is_cuda or not k.is_cuda or not v.is_cuda:
        raise ValueError("FlashAttention requires CUDA tensors.")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must be 4-D tensors.")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("Only FP16 and BF16 are supported.")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("q, k and v must have identical dtype.")
    if q.device != k.device or q.device != v.device:
        raise ValueError("q, k and v must share the same device.")
    bq, hq, q_len, d = q.shape
    bk, hk, kv_len, dk = k.shape
    bv, hv, kv_len_v, dv = v.shape
    if bq != bk or bq != bv:
        raise ValueError("Batch dimensions must match.")
    if hk != hv or hk <= 0 or hq % hk != 0:
        raise ValueError("Head counts must match.")
    if kv_len != kv_len_v:
        raise ValueError("K and V sequence lengths must match.")
    if d != dk or d != dv:
        raise ValueError("Head dimensions must match.")
    if q_len <= 0 or kv_len <= 0:
        raise ValueError("Sequence lengths must be positive.")
    if q_len > kv_len:
        raise ValueError("Q_LEN cannot exceed KV_LEN.")
    if d not in (32, 64, 128):
        raise ValueError("Supported head dimensions: 32, 64, 128.")
    if sm_scale is None:
        sm_scale = d ** -0.5
    q = q.contiguous()
    if not _kv_layout_ok(k, v):
        k = k.contiguous()
        v = v.contiguous()

    if q_len == 1:
        # one query per sequence: the whole prefix is visible, causal or not.
        # Read K/V in place when they are a sequence slice of a [B, H, S_max, D]
        # cache (row pitch S_max); otherwise pack them.
        kb, kh = _strides(k)
        if kb == hk * kh and kh % d == 0 and kh >= kv_len * d:
            smax = kh // d
            shape = (bq, hk, smax, d)
            stride = (hk * smax * d, smax * d, d, 1)
            kc = k.as_strided(shape, stride)
            vc = v.as_strided(shape, stride)
        else:
            kc, vc = k.contiguous(), v.contiguous()
        lens = torch.full((bq,), kv_len, dtype=torch.int32, device=q.device)
        out = decode_attention(q.view(bq, hq, d), kc, vc, lens, sm_scale)
        return out.view(bq, hq, 1, d)

    if d == 32:
        pad = lambda t: torch.nn.functional.pad(t, (0, 32))  # noqa: E731
        out = flash_attention_v2(pad(q), pad(k), pad(v), causal=causal, sm_scale=sm_scale)
        return out[..., :32].contiguous()
    out = torch.empty_like(q)
    rc = _lib.load().lpc_flash_attention(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), bq, hq, hk, q_len, kv_len, d,
        *_strides(k), 1 if causal else 0, float(sm_scale),
        _lib.dtype_code(q.dtype, "flash_attention"), _lib.stream_of(q))
    _lib.check(rc, "flash_attention")
    _lib.count_launch("lpc_flash_attention")
    return out
