"""Operator boundary of the Llama hot path, backed by the sm_100a C-ABI library.

Public names and signatures are those of the reference operator module
(src/llama_pure_compute/ops.py:95-170): ``rope_forward``, ``rmsswiglu_forward``,
``update_kv_cache`` and ``is_cuda_backend_available``.  Unlike the reference
there is no PyTorch fallback: every op runs the hand-written CUDA kernels and
raises if they cannot run (CPU tensors, missing library).

Conventions kept from the reference bindings (src/csrc/ops/bindings.cpp:51-105):
inputs are made contiguous (ops.py:102-107), outputs are allocated through the
torch caching allocator on the current stream, nothing synchronises, invalid
arguments raise ValueError.

Extra ops used by the model's fused attention block (not in the reference's
ops module): ``rmsnorm_forward``, ``rope_kv_append`` and ``decode_attention``.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib

__all__ = [
    "rope_forward",
    "rmsswiglu_forward",
    "update_kv_cache",
    "is_cuda_backend_available",
    "rmsnorm_forward",
    "rope_kv_append",
    "decode_attention",
    "rope_kv_append_ragged",
    "qkv_rope_append",
    "decode_attention_ragged",
]


def _require_cuda(t: Optional[torch.Tensor], name: str) -> None:
    # bindings.cpp:51-61 validate_cuda_tensor
    if t is None:
        raise ValueError(f"LlamaPureComputeError: {name} Tensor is undefined.")
    if not t.is_cuda:
        raise ValueError(f"LlamaPureComputeError: {name} must be on CUDA device.")


def is_cuda_backend_available() -> bool:
    """True when the sm_100a library loads and a CUDA device is present (ops.py:169-170)."""
    return torch.cuda.is_available() and _lib.available()


# ---------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------
def rope_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    position_ids: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Rotary embedding applied in place to q [..., H, D] and k [..., Hkv, D].

    Reference: ops.py:95-117 (dispatch), rope.cu:143-193 (CUDA), ops.py:27-42
    (rotate_half math).  Accepted table forms:
      * ``[max_pos, D/2]`` half tables indexed by ``position_ids`` (or by token
        index when ``position_ids`` is None) -- the CUDA kernel/test convention;
      * per-token full-width tables broadcastable to ``[..., 1, D]`` -- what
        ``LlamaModel.forward`` passes (model.py:388-393);
      * a ``[max_pos, D]`` full table with ``position_ids`` (gathered here).
    Returns the same (contiguous) q and k tensors, rotated.
    """
    for t, n in ((q, "q"), (k, "k"), (cos, "cos"), (sin, "sin")):
        _require_cuda(t, n)
    if position_ids is not None:
        _require_cuda(position_ids, "position_ids")
    if q.dtype != k.dtype:
        raise ValueError("LlamaPureComputeError: Query (q) and Key (k) must have same scalar type.")
    if cos.dtype != sin.dtype or cos.shape != sin.shape:
        raise ValueError("LlamaPureComputeError: cos and sin must share shape and dtype.")
    q = q.contiguous()
    k = k.contiguous()
    D = q.shape[-1]
    H = q.shape[-2]
    Hkv = k.shape[-2]
    if k.shape[-1] != D:
        raise ValueError("LlamaPureComputeError: q and k head dims differ.")
    T = q.numel() // (H * D)
    if k.numel() // (Hkv * D) != T:
        raise ValueError("LlamaPureComputeError: q and k token counts differ.")
    pos = None
    if cos.dim() == 2 and cos.shape[-1] == D // 2:
        mode = 0
        rows = cos.shape[0]
        cos_c, sin_c = cos.contiguous(), sin.contiguous()
        if position_ids is not None:
            pos = position_ids.reshape(-1).to(torch.int64).contiguous()
            if pos.numel() != T:
                raise ValueError("LlamaPureComputeError: position_ids must have one entry per token.")
    elif cos.shape[-1] == D:
        mode = 1
        if cos.dim() == 2 and position_ids is not None and cos.shape[0] != T:
            idx = position_ids.reshape(-1).to(torch.int64)
            cos_c, sin_c = cos[idx].contiguous(), sin[idx].contiguous()
        else:
            lead = q.shape[:-2]
            try:
                cos_c = cos.expand(*lead, 1, D).reshape(T, D).contiguous()
                sin_c = sin.expand(*lead, 1, D).reshape(T, D).contiguous()
            except RuntimeError:
                cos_c = cos.reshape(-1, D).expand(T, D).contiguous() if cos.numel() == D else None
                sin_c = sin.reshape(-1, D).expand(T, D).contiguous() if sin.numel() == D else None
                if cos_c is None:
                    raise ValueError(
                        f"LlamaPureComputeError: cos/sin shape {tuple(cos.shape)} does not "
                        f"broadcast to the tokens of q {tuple(q.shape)}.") from None
        rows = T
    else:
        raise ValueError(
            f"LlamaPureComputeError: cos/sin last dim must be head_dim ({D}) or head_dim/2.")
    lib = _lib.load()
    rc = lib.lpc_rope_forward(
        q.data_ptr(), k.data_ptr(), cos_c.data_ptr(), sin_c.data_ptr(), _lib.ptr(pos), T, H, Hkv, D,
        mode, rows, _lib.dtype_code(q.dtype, "rope_forward"),
        _lib.dtype_code(cos_c.dtype, "rope_forward"), _lib.stream_of(q))
    _lib.check(rc, "rope_forward")
    _lib.count_launch("lpc_rope_forward")
    return q, k


# ---------------------------------------------------------------------------
# RMSNorm and fused RMSNorm + SwiGLU
# ---------------------------------------------------------------------------
def rmsnorm_forward(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Row RMSNorm, fp32 math (triton_kernels/rmsnorm.py:58-96)."""
    _require_cuda(x, "x")
    _require_cuda(weight, "weight")
    x = x.contiguous()
    weight = weight.contiguous()
    D = x.shape[-1]
    if weight.numel() != D:
        raise ValueError(f"LlamaPureComputeError: Expected hidden dimension {weight.numel()}, got {D}")
    out = torch.empty_like(x)
    rows = x.numel() // D if D else 0
    rc = _lib.load().lpc_rmsnorm_forward(
        x.data_ptr(), weight.data_ptr(), out.data_ptr(), rows, D, float(eps),
        _lib.dtype_code(x.dtype, "rmsnorm"), _lib.dtype_code(weight.dtype, "rmsnorm"),
        _lib.stream_of(x))
    _lib.check(rc, "rmsnorm_forward")
    _lib.count_launch("lpc_rmsnorm_forward")
    return out


def rmsswiglu_forward(
    x: torch.Tensor,
    rms_weight: torch.Tensor,
    gate_w: torch.Tensor,
    up_w: torch.Tensor,
    eps: float = 1e-5,
) -> torch.Tensor:
    """silu(norm(x) gate_w^T) * (norm(x) up_w^T) in one op (ops.py:120-136).

    ``up_w`` with no elements means ``gate_w`` holds the fused ``[2I, D]``
    weight (rmsswiglu.cu:167-173).  bf16/fp16 run on tcgen05 tensor cores with
    fp32 accumulation; fp32 runs the CUDA-core streaming kernel (no TF32).
    """
    for t, n in ((x, "x"), (rms_weight, "rms_weight"), (gate_w, "gate_w"), (up_w, "up_w")):
        _require_cuda(t, n)
    if eps <= 0.0:
        raise ValueError("LlamaPureComputeError: eps must be strictly positive.")
    x = x.contiguous()
    rms_weight = rms_weight.contiguous()
    gate_w = gate_w.contiguous()
    fused = up_w.numel() == 0
    up_c = None if fused else up_w.contiguous()
    D = x.shape[-1]
    if gate_w.dim() != 2 or gate_w.shape[1] != D:
        raise ValueError("LlamaPureComputeError: gate_w must be [inter, dim].")
    inter = gate_w.shape[0] // 2 if fused else gate_w.shape[0]
    if fused and gate_w.shape[0] % 2:
        raise ValueError("LlamaPureComputeError: fused gate/up weight needs an even row count.")
    if up_c is not None and tuple(up_c.shape) != (inter, D):
        raise ValueError("LlamaPureComputeError: up_w must match gate_w's shape.")
    if rms_weight.numel() != D:
        raise ValueError("LlamaPureComputeError: rms_weight must have dim elements.")
    if gate_w.dtype != x.dtype or (up_c is not None and up_c.dtype != x.dtype):
        raise TypeError("LlamaPureComputeError: gate_w/up_w must have x's dtype.")
    tokens = x.numel() // D
    out = torch.empty(*x.shape[:-1], inter, dtype=x.dtype, device=x.device)
    lib = _lib.load()
    code = _lib.dtype_code(x.dtype, "rmsswiglu_forward")
    ws_bytes = lib.lpc_rmsswiglu_workspace_bytes(tokens, D, code)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=x.device)
    rc = lib.lpc_rmsswiglu_forward(
        x.data_ptr(), rms_weight.data_ptr(), gate_w.data_ptr(), _lib.ptr(up_c), out.data_ptr(),
        ws.data_ptr(), ws.numel(), tokens, D, inter, float(eps), code,
        _lib.dtype_code(rms_weight.dtype, "rmsswiglu_forward"), _lib.stream_of(x))
    _lib.check(rc, "rmsswiglu_forward")
    _lib.count_launch("lpc_rmsswiglu_forward", 1 if x.dtype == torch.float32 else 2)
    return out


def rmsswiglu_folded_forward(x: torch.Tensor, gate_w: torch.Tensor, up_w: Optional[torch.Tensor],
                             eps: float = 1e-5) -> torch.Tensor:
    """``silu(norm(x) Wg^T) * (norm(x) Wu^T)`` in one kernel, for weights that
    already carry the norm weight (``gate_w = Wg * rms_weight`` column-wise,
    e.g. folded once when a model is loaded; ``up_w`` None: ``gate_w`` is the
    fused ``[2I, D]`` form).  The tcgen05 CTA-pair GEMM reads the raw rows of
    ``x``, takes each row's sum of squares from the tiles it feeds the tensor
    core and scales the accumulators by ``rsqrt(mean(x^2) + eps)``: the norm of
    ops.py:45-59 without its HBM round trip (rmsswiglu.cu:176-196)."""
    for t, n in ((x, "x"), (gate_w, "gate_w")):
        _require_cuda(t, n)
    if eps <= 0.0:
        raise ValueError("LlamaPureComputeError: eps must be strictly positive.")
    x = x.contiguous()
    gate_w = gate_w.contiguous()
    D = x.shape[-1]
    fused = up_w is None
    inter = gate_w.shape[0] // 2 if fused else gate_w.shape[0]
    if gate_w.dim() != 2 or gate_w.shape[1] != D or (up_w is not None and tuple(up_w.shape) != (inter, D)):
        raise ValueError("LlamaPureComputeError: gate_w/up_w must be [inter, dim].")
    if gate_w.dtype != x.dtype or (up_w is not None and up_w.dtype != x.dtype):
        raise TypeError("LlamaPureComputeError: gate_w/up_w must have x's dtype.")
    up_c = None if up_w is None else up_w.contiguous()
    tokens = x.numel() // D
    out = torch.empty(*x.shape[:-1], inter, dtype=x.dtype, device=x.device)
    rc = _lib.load().lpc_rmsswiglu_folded_forward(
        x.data_ptr(), gate_w.data_ptr(), _lib.ptr(up_c), out.data_ptr(), tokens, D, inter,
        float(eps), _lib.dtype_code(x.dtype, "rmsswiglu_folded_forward"), _lib.stream_of(x))
    _lib.check(rc, "rmsswiglu_folded_forward")
    if tokens:
        _lib.count_launch("lpc_rmsswiglu_folded_forward")
    return out


# ---------------------------------------------------------------------------
# KV cache
# ---------------------------------------------------------------------------
def update_kv_cache(
    key_src: torch.Tensor,
    value_src: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: Optional[torch.Tensor] = None,
) -> None:
    """Scatter new K/V tokens into ``[B, Hkv, S, D]`` caches in place (ops.py:139-166).

    ``slot_mapping`` (int64, one per token) encodes ``b * S + pos``; negative
    slots are skipped (kv_cache.cu:25-42).  None means slot = token index.
    """
    for t, n in ((key_src, "key_src"), (value_src, "value_src"), (key_cache, "key_cache"),
                 (value_cache, "value_cache")):
        _require_cuda(t, n)
    if key_cache.dim() != 4 or value_cache.shape != key_cache.shape:
        raise ValueError("LlamaPureComputeError: caches must be matching [B, H, S, D] tensors.")
    if not key_cache.is_contiguous() or not value_cache.is_contiguous():
        raise ValueError("LlamaPureComputeError: key_cache must be memory-contiguous.")
    if key_src.shape != value_src.shape:
        raise ValueError("LlamaPureComputeError: K/V shapes must match")
    if key_src.dtype != key_cache.dtype or value_src.dtype != value_cache.dtype:
        raise TypeError("LlamaPureComputeError: source and cache dtypes differ.")
    Bmax, Hkv, Smax, D = key_cache.shape
    if key_src.shape[-1] != D or key_src.shape[-2] != Hkv:
        raise ValueError("LlamaPureComputeError: source rows must be [..., kv_heads, head_dim].")
    k = key_src.contiguous()
    v = value_src.contiguous()
    T = k.numel() // (Hkv * D)
    slots = None
    if slot_mapping is not None:
        _require_cuda(slot_mapping, "slot_mapping")
        slots = slot_mapping.reshape(-1).to(torch.int64).contiguous()
        if slots.numel() != T:
            raise ValueError("LlamaPureComputeError: slot_mapping must have one entry per token.")
    rc = _lib.load().lpc_update_kv_cache(
        k.data_ptr(), v.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), _lib.ptr(slots),
        T, Hkv * D, Hkv, D, Bmax, Smax, k.element_size(), _lib.stream_of(k))
    _lib.check(rc, "update_kv_cache")
    if T:
        _lib.count_launch("lpc_update_kv_cache")


def rope_kv_append(
    qkv: torch.Tensor,
    positions: torch.Tensor,
    cos_table: torch.Tensor,
    sin_table: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    num_heads: int,
    num_kv_heads: int,
    q_out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Fused attention prologue: rotate q/k of ``qkv`` [B, S, (H+2Hkv)*D] at
    ``positions`` [B, S], append rotated k and v to the caches at those
    positions, return q as [B, H, S, D].  Replaces model.py:146-168 +
    kv_manager.py:260-300."""
    for t, n in ((qkv, "qkv"), (positions, "positions"), (cos_table, "cos"), (sin_table, "sin"),
                 (key_cache, "key_cache"), (value_cache, "value_cache")):
        _require_cuda(t, n)
    B, S, W = qkv.shape
    Bmax, Hkv, Smax, D = key_cache.shape
    if Hkv != num_kv_heads or W != (num_heads + 2 * num_kv_heads) * D:
        raise ValueError("LlamaPureComputeError: qkv width does not match heads * head_dim.")
    if cos_table.shape[-1] != D or cos_table.dim() != 2:
        raise ValueError("LlamaPureComputeError: rope tables must be [max_pos, head_dim].")
    qkv = qkv.contiguous()
    pos = positions.to(torch.int64).contiguous()
    if pos.shape != (B, S):
        raise ValueError("LlamaPureComputeError: positions must be [batch, seq].")
    if q_out is None:
        q_out = torch.empty(B, num_heads, S, D, dtype=qkv.dtype, device=qkv.device)
    rc = _lib.load().lpc_rope_kv_append(
        qkv.data_ptr(), pos.data_ptr(), cos_table.data_ptr(), sin_table.data_ptr(),
        cos_table.shape[0], q_out.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), B, S,
        num_heads, num_kv_heads, D, Bmax, Smax, _lib.dtype_code(qkv.dtype, "rope_kv_append"),
        _lib.dtype_code(cos_table.dtype, "rope_kv_append"), _lib.stream_of(qkv))
    _lib.check(rc, "rope_kv_append")
    _lib.count_launch("lpc_rope_kv_append")
    return q_out


def decode_attention_workspace(batch: int, heads: int, max_seq_len: int, head_dim: int,
                               device) -> torch.Tensor:
    n = _lib.load().lpc_decode_attention_workspace_bytes(batch, heads, max_seq_len, head_dim)
    return torch.empty(max(n, 16), dtype=torch.uint8, device=device)


def decode_attention(
    q: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    seq_lens: torch.Tensor,
    sm_scale: Optional[float] = None,
    out: Optional[torch.Tensor] = None,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One-token attention per sequence over ragged cache lengths.

    q: [B, H, D] (or [B, H, 1, D]); caches [Bmax, Hkv, Smax, D]; seq_lens int32
    [B] on the device (keys [0, seq_lens[b]) are attended).  Generalises the
    reference decode kernel (flash_attention.py:450-710) from one KV_LEN per
    call to per-sequence lengths.  Returns [B, H, D] (same rank as q).
    """
    for t, n in ((q, "q"), (key_cache, "key_cache"), (value_cache, "value_cache"),
                 (seq_lens, "seq_lens")):
        _require_cuda(t, n)
    if seq_lens.dtype != torch.int32:
        raise TypeError("LlamaPureComputeError: seq_lens must be int32.")
    Bmax, Hkv, Smax, D = key_cache.shape
    B, H = q.shape[0], q.shape[1]
    if q.shape[-1] != D or q.numel() != B * H * D:
        raise ValueError("LlamaPureComputeError: q must be [B, H, D] with the cache's head_dim.")
    if seq_lens.numel() < B:
        raise ValueError("LlamaPureComputeError: seq_lens must have an entry per sequence.")
    if q.dtype != key_cache.dtype:
        raise TypeError("LlamaPureComputeError: q and cache dtypes differ.")
    qc = q.contiguous()
    if sm_scale is None:
        sm_scale = D ** -0.5
    if out is None:
        out = torch.empty_like(qc)
    lib = _lib.load()
    need = lib.lpc_decode_attention_workspace_bytes(B, H, Smax, D)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    rc = lib.lpc_decode_attention(
        qc.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), seq_lens.data_ptr(),
        out.data_ptr(), workspace.data_ptr(), workspace.numel(), B, H, Hkv, D, Bmax, Smax,
        float(sm_scale), _lib.dtype_code(q.dtype, "decode_attention"), _lib.stream_of(q))
    _lib.check(rc, "decode_attention")
    _lib.count_launch("lpc_decode_attention", _lib.decode_kernels(B, Hkv, Smax))
    return out


# ---------------------------------------------------------------------------
# Ragged KV layout: caches [Hkv, total_rows, D], sequence b owns rows
# [seq_base[b], seq_base[b] + seq_cap[b]) of every head.
# ---------------------------------------------------------------------------
def _check_ragged_index(seq_base: torch.Tensor, seq_cap: torch.Tensor, B: int) -> None:
    _require_cuda(seq_base, "seq_base")
    _require_cuda(seq_cap, "seq_cap")
    if seq_base.dtype != torch.int64 or seq_cap.dtype != torch.int32:
        raise TypeError("LlamaPureComputeError: seq_base must be int64 and seq_cap int32.")
    if seq_base.numel() < B or seq_cap.numel() < B or not seq_base.is_contiguous() \
            or not seq_cap.is_contiguous():
        raise ValueError("LlamaPureComputeError: seq_base/seq_cap need a contiguous entry per sequence.")


def rope_kv_append_ragged(
    qkv: torch.Tensor,
    positions: torch.Tensor,
    cos_table: torch.Tensor,
    sin_table: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    seq_base: torch.Tensor,
    seq_cap: torch.Tensor,
    num_heads: int,
    num_kv_heads: int,
    q_out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``rope_kv_append`` into a ragged cache ``[Hkv, total_rows, D]``: row b of
    ``qkv`` [B, S, (H+2Hkv)*D] is sequence b, its position p goes to cache row
    ``seq_base[b] + p``.  Returns q as [B, H, S, D]."""
    for t, n in ((qkv, "qkv"), (positions, "positions"), (cos_table, "cos"), (sin_table, "sin"),
                 (key_cache, "key_cache"), (value_cache, "value_cache")):
        _require_cuda(t, n)
    B, S, W = qkv.shape
    Hkv, total_rows, D = key_cache.shape
    if Hkv != num_kv_heads or W != (num_heads + 2 * num_kv_heads) * D:
        raise ValueError("LlamaPureComputeError: qkv width does not match heads * head_dim.")
    if value_cache.shape != key_cache.shape:
        raise ValueError("LlamaPureComputeError: key and value caches differ in shape.")
    if cos_table.shape[-1] != D or cos_table.dim() != 2:
        raise ValueError("LlamaPureComputeError: rope tables must be [max_pos, head_dim].")
    _check_ragged_index(seq_base, seq_cap, B)
    qkv = qkv.contiguous()
    pos = positions.to(torch.int64).contiguous()
    if pos.shape != (B, S):
        raise ValueError("LlamaPureComputeError: positions must be [batch, seq].")
    if q_out is None:
        q_out = torch.empty(B, num_heads, S, D, dtype=qkv.dtype, device=qkv.device)
    rc = _lib.load().lpc_rope_kv_append_ragged(
        qkv.data_ptr(), pos.data_ptr(), cos_table.data_ptr(), sin_table.data_ptr(),
        cos_table.shape[0], q_out.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
        seq_base.data_ptr(), seq_cap.data_ptr(), B, S, num_heads, num_kv_heads, D, total_rows,
        _lib.dtype_code(qkv.dtype, "rope_kv_append_ragged"),
        _lib.dtype_code(cos_table.dtype, "rope_kv_append_ragged"), _lib.stream_of(qkv))
    _lib.check(rc, "rope_kv_append_ragged")
    _lib.count_launch("lpc_rope_kv_append_ragged")
    return q_out


def qkv_rope_append(
    x: torch.Tensor,
    packed_qkv,
    positions: torch.Tensor,
    cos_table: torch.Tensor,
    sin_table: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    num_heads: int,
    num_kv_heads: int,
    seq_base: Optional[torch.Tensor] = None,
    seq_cap: Optional[torch.Tensor] = None,
    q_out: Optional[torch.Tensor] = None,
    norm_eps: float = 0.0,
) -> torch.Tensor:
    """The attention block's q/k/v projection with RoPE and the KV append in
    its epilogue (model.py:125-168 + kv_manager.py:260-300 in one kernel).

    ``norm_eps > 0``: ``x`` are the raw hidden states and the input RMSNorm
    (model.py:305) runs inside the kernel; ``packed_qkv`` must then be packed
    with that norm's weight (``PackedWeight(..., norm_weight=w)``).

    ``x`` [B, S, dim] are the normed hidden states, ``packed_qkv`` the stacked
    q/k/v weight packed with layout "heads" (head_dim 128), B * S <= 256.
    Equivalent to ``rope_kv_append(x @ W^T, ...)`` (dense cache
    ``[Bmax, Hkv, Smax, D]``) or ``rope_kv_append_ragged`` (cache
    ``[Hkv, total_rows, D]`` with ``seq_base`` / ``seq_cap``), with the
    projection rounded to the dtype before the rotation.  Returns q as
    [B, H, S, D]."""
    for t, n in ((x, "x"), (positions, "positions"), (cos_table, "cos"), (sin_table, "sin"),
                 (key_cache, "key_cache"), (value_cache, "value_cache")):
        _require_cuda(t, n)
    if getattr(packed_qkv, "layout", None) != "heads":
        raise ValueError("LlamaPureComputeError: qkv_rope_append needs a weight packed with "
                         "layout 'heads'.")
    if x.dim() != 3:
        raise ValueError("LlamaPureComputeError: x must be [batch, seq, dim].")
    B, S, dim = x.shape
    ragged = seq_base is not None
    if ragged:
        Hkv, total_rows, D = key_cache.shape
        _check_ragged_index(seq_base, seq_cap, B)
        Bmax = Smax = 0
    else:
        Bmax, Hkv, Smax, D = key_cache.shape
        total_rows = 0
        if B > Bmax:
            raise ValueError("LlamaPureComputeError: batch size exceeds cache capacity.")
    if value_cache.shape != key_cache.shape:
        raise ValueError("LlamaPureComputeError: key and value caches differ in shape.")
    if Hkv != num_kv_heads or packed_qkv.n_out != (num_heads + 2 * num_kv_heads) * D:
        raise ValueError("LlamaPureComputeError: packed weight does not match heads * head_dim.")
    if dim != packed_qkv.k or x.dtype != packed_qkv.dtype:
        raise ValueError("LlamaPureComputeError: x must be [..., k] in the weight's dtype.")
    if norm_eps < 0 or (norm_eps > 0) != getattr(packed_qkv, "folds_norm", False):
        raise ValueError("LlamaPureComputeError: norm_eps > 0 needs a weight packed with its "
                         "norm_weight (and only such a weight).")
    if cos_table.shape[-1] != D or cos_table.dim() != 2:
        raise ValueError("LlamaPureComputeError: rope tables must be [max_pos, head_dim].")
    x = x.contiguous()
    pos = positions.to(torch.int64).contiguous()
    if pos.shape != (B, S):
        raise ValueError("LlamaPureComputeError: positions must be [batch, seq].")
    if q_out is None:
        q_out = torch.empty(B, num_heads, S, D, dtype=x.dtype, device=x.device)
    rc = _lib.load().lpc_qkv_rope_append(
        x.data_ptr(), packed_qkv.data.data_ptr(), pos.data_ptr(), cos_table.data_ptr(),
        sin_table.data_ptr(), cos_table.shape[0], q_out.data_ptr(), key_cache.data_ptr(),
        value_cache.data_ptr(), _lib.ptr(seq_base), _lib.ptr(seq_cap), B, S, num_heads,
        num_kv_heads, D, dim, Bmax, Smax, total_rows, _lib.dtype_code(x.dtype, "qkv_rope_append"),
        _lib.dtype_code(cos_table.dtype, "qkv_rope_append"), float(norm_eps), _lib.stream_of(x))
    _lib.check(rc, "qkv_rope_append")
    _lib.count_launch("lpc_qkv_rope_append")
    return q_out


def decode_attention_ragged(
    q: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    seq_lens: torch.Tensor,
    seq_base: torch.Tensor,
    seq_cap: torch.Tensor,
    max_seq_len: int,
    sm_scale: Optional[float] = None,
    out: Optional[torch.Tensor] = None,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``decode_attention`` over a ragged cache ``[Hkv, total_rows, D]``:
    sequence b attends to rows ``seq_base[b] .. seq_base[b] + seq_lens[b]``.
    ``max_seq_len`` must bound every ``seq_cap`` entry."""
    for t, n in ((q, "q"), (key_cache, "key_cache"), (value_cache, "value_cache"),
                 (seq_lens, "seq_lens")):
        _require_cuda(t, n)
    if seq_lens.dtype != torch.int32:
        raise TypeError("LlamaPureComputeError: seq_lens must be int32.")
    Hkv, total_rows, D = key_cache.shape
    B, H = q.shape[0], q.shape[1]
    if q.shape[-1] != D or q.numel() != B * H * D:
        raise ValueError("LlamaPureComputeError: q must be [B, H, D] with the cache's head_dim.")
    if seq_lens.numel() < B:
        raise ValueError("LlamaPureComputeError: seq_lens must have an entry per sequence.")
    if q.dtype != key_cache.dtype:
        raise TypeError("LlamaPureComputeError: q and cache dtypes differ.")
    _check_ragged_index(seq_base, seq_cap, B)
    qc = q.contiguous()
    if sm_scale is None:
        sm_scale = D ** -0.5
    if out is None:
        out = torch.empty_like(qc)
    lib = _lib.load()
    need = lib.lpc_decode_attention_workspace_bytes(B, H, max_seq_len, D)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    rc = lib.lpc_decode_attention_ragged(
        qc.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), seq_lens.data_ptr(),
        seq_base.data_ptr(), seq_cap.data_ptr(), out.data_ptr(), workspace.data_ptr(),
        workspace.numel(), B, H, Hkv, D, total_rows, max_seq_len, float(sm_scale),
        _lib.dtype_code(q.dtype, "decode_attention_ragged"), _lib.stream_of(q))
    _lib.check(rc, "decode_attention_ragged")
    _lib.count_launch("lpc_decode_attention_ragged",
                      _lib.decode_kernels(B, Hkv, max_seq_len, total_rows))
    return out
