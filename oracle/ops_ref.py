"""Op-level oracle (CPU).  Test infrastructure only -- see oracle/__init__.py.

All math is fp32 unless a function says otherwise; fp32 tensor ops on the CPU
round every elementwise operation separately (no FMA contraction), which is
what the kernels reproduce where bit-exactness is claimed.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F


def rope_ref(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
             position_ids: Optional[torch.Tensor] = None, table_mode: Optional[int] = None):
    """Half-split RoPE.  Math of `_rope_forward_pytorch` (src/llama_pure_compute/ops.py:27-42):
    x*cos + rotate_half(x)*sin, each product and the sum rounded in fp32, then
    one rounding to the storage dtype as src/csrc/ops/rope.cu:39-45 does.

    q [..., H, D], k [..., Hkv, D].  table_mode 0: cos/sin [max_pos, D/2] rows
    picked by position_ids (or token index); 1: per-token [T, D] (or anything
    broadcastable to [..., 1, D])."""
    D = q.shape[-1]
    h = D // 2
    T = q.numel() // (q.shape[-2] * D)
    if table_mode is None:
        table_mode = 0 if (cos.dim() == 2 and cos.shape[-1] == h) else 1
    if table_mode == 0:
        idx = (position_ids.reshape(-1).long() if position_ids is not None
               else torch.arange(T))
        c = cos.float()[idx]
        s = sin.float()[idx]
        c = torch.cat([c, c], -1)
        s = torch.cat([s, s], -1)
    else:
        lead = q.shape[:-2]
        c = cos.float().expand(*lead, 1, D).reshape(T, D)
        s = sin.float().expand(*lead, 1, D).reshape(T, D)

    def rot(x):
        xf = x.float().reshape(T, -1, D)
        x0, x1 = xf[..., :h], xf[..., h:]
        c0, c1 = c[:, None, :h], c[:, None, h:]
        s0, s1 = s[:, None, :h], s[:, None, h:]
        o0 = x0 * c0 - x1 * s0
        o1 = x1 * c1 + x0 * s1
        return torch.cat([o0, o1], -1).reshape(x.shape).to(x.dtype)

    return rot(q), rot(k)


def kv_append_ref(k_src: np.ndarray, v_src: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                  slots: Optional[np.ndarray]) -> None:
    """In-place slot scatter: cache[b, h, pos] = src[t, h] with (b, pos) =
    divmod(slot, S_max), slot < 0 skipped (src/csrc/ops/kv_cache.cu:25-42;
    tests/test_kv_cache.py:85-118).  Out-of-range batch rows are skipped.
    Works on raw bytes (any dtype), so equality is bit-exact."""
    Bmax, H, S, D = k_cache.shape
    T = k_src.shape[0]
    sl = np.arange(T, dtype=np.int64) if slots is None else np.asarray(slots, dtype=np.int64)
    for t in range(T):
        s = int(sl[t])
        if s < 0:
            continue
        b, pos = divmod(s, S)
        if b >= Bmax:
            continue
        k_cache[b, :, pos, :] = k_src[t]
        v_cache[b, :, pos, :] = v_src[t]


def rmsnorm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """`_rmsnorm_pytorch_fallback` (src/llama_pure_compute/triton_kernels/rmsnorm.py:88-96)."""
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return ((xf * r) * w.float()).to(x.dtype)


def rmsswiglu_ref(x: torch.Tensor, w: torch.Tensor, gate_w: torch.Tensor, up_w: Optional[torch.Tensor],
                  eps: float, compute: torch.dtype = torch.float32,
                  round_normed: bool = False) -> torch.Tensor:
    """RMSNorm -> gate/up -> silu(gate)*up in `compute` precision, cast back to
    x.dtype once: `_rmsswiglu_forward_pytorch` (src/llama_pure_compute/ops.py:45-59)
    evaluated the way tests/test_rmsswiglu_correctness.py:35-54 builds its
    ground truth.  up_w None/empty -> gate_w is the fused [2I, D] matrix
    (src/csrc/ops/rmsswiglu.cu:167-173).

    round_normed: store the normalised activations in x's dtype before the
    projections, as the reference CUDA op does (rmsswiglu.cu:178-196 writes
    x_normed with x's dtype and feeds it to the GEMM)."""
    if up_w is None or up_w.numel() == 0:
        inter = gate_w.shape[0] // 2
        gate_w, up_w = gate_w[:inter], gate_w[inter:]
    xf = x.to(compute)
    var = xf.pow(2).mean(-1, keepdim=True)
    xn = xf * torch.rsqrt(var + eps) * w.to(compute)
    if round_normed:
        xn = xn.to(x.dtype).to(compute)
    g = F.linear(xn, gate_w.to(compute))
    u = F.linear(xn, up_w.to(compute))
    return (F.silu(g) * u).to(x.dtype)


def attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                  sm_scale: Optional[float] = None) -> torch.Tensor:
    """fp32 softmax attention with queries at the LAST q_len key positions
    (bottom-right causal mask): `reference_attention`,
    tests/test_attention_correctness.py:10-76.  GQA by repeating K/V heads
    (model.py:170-179).  q [B,H,Sq,D], k/v [B,Hkv,Skv,D]."""
    B, H, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    if sm_scale is None:
        sm_scale = D ** -0.5
    kf, vf = k.float(), v.float()
    if Hkv != H:
        kf = kf.repeat_interleave(H // Hkv, dim=1)
        vf = vf.repeat_interleave(H // Hkv, dim=1)
    s = torch.matmul(q.float(), kf.transpose(-2, -1)) * sm_scale
    if causal:
        qp = torch.arange(Skv - Sq, Skv, device=q.device).view(1, 1, Sq, 1)
        kp = torch.arange(Skv, device=q.device).view(1, 1, 1, Skv)
        s = s.masked_fill(kp > qp, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, vf).to(q.dtype)


def decode_attention_ref(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                         seq_lens, sm_scale: Optional[float] = None) -> torch.Tensor:
    """One query per sequence over its own prefix [0, L_b) of the cache:
    attention_ref with q_len = 1 per sequence (the decode semantics of
    flash_attention.py:450-710, generalised to ragged lengths).
    q [B,H,D]; caches [Bmax,Hkv,Smax,D]; returns [B,H,D] in q.dtype."""
    B, H, D = q.shape
    out = torch.empty(B, H, D, dtype=q.dtype)
    for b in range(B):
        L = int(seq_lens[b])
        if L <= 0:
            out[b] = 0
            continue
        o = attention_ref(q[b:b + 1, :, None, :], k_cache[b:b + 1, :, :L], v_cache[b:b + 1, :, :L],
                          causal=True, sm_scale=sm_scale)
        out[b] = o[0, :, 0]
    return out


def rope_kv_append_ref(qkv: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor,
                       sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       num_heads: int, num_kv_heads: int) -> torch.Tensor:
    """Composition the fused prologue replaces (model.py:146-168 with
    kv_manager.py:260-300): rope_forward on q/k with the position rows of the
    full tables, then the slot scatter of k (rotated) and v at (b, pos).
    Mutates the caches, returns rotated q as [B, H, S, D]."""
    B, S, W = qkv.shape
    D = k_cache.shape[-1]
    H, Hkv = num_heads, num_kv_heads
    q = qkv[..., : H * D].reshape(B, S, H, D)
    k = qkv[..., H * D:(H + Hkv) * D].reshape(B, S, Hkv, D)
    v = qkv[..., (H + Hkv) * D:].reshape(B, S, Hkv, D)
    pos = positions.long()
    c = cos[pos].unsqueeze(2)
    s = sin[pos].unsqueeze(2)
    qr, kr = rope_ref(q, k, c, s, table_mode=1)
    Smax = k_cache.shape[2]
    for b in range(B):
        for t in range(S):
            p = int(pos[b, t])
            if p < 0:
                continue
            k_cache[b, :, p] = kr[b, t]
            v_cache[b, :, p] = v[b, t]
    return qr.permute(0, 2, 1, 3).contiguous()
