"""Decode-step projections on pre-packed weights (``lpc_pack_weights`` +
``lpc_wsgemm``).

The reference runs every projection of a decode step as an ``nn.Linear``
(src/llama_pure_compute/model.py:86-108, 276-293, 421-425) and the gate/up
GEMMs inside ``rmsswiglu_forward`` (src/llama_pure_compute/ops.py:118-131).
With at most a few hundred tokens per step those GEMMs only stream weights,
so the weights are packed once into contiguous tensor-core tiles and each
projection is one kernel with its epilogue (residual add, SiLU * up) fused.

``PackedWeight`` owns the packed bytes.  ``packed_linear`` runs one product.
Layers with few 128-row weight tiles split k over clusters of CTAs (the
partial tiles are reduce-scattered through distributed shared memory), and
every launch overlaps its prologue and first weight chunks with the previous
kernel (programmatic dependent launch).  The packed "heads" layout feeds
``ops.qkv_rope_append``: the attention block's projection with RoPE and the
KV append in the epilogue.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

EPILOGUES = {"store": 0, "residual": 1, "swiglu": 2}
LAYOUTS = {"linear": 0, "swiglu": 1, "heads": 2}
MAX_TOKENS = 256


class PackedWeight:
    """A weight matrix in the packed tile layout.

    layout "linear": ``w0`` is ``[n_out, k]`` (``y = x w0^T``).
    layout "swiglu": ``w0`` holds the gate rows ``[n_out, k]`` and ``w1`` the up
    rows, or ``w1`` is None and ``w0`` is the fused ``[2 n_out, k]`` gate_up
    weight (ops.py:118-131 accepts both forms).
    layout "heads": ``w0`` is the stacked q/k/v projection weight
    ``[(H + 2 Hkv) * 128, k]`` (head_dim 128), for ``ops.qkv_rope_append``.

    ``norm_weight`` (``[k]``, optional) is the weight of the RMSNorm whose
    output this projection consumes.  It is folded into the packed copy
    (``W[n, k] * norm_weight[k]``, one rounding), so that the product can
    normalise its raw input rows itself: ``packed_linear(..., norm_eps=eps)``
    / ``qkv_rope_append(..., norm_eps=eps)``.  ``folds_norm`` records it.
    """

    def __init__(self, w0: torch.Tensor, w1: Optional[torch.Tensor] = None,
                 layout: str = "linear", norm_weight: Optional[torch.Tensor] = None):
        if layout not in LAYOUTS:
            raise ValueError(f"LlamaPureComputeError: unknown packed layout {layout!r}")
        if not w0.is_cuda:
            raise ValueError("LlamaPureComputeError: weights must be on CUDA device.")
        if w0.dim() != 2:
            raise ValueError("LlamaPureComputeError: weight must be 2-D.")
        lay = LAYOUTS[layout]
        w0 = w0.detach().contiguous()
        k = w0.shape[1]
        if layout == "swiglu" and w1 is None:
            if w0.shape[0] % 2:
                raise ValueError("LlamaPureComputeError: fused gate/up weight needs an even row count.")
            n_out = w0.shape[0] // 2
        else:
            n_out = w0.shape[0]
        if w1 is not None:
            w1 = w1.detach().contiguous()
            if tuple(w1.shape) != (n_out, k) or w1.dtype != w0.dtype or w1.device != w0.device:
                raise ValueError("LlamaPureComputeError: up weight must match the gate weight.")
        self.n_out, self.k, self.layout, self.dtype = n_out, k, layout, w0.dtype
        self.device = w0.device
        scale = None
        if norm_weight is not None:
            if norm_weight.numel() != k or norm_weight.device != w0.device:
                raise ValueError("LlamaPureComputeError: norm_weight must be [k] on the weight's "
                                 "device.")
            scale = norm_weight.detach().reshape(-1).to(torch.float32).contiguous()
        self.folds_norm = scale is not None
        lib = _lib.load()
        code = _lib.dtype_code(w0.dtype, "pack_weights")
        nbytes = lib.lpc_packed_weight_bytes(n_out, k, lay)
        if nbytes <= 0:
            raise ValueError(f"LlamaPureComputeError: cannot pack a [{n_out}, {k}] weight "
                             "(k must be a multiple of 64; layout 'heads' needs n_out a "
                             "multiple of 128).")
        with torch.cuda.device(w0.device):
            self.data = torch.empty(nbytes, dtype=torch.uint8, device=w0.device)
            rc = lib.lpc_pack_weights(w0.data_ptr(), _lib.ptr(w1), _lib.ptr(scale),
                                      self.data.data_ptr(), n_out, k, lay, code,
                                      _lib.stream_of(w0))
        _lib.check(rc, "pack_weights")
        _lib.count_launch("lpc_pack_weights")

    @staticmethod
    def supported(w: torch.Tensor) -> bool:
        return (w.is_cuda and w.dim() == 2 and w.dtype in (torch.bfloat16, torch.float16)
                and w.shape[1] % 64 == 0)


def packed_linear(x: torch.Tensor, w: PackedWeight, epilogue: str = "store",
                  resid: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None, norm_eps: float = 0.0) -> torch.Tensor:
    """``epilogue(x w^T)`` for ``x [..., k]`` with at most 256 rows.

    "store": x w^T.  "residual": resid + x w^T (``out`` may be ``resid``).
    "swiglu": silu(x Wg^T) * (x Wu^T) on a weight packed with layout "swiglu".
    fp32 accumulation, one rounding to x's dtype.

    ``norm_eps > 0`` (a weight packed with ``norm_weight``): ``x`` are the raw
    rows of an RMSNorm and the product is that of the normalised rows, i.e.
    ``epilogue(rmsnorm(x) W^T)``, computed without writing them: each token's
    accumulators are scaled by rsqrt(mean(x^2) + eps), its sum of squares taken
    from the activation tiles inside the kernel.
    """
    if epilogue not in EPILOGUES:
        raise ValueError(f"LlamaPureComputeError: unknown epilogue {epilogue!r}")
    if (epilogue == "swiglu") != (w.layout == "swiglu"):
        raise ValueError("LlamaPureComputeError: the swiglu epilogue needs a swiglu-packed weight.")
    if w.layout == "heads":
        raise ValueError("LlamaPureComputeError: a 'heads'-packed weight is for qkv_rope_append.")
    if norm_eps < 0 or (norm_eps > 0) != w.folds_norm:
        raise ValueError("LlamaPureComputeError: norm_eps > 0 needs a weight packed with its "
                         "norm_weight (and only such a weight).")
    if not x.is_cuda:
        raise ValueError("LlamaPureComputeError: x must be on CUDA device.")
    if x.shape[-1] != w.k or x.dtype != w.dtype:
        raise ValueError("LlamaPureComputeError: x must be [..., k] in the weight's dtype.")
    x2 = x.reshape(-1, w.k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    tokens = x2.shape[0]
    if tokens > MAX_TOKENS:
        raise ValueError(f"LlamaPureComputeError: packed_linear takes at most {MAX_TOKENS} rows.")
    shape = (*x.shape[:-1], w.n_out)
    if tokens == 0:
        return torch.empty(shape, dtype=x.dtype, device=x.device) if out is None else out
    epi = EPILOGUES[epilogue]
    rp = None
    if epilogue == "residual":
        if resid is None or resid.numel() != tokens * w.n_out or not resid.is_contiguous():
            raise ValueError("LlamaPureComputeError: residual must be a contiguous [..., n_out] tensor.")
        rp = resid.data_ptr()
    if out is None:
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
    elif out.numel() != tokens * w.n_out or not out.is_contiguous() or out.dtype != x.dtype:
        raise ValueError("LlamaPureComputeError: out must be a contiguous [..., n_out] tensor.")
    rc = _lib.load().lpc_wsgemm(x2.data_ptr(), w.data.data_ptr(), out.data_ptr(), rp, tokens,
                                w.n_out, w.k, epi, _lib.dtype_code(x.dtype, "packed_linear"),
                                float(norm_eps), _lib.stream_of(x))
    _lib.check(rc, "packed_linear")
    _lib.count_launch("lpc_wsgemm")
    return out
