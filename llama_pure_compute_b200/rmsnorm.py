"""RMSNorm module on the sm_100a row-norm kernel.

Mirrors ``RMSNorm`` / ``rmsnorm_triton_forward``
(src/llama_pure_compute/triton_kernels/rmsnorm.py:58-119): weight initialised
to ones, fp32 statistics, output in the input dtype.  CUDA only.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .ops import rmsnorm_forward

__all__ = ["RMSNorm", "rmsnorm_forward"]


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.dim:
            raise ValueError(f"Expected hidden dimension {self.dim}, got {x.shape[-1]}")
        return rmsnorm_forward(x, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"dim={self.dim}, eps={self.eps}"
