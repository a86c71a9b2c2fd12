"""RMSNorm and LayerNorm (reference ``mamformer/layers/norm.py:16-71``).

RMSNorm: ``x / sqrt(mean(x^2) + eps) * w (+ b)`` with the statistics in fp32.  On CUDA the
forward and backward run in the native ``rmsnorm`` kernel (one warp per row, fp32 statistics,
bf16 in/out); on CPU the same formula runs in PyTorch.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from mamformer_b200 import ops


class RMSNorm(nn.Module):
    def __init__(self, d_model: int, eps: float = 1e-6, bias: bool = False) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d_model))
        self.bias = nn.Parameter(torch.zeros(d_model)) if bias else None
        self.eps = float(eps)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out = ops.rms_norm(x, self.weight, self.eps)
        if self.bias is not None:
            out = out + self.bias.to(out.dtype)
        return out

    def extra_repr(self) -> str:
        return f"d_model={self.weight.shape[0]}, eps={self.eps}, bias={self.bias is not None}"


class LayerNorm(nn.Module):
    """Plain LayerNorm with fp32 statistics (ablation baseline)."""

    def __init__(self, d_model: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d_model))
        self.bias = nn.Parameter(torch.zeros(d_model))
        self.eps = float(eps)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        mu = xf.mean(-1, keepdim=True)
        var = (xf - mu).pow(2).mean(-1, keepdim=True)
        y = ((xf - mu) * torch.rsqrt(var + self.eps)).to(x.dtype)
        return y * self.weight.to(y.dtype) + self.bias.to(y.dtype)

    def extra_repr(self) -> str:
        return f"d_model={self.weight.shape[0]}, eps={self.eps}"
