"""Mixed-precision layout for B200: bf16 matrices, fp32 vectors.

``to_compute_dtype(model, bf16)`` converts every parameter of a Linear/Embedding module and
every other parameter with >= 2 dims (stacked experts, conv kernels) to bf16, and keeps the
remaining 1-D parameters (norm weights, GroupNorm affine, A_log, D, gates, lambdas) and all
buffers in fp32.  The fused optimizer keeps fp32 master copies of the bf16 weights.
"""

from __future__ import annotations

import torch
import torch.nn as nn


def to_compute_dtype(model: nn.Module, dtype: torch.dtype = torch.bfloat16) -> nn.Module:
    for mod in model.modules():
        dense = isinstance(mod, (nn.Linear, nn.Embedding))
        for name, p in list(mod.named_parameters(recurse=False)):
            want = dtype if (p.dim() >= 2 or dense) else torch.float32
            if p.dtype != want:
                p.data = p.data.to(want)
    return model


def compute_dtype_of(model: nn.Module) -> torch.dtype:
    for p in model.parameters():
        if p.dim() >= 2:
            return p.dtype
    return torch.float32
