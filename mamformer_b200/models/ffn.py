"""Dense feed-forward blocks (reference ``mamformer/layers/ffn.py``).

``SwiGLUFFN``: ``down(silu(gate(x)) * up(x))``; the SiLU-product runs in the native
``swiglu`` kernel on CUDA.  ``GEGLUFFN`` and ``StandardFFN`` are ablation variants.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamformer_b200 import ops


class SwiGLUFFN(nn.Module):
    def __init__(self, d_model: int, d_ff: int, dropout: float = 0.0, bias: bool = False) -> None:
        super().__init__()
        self.d_model = d_model
        self.d_ff = d_ff
        self.dropout = dropout
        self.gate_proj = nn.Linear(d_model, d_ff, bias=bias)
        self.up_proj = nn.Linear(d_model, d_ff, bias=bias)
        self.down_proj = nn.Linear(d_ff, d_model, bias=bias)
        self.dropout_layer = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        for p in (self.gate_proj, self.up_proj, self.down_proj):
            nn.init.normal_(p.weight, mean=0.0, std=0.02)
            if p.bias is not None:
                nn.init.zeros_(p.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = ops.swiglu(self.gate_proj(x), self.up_proj(x))
        return self.down_proj(self.dropout_layer(h))

    def extra_repr(self) -> str:
        return f"d_model={self.d_model}, d_ff={self.d_ff}, dropout={self.dropout}"


class GEGLUFFN(nn.Module):
    def __init__(self, d_model: int, d_ff: int, dropout: float = 0.0, bias: bool = False) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(d_model, d_ff, bias=bias)
        self.up_proj = nn.Linear(d_model, d_ff, bias=bias)
        self.down_proj = nn.Linear(d_ff, d_model, bias=bias)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        for p in (self.gate_proj, self.up_proj, self.down_proj):
            nn.init.normal_(p.weight, mean=0.0, std=0.02)
            if p.bias is not None:
                nn.init.zeros_(p.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(self.dropout(F.gelu(self.gate_proj(x)) * self.up_proj(x)))


class StandardFFN(nn.Module):
    def __init__(self, d_model: int, d_ff: int, dropout: float = 0.0, bias: bool = False) -> None:
        super().__init__()
        self.fc1 = nn.Linear(d_model, d_ff, bias=bias)
        self.fc2 = nn.Linear(d_ff, d_model, bias=bias)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        for p in (self.fc1, self.fc2):
            nn.init.normal_(p.weight, mean=0.0, std=0.02)
            if p.bias is not None:
                nn.init.zeros_(p.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc2(self.dropout(F.relu(self.fc1(x))))
