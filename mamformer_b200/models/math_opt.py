"""Optional math extensions (reference ``mamformer/layers/math_opt.py``).

Exported for API parity; like the reference, the model does not enable them by default
(``MamformerBlock(use_dynamic_gate=True)`` / ``use_deepnorm=True`` switch the first and the
last on).

* ``DynamicGate``: ``mean_dim0(sigmoid(W2 silu(W1 normalize(mean_t x)) + b))`` per-dim fusion gate.
* ``EntropyRouter``: router logits mixed with Gaussian noise in proportion to the entropy
  deficit (training only), mix clamped to [0, 0.3].
* ``AdaptiveLambda``: ``lam = sigmoid(scale * (std(q1)+std(q2))/2 + bias) * max_lambda`` per head.
* ``DeepNorm``: ``gamma * residual + update`` with gamma initialised to ``(2 N)^(-1/4)``.
* ``compute_moe_entropy_loss``: ``weight * mean_l (mean(H_l) - target)^2``.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F
from mamformer_b200.ops.linear import linear as _native_linear


class DynamicGate(nn.Module):
    def __init__(self, d_model: int, bottleneck: int = 0):
        super().__init__()
        if bottleneck <= 0:
            bottleneck = max(d_model // 16, 16)
        self.mlp = nn.Sequential(nn.Linear(d_model, bottleneck, bias=False), nn.SiLU(),
                                 nn.Linear(bottleneck, d_model, bias=True))
        nn.init.normal_(self.mlp[0].weight, std=0.02 / bottleneck ** 0.5)
        nn.init.normal_(self.mlp[2].weight, std=0.02 / d_model ** 0.5)
        nn.init.zeros_(self.mlp[2].bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        pooled = F.normalize(x.mean(dim=1).unsqueeze(0), dim=-1).squeeze(0)
        return torch.sigmoid(self.mlp(pooled.to(self.mlp[0].weight.dtype))).mean(dim=0)


class EntropyRouter(nn.Module):
    def __init__(self, d_model: int, n_experts: int, entropy_weight: float = 0.01):
        super().__init__()
        self.d_model = d_model
        self.n_experts = n_experts
        self.entropy_weight = entropy_weight
        self.weight = nn.Parameter(torch.empty(n_experts, d_model))
        nn.init.normal_(self.weight, std=0.02 / n_experts ** 0.5)

    def forward(self, x: torch.Tensor, expert_bias: Optional[torch.Tensor] = None):
        flat = x.reshape(-1, self.d_model)
        logits = _native_linear(flat, self.weight.to(flat.dtype))
        if expert_bias is not None:
            logits = logits + expert_bias
        logp = F.log_softmax(logits, dim=-1)
        entropy = -(logp.exp() * logp).sum(-1)
        max_ent = math.log(self.n_experts)
        norm_ent = entropy / max_ent if max_ent > 0 else entropy
        mix = (self.entropy_weight * (1.0 - norm_ent).unsqueeze(-1)).clamp(0.0, 0.3)
        if self.training:
            scores = (1.0 - mix) * logits + mix * (torch.randn_like(logits) * 0.1)
        else:
            scores = logits
        aux = {"entropy_mean": entropy.mean().detach(), "entropy_normalized": norm_ent.mean().detach(),
               "entropy_weight": self.entropy_weight}
        return scores, entropy, aux


class AdaptiveLambda(nn.Module):
    def __init__(self, n_heads: int, max_lambda: float = 0.99):
        super().__init__()
        self.n_heads = n_heads
        self.max_lambda = max_lambda
        self.scale = nn.Parameter(torch.ones(n_heads) * 0.5)
        self.bias = nn.Parameter(torch.zeros(n_heads))

    def forward(self, q1: torch.Tensor, q2: torch.Tensor) -> torch.Tensor:
        u = (q1.std(dim=(0, 2, 3)) + q2.std(dim=(0, 2, 3))) / 2.0
        return torch.sigmoid(self.scale * u + self.bias) * self.max_lambda


class DeepNorm(nn.Module):
    def __init__(self, d_model: int, n_layers: int = 52, alpha: Optional[float] = None):
        super().__init__()
        self.alpha = alpha if alpha is not None else (2.0 * n_layers) ** (-0.25)
        self.gamma = nn.Parameter(torch.ones(d_model) * self.alpha)

    def forward(self, residual: torch.Tensor, updated: torch.Tensor) -> torch.Tensor:
        return self.gamma.to(residual.dtype) * residual + updated

    def extra_repr(self) -> str:
        return f"alpha={self.alpha:.4f}"


def compute_moe_entropy_loss(entropies, target_entropy: float = 0.5, weight: float = 0.01) -> torch.Tensor:
    terms = [(h.mean() - target_entropy) ** 2 for h in entropies if h.numel() > 0]
    if not terms:
        dev = entropies[0].device if entropies else None
        return torch.tensor(0.0, device=dev)
    return weight * torch.stack(terms).mean()
