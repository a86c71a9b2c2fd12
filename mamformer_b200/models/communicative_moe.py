"""Communicative MoE: attention among the k selected expert outputs of each token.

Reference: ``mamformer/layers/communicative_moe.py``.  For each token the k (unweighted)
expert outputs form a length-k sequence; a pre-norm block ``x += MHA(norm x)``,
``x += FFN(norm x)`` (FFN: d -> 4d -> d with SiLU) mixes them; the result is blended with the
originals by ``sigmoid(comm_strength)``; gates are re-weighted by
``sigmoid(gate_adjustment + 1)`` and renormalised; shared experts are added.

On CUDA the per-slot expert outputs come from the native grouped-GEMM path
(``ops.moe_expert_outputs``), i.e. the same permutation and grouped GEMMs as plain MoE
without the gate-weighted combine.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamformer_b200 import ops
from mamformer_b200.models.norm import RMSNorm
from mamformer_b200.ops.linear import linear as _native_linear


class ExpertCommunicationLayer(nn.Module):
    def __init__(self, d_model: int, n_heads: int = 4, depth: int = 1, dropout: float = 0.0) -> None:
        super().__init__()
        if d_model % n_heads:
            raise ValueError(f"d_model {d_model} must be divisible by n_heads {n_heads}")
        self.d_model = d_model
        self.n_heads = n_heads
        self.depth = depth
        self.head_dim = d_model // n_heads
        self.attn_norms = nn.ModuleList([RMSNorm(d_model) for _ in range(depth)])
        self.cross_attns = nn.ModuleList([
            nn.MultiheadAttention(d_model, n_heads, dropout=dropout, batch_first=True)
            for _ in range(depth)])
        self.ffn_norms = nn.ModuleList([RMSNorm(d_model) for _ in range(depth)])
        self.ffns = nn.ModuleList([
            nn.Sequential(nn.Linear(d_model, 4 * d_model, bias=False), nn.SiLU(),
                          nn.Linear(4 * d_model, d_model, bias=False))
            for _ in range(depth)])
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        for ffn in self.ffns:
            for m in ffn:
                if isinstance(m, nn.Linear):
                    nn.init.normal_(m.weight, mean=0.0, std=0.02)

    def forward(self, expert_outputs: torch.Tensor) -> torch.Tensor:
        x = expert_outputs
        for i in range(self.depth):
            n = self.attn_norms[i](x)
            a, _ = self.cross_attns[i](n, n, n, need_weights=False)
            x = x + self.dropout(a)
            x = x + self.dropout(self.ffns[i](self.ffn_norms[i](x)))
        return x


class CommunicativeMoE(nn.Module):
    def __init__(self, base_moe: nn.Module, d_model: int, n_comm_heads: int = 4,
                 comm_depth: int = 1, comm_dropout: float = 0.0) -> None:
        super().__init__()
        self.base_moe = base_moe
        self.d_model = d_model
        self.comm_layer = ExpertCommunicationLayer(d_model, n_comm_heads, comm_depth, comm_dropout)
        self.gate_adjustment = nn.Parameter(torch.zeros(1, base_moe.top_k))
        self.comm_strength = nn.Parameter(torch.zeros(1))

    @property
    def n_routed_experts(self) -> int:
        return self.base_moe.n_routed_experts

    @property
    def top_k(self) -> int:
        return self.base_moe.top_k

    def forward(self, x: torch.Tensor, ssm_h_states: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, dict]:
        B, S, d = x.shape
        base = self.base_moe
        xf = x.reshape(-1, d)
        shared = base._shared(xf)
        if hasattr(base, "temporal_proj") and ssm_h_states is not None:
            spatial, temporal = base._temporal_logits(xf, ssm_h_states.reshape(B * S, -1))
            logits = spatial + temporal
            if base.use_balance_lock and self.training:
                logits, _ = base._apply_balance_lock(logits, spatial)
        else:
            logits = _native_linear(xf, base.router.weight.to(xf.dtype)).float()
        if base.router_temperature != 1.0:
            logits = logits / base.router_temperature
        gates, idx = base._select(logits)
        if base.ep_engine is not None:
            outs = base.ep_engine.expert_outputs(base, xf, idx)         # (T, k, d)
        else:
            outs = ops.moe_expert_outputs(xf, idx, base.routed_gate_proj, base.routed_up_proj,
                                          base.routed_down_proj)        # (T, k, d)
        comm = self.comm_layer(outs)
        mix = torch.sigmoid(self.comm_strength)
        outs = (1.0 - mix) * outs + mix * comm
        adj = gates * torch.sigmoid(self.gate_adjustment + 1.0)
        adj = adj / (adj.sum(-1, keepdim=True) + 1e-8)
        routed = (outs * adj.unsqueeze(-1).to(outs.dtype)).sum(1)
        aux: dict = {"routed_expert_count": base.n_routed_experts, "active_experts": base.top_k,
                     "comm_strength": mix.detach().squeeze(),
                     "gate_adjustment": torch.sigmoid(self.gate_adjustment + 1.0).mean().detach()}
        base._after_routing(idx, B * S, aux)
        if hasattr(base, "lambda_value"):
            aux["lambda"] = base._get_lambda_tensor().detach()
        return (shared + routed.to(shared.dtype)).view(B, S, d), aux

    def get_load_statistics(self) -> dict:
        stats = self.base_moe.get_load_statistics() if hasattr(self.base_moe, "get_load_statistics") else {}
        stats["comm_strength"] = float(torch.sigmoid(self.comm_strength).item())
        return stats

    def reset_load_statistics(self) -> None:
        if hasattr(self.base_moe, "reset_load_statistics"):
            self.base_moe.reset_load_statistics()

    @property
    def total_expert_params(self) -> int:
        return self.base_moe.total_expert_params + sum(p.numel() for p in self.comm_layer.parameters())

    @property
    def active_params_per_token(self) -> int:
        return self.base_moe.active_params_per_token + sum(p.numel() for p in self.comm_layer.parameters())
