"""Space-Time MoE: routing logits ``W_g x + lam * W_h h_t`` (reference ``layers/st_moe.py``).

* ``lam = lambda_max * sigmoid(lambda_raw)`` (learnable) or the clamped constant;
* balance lock (``st_moe.py:257-334``): an expert that received more than
  ``max(1.5 * expected, 2)`` assignments in ``balance_lock_threshold`` consecutive training
  forwards loses its temporal term (its logit falls back to the spatial logit);
* everything else as ``DeepSeekMoE``.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn

from mamformer_b200 import ops
from mamformer_b200.models.moe import DeepSeekMoE, _routing_mode


class SpaceTimeMoE(DeepSeekMoE):
    def __init__(self, d_model: int, n_shared_experts: int = 2, shared_expert_dim: int = 2304,
                 n_routed_experts: int = 64, top_k: int = 8, routed_expert_dim: int = 576,
                 d_state: int = 128, lambda_init: float = 0.2, lambda_max: float = 0.3,
                 learnable_lambda: bool = True, use_balance_lock: bool = True,
                 balance_lock_threshold: int = 50, router_temperature: float = 1.0,
                 aux_loss_free: bool = True, bias_update_speed: float = 0.001,
                 dropout: float = 0.0) -> None:
        super().__init__(d_model, n_shared_experts, shared_expert_dim, n_routed_experts, top_k,
                         routed_expert_dim, router_temperature, aux_loss_free, bias_update_speed,
                         dropout)
        self.d_state = d_state
        self.lambda_max = lambda_max
        self.learnable_lambda = learnable_lambda
        self.use_balance_lock = use_balance_lock
        self.balance_lock_threshold = balance_lock_threshold
        if learnable_lambda:
            r = lambda_init / lambda_max
            self.lambda_raw = nn.Parameter(torch.tensor(math.log(r / (1.0 - r)), dtype=torch.float32))
        else:
            self.register_buffer("lambda_raw", torch.tensor(lambda_init, dtype=torch.float32))
        self.temporal_proj = nn.Linear(d_state, n_routed_experts, bias=False)
        if use_balance_lock:
            self.register_buffer("_consecutive_count", torch.zeros(n_routed_experts, dtype=torch.long))
        self.register_buffer("_lock_trigger_count", torch.zeros(1, dtype=torch.long))
        nn.init.normal_(self.temporal_proj.weight, mean=0.0, std=0.001)

    def reinit_in_reference_order(self, std: float) -> None:
        super().reinit_in_reference_order(std)
        with torch.no_grad():
            nn.init.normal_(self.temporal_proj.weight, mean=0.0, std=std)

    @property
    def lambda_value(self) -> float:
        return float(self._get_lambda_tensor().item())

    def _get_lambda_tensor(self) -> torch.Tensor:
        if self.learnable_lambda:
            return self.lambda_max * torch.sigmoid(self.lambda_raw)
        return self.lambda_raw.clamp(0.0, self.lambda_max)

    def _temporal_logits(self, xf, h_flat):
        spatial = torch.nn.functional.linear(xf, self.router.weight.to(xf.dtype)).float()
        lam = self._get_lambda_tensor()
        temporal = torch.zeros_like(spatial)
        if h_flat is not None and bool(lam > 0):
            temporal = self.temporal_proj(h_flat.to(self.temporal_proj.weight.dtype)).float() * lam
        return spatial, temporal

    def _apply_balance_lock(self, combined: torch.Tensor, spatial: torch.Tensor):
        info = {"locks_triggered": 0}
        locked = self._replayed("consecutive_count", self._consecutive_count) >= self.balance_lock_threshold
        n = int(locked.sum().item())
        if n > 0:
            info["locks_triggered"] = n
            m = locked.to(combined.dtype).view(1, -1)
            combined = m * spatial + (1.0 - m) * combined
            self._lock_trigger_count += n
        return combined, info

    def _update_consecutive_counts(self, idx: torch.Tensor) -> None:
        total = idx.numel() // self.top_k
        thresh = max(total * self.top_k / self.n_routed_experts * 1.5, 2.0)
        counts = ops.expert_histogram(idx, self.n_routed_experts).float()
        over = counts > thresh
        self._consecutive_count = torch.where(over, self._consecutive_count + 1,
                                              torch.zeros_like(self._consecutive_count))

    def forward(self, x: torch.Tensor, ssm_h_states: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, dict]:
        B, S, d = x.shape
        xf = x.reshape(-1, d)
        h_flat = ssm_h_states.reshape(B * S, -1) if ssm_h_states is not None else None
        aux: dict = {}
        shared = self._shared(xf)
        spatial, temporal = self._temporal_logits(xf, h_flat)
        logits = spatial + temporal
        if self.router_temperature != 1.0:
            logits = logits / self.router_temperature
        if self.use_balance_lock and self.training and h_flat is not None:
            logits, info = self._apply_balance_lock(logits, spatial)
            aux["locks_triggered"] = info["locks_triggered"]
        gates, idx = self._select(logits)
        routed = self._routed(xf, idx, gates)
        if self.aux_loss_free and self.training:
            pass  # bias update happens in _after_routing
        if self.use_balance_lock and self.training and h_flat is not None and _routing_mode() != "replay":
            self._update_consecutive_counts(idx)
        self._after_routing(idx, B * S, aux)
        aux["routed_expert_count"] = self.n_routed_experts
        aux["active_experts"] = self.top_k
        aux["lambda"] = self._get_lambda_tensor().detach()
        if h_flat is not None:
            aux["temporal_bias_mean"] = temporal.mean().detach()
            aux["temporal_bias_std"] = temporal.std().detach()
        return (shared + routed.to(shared.dtype)).view(B, S, d), aux

    def get_load_statistics(self) -> dict:
        stats = super().get_load_statistics()
        stats["lambda"] = self.lambda_value
        stats["consecutive_max"] = int(self._consecutive_count.max().item()) if self.use_balance_lock else 0
        stats["locks_triggered"] = int(self._lock_trigger_count.item()) if self.use_balance_lock else 0
        return stats

    def reset_load_statistics(self) -> None:
        super().reset_load_statistics()
        if self.use_balance_lock:
            self._consecutive_count.zero_()
            self._lock_trigger_count.zero_()

    @property
    def total_expert_params(self) -> int:
        return super().total_expert_params + self.temporal_proj.weight.numel()

    @property
    def active_params_per_token(self) -> int:
        return super().active_params_per_token + self.temporal_proj.weight.numel()
