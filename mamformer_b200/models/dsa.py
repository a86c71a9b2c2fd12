"""Differential state-aware attention, the pre-KDA variant (reference ``layers/dsa.py``).

Same differential softmax as ``FullDiffAttention`` with plain K/V projections.  Two injection
paths: per-timestep ``h_states`` (``k += W h[..., :64]``) or, when only a final SSM state is
given (legacy cached decode), ``state_summary = mean_N(ssm_state)`` padded/truncated to
d_model through a 2-layer SiLU MLP and broadcast over time.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamformer_b200 import ops
from mamformer_b200.models.kda_diff import _lambda, _logit, state_injection_input
from mamformer_b200.models.rope import RotaryEmbedding


class DifferentialStateAttention(nn.Module):
    def __init__(self, d_model: int, n_heads: int = 32, n_kv_heads: int = 8, head_dim: int = 128,
                 max_seq_len: int = 8192, rope_theta: float = 10000.0, lambda_init: float = 0.8,
                 use_state_injection: bool = True, state_injection_dim: int = 64,
                 dropout: float = 0.0, sliding_window: int = 0, use_yarn: bool = False,
                 yarn_scale: float = 1.0, yarn_original_max_seq_len: int = 8192,
                 window_mode: str = "reference") -> None:
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.n_head_groups = n_heads // n_kv_heads
        self.dropout = dropout
        self.sliding_window = sliding_window
        self.window_mode = window_mode
        self.use_state_injection = use_state_injection
        self.state_injection_dim = state_injection_dim
        kv = n_kv_heads * head_dim
        self.q1_proj = nn.Linear(d_model, n_heads * head_dim, bias=False)
        self.q2_proj = nn.Linear(d_model, n_heads * head_dim, bias=False)
        self.k_proj = nn.Linear(d_model, kv, bias=False)
        self.v_proj = nn.Linear(d_model, kv, bias=False)
        self.o_proj = nn.Linear(n_heads * head_dim, d_model, bias=False)
        self.lambda_raw = nn.Parameter(torch.full((n_heads,), _logit(lambda_init)))
        if use_state_injection:
            self.state_k_proj = nn.Sequential(nn.Linear(d_model, state_injection_dim, bias=False),
                                              nn.SiLU(), nn.Linear(state_injection_dim, kv, bias=False))
            self.state_v_proj = nn.Sequential(nn.Linear(d_model, state_injection_dim, bias=False),
                                              nn.SiLU(), nn.Linear(state_injection_dim, kv, bias=False))
            self.h_state_k_proj = nn.Linear(state_injection_dim, kv, bias=False)
            self.h_state_v_proj = nn.Linear(state_injection_dim, kv, bias=False)
        self.group_norm = nn.GroupNorm(n_heads, n_heads * head_dim, eps=1e-6)
        self.rope = RotaryEmbedding(head_dim, max_seq_len, rope_theta, use_yarn, yarn_scale,
                                    yarn_original_max_seq_len)
        for p in (self.q1_proj, self.q2_proj, self.k_proj, self.v_proj):
            nn.init.normal_(p.weight, mean=0.0, std=0.02)
        nn.init.normal_(self.o_proj.weight, mean=0.0, std=0.02)
        if use_state_injection:
            for seq in (self.state_k_proj, self.state_v_proj):
                for m in seq:
                    if isinstance(m, nn.Linear):
                        nn.init.normal_(m.weight, mean=0.0, std=0.01)
            nn.init.normal_(self.h_state_k_proj.weight, mean=0.0, std=0.01)
            nn.init.normal_(self.h_state_v_proj.weight, mean=0.0, std=0.01)

    def _compute_state_injection(self, h_states: torch.Tensor, proj: nn.Module) -> torch.Tensor:
        return proj(state_injection_input(h_states, self.state_injection_dim))

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                use_cache: bool = False, cache: Optional[dict] = None,
                ssm_state: Optional[torch.Tensor] = None, h_states: Optional[torch.Tensor] = None,
                rope_offset: int = 0):
        B, S, _ = x.shape
        H, G, hd = self.n_heads, self.n_kv_heads, self.head_dim
        q1 = self.q1_proj(x).view(B, S, H, hd)
        q2 = self.q2_proj(x).view(B, S, H, hd)
        k = self.k_proj(x)
        v = self.v_proj(x)
        if self.use_state_injection:
            if h_states is not None:
                hin = state_injection_input(h_states, self.state_injection_dim).to(k.dtype)
                k = k + self.h_state_k_proj(hin)
                v = v + self.h_state_v_proj(hin)
            elif ssm_state is not None:
                summ = ssm_state.mean(dim=-1).to(x.dtype)
                if summ.shape[-1] < self.d_model:
                    summ = F.pad(summ, (0, self.d_model - summ.shape[-1]))
                else:
                    summ = summ[..., : self.d_model]
                k = k + self.state_k_proj(summ).unsqueeze(1)
                v = v + self.state_v_proj(summ).unsqueeze(1)
        k, v = k.view(B, S, G, hd), v.view(B, S, G, hd)
        cos, sin = self.rope(S, x.device, rope_offset)
        c, s = cos[0, 0, :, : hd // 2], sin[0, 0, :, : hd // 2]
        q1, q2, k = ops.rope(q1, c, s), ops.rope(q2, c, s), ops.rope(k, c, s)
        if use_cache and cache is not None:
            k = torch.cat([cache["k"], k], dim=1)
            v = torch.cat([cache["v"], v], dim=1)
        new_cache = {"k": k, "v": v} if use_cache else None
        out = ops.diff_attention(q1, q2, k, v, _lambda(self.lambda_raw), window=self.sliding_window,
                                 window_mode=self.window_mode, attention_mask=attention_mask)
        flat = out.reshape(B, S, -1)
        normed = ops.head_group_norm(flat, H, self.group_norm.weight, self.group_norm.bias,
                                     self.group_norm.eps)
        return self.o_proj(normed), new_cache

    def get_lambda_values(self) -> torch.Tensor:
        return torch.sigmoid(self.lambda_raw).detach()
