"""Diagonal selective-SSM block ("Mamba2Block" in the reference API).

Reference: ``mamformer/layers/mamba2.py``.  Semantics kept exactly:

* ``xz = in_proj(u)``; ``x, z = split``; depthwise causal conv (k=d_conv, no bias) + SiLU;
* ``dt = softplus(W2 (W1 x))`` (dt_rank = ceil(d_model/32), no biases); ``B = W_B x``;
  ``C = W_C x``;
* ``h_t = exp(-exp(clamp(A_log,-5,5)) dt_t) * h_{t-1} + B_t dt_t x_t`` with the decay per
  (channel, state) - a Mamba-1-style diagonal scan, *not* scalar-decay SSD;
* ``y = (C_t . h_t + D x_t) * silu(z_t)``; ``out = out_proj(y)``;
* ``h_states[t] = mean_channels(h_t)`` (B, S, d_state), fed to attention K/V injection;
* decode: conv state = last d_conv-1 raw inputs, SSM state = h_T; the single-step recurrence
  uses the *unclamped* ``exp(A_log)`` (reference ``mamba2.py:441-443``) and, like the
  reference, only the last input position.

On CUDA the conv+SiLU and the scan (softplus, decay, D skip, SiLU(z) gate, h_states mean) run
in native kernels; the scan keeps its state in registers and saves chunk states for the
backward recompute.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamformer_b200 import ops
from mamformer_b200.ops import reference as ref


def selective_scan(x, dt, A, B, C, D, return_h_states: bool = False,
                   return_final_state: bool = False):
    """Functional selective scan with the reference signature (``mamba2.py:31-67``).

    ``A`` is the log-parameter ``A_log``.  Differentiable; native on CUDA."""
    return ops.selective_scan(x, dt, A, B, C, D, return_h_states, return_final_state)


class Mamba2Block(nn.Module):
    def __init__(self, d_model: int, d_state: int = 128, d_conv: int = 4, expand: int = 1,
                 dt_rank: Optional[int] = None, bias: bool = False,
                 use_compile: bool = False) -> None:
        super().__init__()
        self.d_model = d_model
        self.d_inner = d_model * expand
        self.d_state = d_state
        self.d_conv = d_conv
        self.dt_rank = dt_rank if dt_rank is not None else math.ceil(d_model / 32)
        self.in_proj = nn.Linear(d_model, 2 * self.d_inner, bias=bias)
        self.conv1d = nn.Conv1d(self.d_inner, self.d_inner, d_conv, groups=self.d_inner,
                                padding=0, bias=bias)
        self.dt_proj = nn.Sequential(nn.Linear(self.d_inner, self.dt_rank, bias=bias),
                                     nn.Linear(self.dt_rank, self.d_inner, bias=bias))
        self.B_proj = nn.Linear(self.d_inner, d_state, bias=bias)
        self.C_proj = nn.Linear(self.d_inner, d_state, bias=bias)
        self.A_log = nn.Parameter(torch.log(torch.linspace(0.5, 8, d_state)))
        self.D = nn.Parameter(torch.ones(self.d_inner))
        self.out_proj = nn.Linear(self.d_inner, d_model, bias=bias)
        nn.init.normal_(self.in_proj.weight, mean=0.0, std=0.02)
        nn.init.normal_(self.out_proj.weight, mean=0.0, std=0.02)
        for lin in self.dt_proj:
            nn.init.normal_(lin.weight, mean=0.0, std=0.001)
        nn.init.normal_(self.B_proj.weight, mean=0.0, std=0.02)
        nn.init.normal_(self.C_proj.weight, mean=0.0, std=0.02)
        nn.init.normal_(self.conv1d.weight, mean=0.0, std=0.02)

    # -- helpers ---------------------------------------------------------------------------
    def _conv_weight(self) -> torch.Tensor:
        return self.conv1d.weight.view(self.d_inner, self.d_conv)

    def _dbc(self, x_act: torch.Tensor):
        dt_raw = self.dt_proj[1](self.dt_proj[0](x_act))
        return dt_raw, self.B_proj(x_act), self.C_proj(x_act)

    def forward(self, u: torch.Tensor, use_cache: bool = False, cache: Optional[dict] = None,
                return_h_states: bool = False):
        Bsz, S, _ = u.shape
        xz = self.in_proj(u)
        x, z = xz.chunk(2, dim=-1)
        raw_x = x
        conv_state = cache.get("conv_state") if (use_cache and cache is not None) else None
        incremental = use_cache and cache is not None and cache.get("ssm_state") is not None
        if conv_state is not None:
            x_act = F.silu(ref.causal_conv1d(x, self._conv_weight(), conv_state))
        else:
            x_act = ops.causal_conv1d_silu(x, self._conv_weight())
        dt_raw, Bm, Cm = self._dbc(x_act)
        h_states = None
        if incremental:
            y, final = self._recurrent_step(x_act, F.softplus(dt_raw), Bm, Cm, cache["ssm_state"])
            y = y * F.silu(z)
        else:
            y, h_states, final = ops.mamba_inner(x_act, dt_raw, self.A_log, Bm, Cm, self.D, z,
                                                 need_h_states=return_h_states,
                                                 return_final=use_cache)
            if h_states is not None and getattr(self, "tp_group", None) is not None:
                from mamformer_b200.parallel.tensor_parallel import mean_from_tp
                h_states = mean_from_tp(h_states, self.tp_group)   # channel mean over all TP shards
        out = self.out_proj(y)
        new_cache = None
        if use_cache:
            cx = raw_x[:, -(self.d_conv - 1):] if raw_x.shape[1] >= self.d_conv else raw_x
            if cache is not None and "conv_state" in cache:
                cx = torch.cat([cache["conv_state"], cx], 1)[:, -(self.d_conv - 1):]
            new_cache = {"conv_state": cx, "ssm_state": final}
        if return_h_states:
            return out, new_cache, h_states
        return out, new_cache

    def _causal_conv1d(self, x: torch.Tensor, cache: Optional[dict] = None) -> torch.Tensor:
        state = cache.get("conv_state") if cache is not None else None
        return ref.causal_conv1d(x, self._conv_weight(), state)

    def _recurrent_step(self, x, dt, B, C, h_prev):
        """Last-position recurrence with the unclamped decay (reference ``mamba2.py:407-458``)."""
        xt, dtt, Bt, Ct = x[:, -1], dt[:, -1], B[:, -1], C[:, -1]
        a = torch.exp(-torch.exp(self.A_log.float()).unsqueeze(0) * dtt.float().unsqueeze(-1))
        if h_prev is None:
            h_prev = torch.zeros(x.shape[0], self.d_inner, self.d_state, device=x.device,
                                 dtype=torch.float32)
        h = a * h_prev.float() + (Bt.float().unsqueeze(1) * dtt.float().unsqueeze(-1)) * xt.float().unsqueeze(-1)
        y = (Ct.float().unsqueeze(1) * h).sum(-1) + self.D.float() * xt.float()
        return y.to(x.dtype).unsqueeze(1), h.to(h_prev.dtype if h_prev.dtype != torch.float32 else torch.float32)

    def extra_repr(self) -> str:
        return (f"d_model={self.d_model}, d_inner={self.d_inner}, d_state={self.d_state}, "
                f"d_conv={self.d_conv}")
