"""Hybrid block: attention-only, SSM-only or fusion (reference ``layers/hybrid.py:49-602``).

* fusion:    ``x + sigmoid(gate_alpha) * attn(n x) + (1 - sigmoid(gate_alpha)) * ssm(n x)``; the
             attention (DSA / KDA-Diff) receives the same layer's SSM ``h_states``;
* attn-only: ``x + attn(n x, h_states from the preceding SSM-only layer)``;
* SSM-only:  ``x + ssm(n x)``; emits ``h_states`` for the next attention-only layer;
* then ``x + FFN(post_norm x)`` with SwiGLU, DeepSeekMoE, SpaceTimeMoE or CommunicativeMoE.

``h_states_needed`` (set by ``MamformerModel``) lets an SSM-only layer skip the channel-mean
reduction when no attention layer will read its state; outputs are unchanged.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from mamformer_b200.models.attention import GroupedQueryAttention
from mamformer_b200.models.dsa import DifferentialStateAttention
from mamformer_b200.models.ffn import SwiGLUFFN
from mamformer_b200.models.kda_diff import KDADiffAttention
from mamformer_b200.models.mamba2 import Mamba2Block
from mamformer_b200.models.math_opt import DynamicGate
from mamformer_b200.models.moe import DeepSeekMoE
from mamformer_b200.models.norm import RMSNorm


class MamformerBlock(nn.Module):
    def __init__(self, d_model: int = 4096, n_heads: int = 32, n_kv_heads: int = 8,
                 head_dim: int = 128, d_ff: int = 9216, d_state: int = 128, d_conv: int = 4,
                 mamba_expand: int = 1, max_seq_len: int = 8192, rope_theta: float = 10000.0,
                 dropout: float = 0.0, rms_norm_eps: float = 1e-6, sliding_window: int = 0,
                 has_attention: bool = True, has_ssm: bool = True, layer_idx: int = 0,
                 use_dsa: bool = False, dsa_lambda_init: float = 0.8, dsa_state_injection: bool = True,
                 rope_use_yarn: bool = False, rope_yarn_scale: float = 1.0,
                 rope_yarn_original_max_seq_len: int = 8192,
                 use_moe: bool = False, moe_n_shared: int = 2, moe_n_routed: int = 64,
                 moe_top_k: int = 8, moe_shared_dim: int = 2304, moe_routed_dim: int = 576,
                 moe_aux_loss_free: bool = True, moe_bias_speed: float = 0.001,
                 moe_router_temperature: float = 1.0,
                 use_st_moe: bool = False, st_moe_lambda_init: float = 0.2, st_moe_lambda_max: float = 0.3,
                 st_moe_learnable_lambda: bool = True, st_moe_use_balance_lock: bool = True,
                 st_moe_balance_lock_threshold: int = 50,
                 use_communicative_moe: bool = False, comm_moe_n_heads: int = 4,
                 comm_moe_depth: int = 1, comm_moe_dropout: float = 0.0,
                 use_kda_diff: bool = False, kda_linear_ratio: int = 3, kda_kernel_dim: int = 128,
                 kda_latent_dim: int = 512, kda_use_dynamic_ratio: bool = True,
                 use_dynamic_gate: bool = False, dynamic_gate_bottleneck: int = 0,
                 use_deepnorm: bool = False, deepnorm_n_layers: int = 52,
                 window_mode: str = "reference") -> None:
        super().__init__()
        self.d_model = d_model
        self.sliding_window = sliding_window
        self.has_attention = has_attention
        self.has_ssm = has_ssm
        self.is_fusion = has_attention and has_ssm
        self.layer_idx = layer_idx
        self.use_dsa = use_dsa and has_attention
        self.use_kda_diff = use_kda_diff and has_attention
        self.use_moe = use_moe
        self.use_st_moe = use_st_moe
        self.use_dynamic_gate = use_dynamic_gate and has_attention
        self.use_deepnorm = use_deepnorm
        self.h_states_needed = True
        if use_deepnorm:
            self.register_buffer("deepnorm_alpha", torch.tensor((2.0 * deepnorm_n_layers) ** (-0.25)))
        else:
            self.deepnorm_alpha = None
        rope_kw = dict(max_seq_len=max_seq_len, rope_theta=rope_theta, use_yarn=rope_use_yarn,
                       yarn_scale=rope_yarn_scale, yarn_original_max_seq_len=rope_yarn_original_max_seq_len)
        self.input_norm = RMSNorm(d_model, eps=rms_norm_eps)
        if has_attention:
            if use_kda_diff:
                self.attention = KDADiffAttention(
                    d_model, n_heads, n_kv_heads, head_dim, kda_linear_ratio, kda_kernel_dim,
                    kda_latent_dim, lambda_init=dsa_lambda_init, use_state_injection=dsa_state_injection,
                    state_injection_dim=64, use_dynamic_ratio=kda_use_dynamic_ratio, d_state=d_state,
                    dropout=dropout, sliding_window=sliding_window, window_mode=window_mode, **rope_kw)
                self.attention.set_layer_idx(layer_idx)
            elif use_dsa:
                self.attention = DifferentialStateAttention(
                    d_model, n_heads, n_kv_heads, head_dim, lambda_init=dsa_lambda_init,
                    use_state_injection=dsa_state_injection, dropout=dropout,
                    sliding_window=sliding_window, window_mode=window_mode, **rope_kw)
            else:
                self.attention = GroupedQueryAttention(
                    d_model, n_heads, n_kv_heads, head_dim, dropout=dropout,
                    sliding_window=sliding_window, window_mode=window_mode, **_gqa_rope(rope_kw))
        else:
            self.attention = None
        self.ssm = Mamba2Block(d_model, d_state, d_conv, mamba_expand) if has_ssm else None
        if self.is_fusion:
            if use_dynamic_gate:
                self.gate_alpha = None
                self.dynamic_gate = DynamicGate(d_model, dynamic_gate_bottleneck)
            else:
                self.gate_alpha = nn.Parameter(torch.zeros(d_model))
                self.dynamic_gate = None
        else:
            self.gate_alpha = None
            self.dynamic_gate = None
        self.post_norm = RMSNorm(d_model, eps=rms_norm_eps)
        base = None
        if use_st_moe:
            from mamformer_b200.models.st_moe import SpaceTimeMoE
            base = SpaceTimeMoE(d_model, moe_n_shared, moe_shared_dim, moe_n_routed, moe_top_k,
                                moe_routed_dim, d_state, st_moe_lambda_init, st_moe_lambda_max,
                                st_moe_learnable_lambda, st_moe_use_balance_lock,
                                st_moe_balance_lock_threshold, moe_router_temperature,
                                moe_aux_loss_free, moe_bias_speed, dropout)
        elif use_moe:
            base = DeepSeekMoE(d_model, moe_n_shared, moe_shared_dim, moe_n_routed, moe_top_k,
                               moe_routed_dim, moe_router_temperature, moe_aux_loss_free,
                               moe_bias_speed, dropout)
        if use_communicative_moe and base is not None:
            from mamformer_b200.models.communicative_moe import CommunicativeMoE
            self.ffn = CommunicativeMoE(base, d_model, comm_moe_n_heads, comm_moe_depth, comm_moe_dropout)
        elif base is not None:
            self.ffn = base
        else:
            self.ffn = SwiGLUFFN(d_model, d_ff, dropout)

    # -------------------------------------------------------------------------------------
    def _residual(self, residual: torch.Tensor, update: torch.Tensor) -> torch.Tensor:
        if self.deepnorm_alpha is not None:
            return self.deepnorm_alpha.to(residual.dtype) * residual + update
        return residual + update

    def _ffn(self, x: torch.Tensor, st_h: Optional[torch.Tensor]):
        if self.use_st_moe:
            return self.ffn(x, ssm_h_states=st_h)
        if self.use_moe:
            return self.ffn(x)
        return self.ffn(x), None

    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                use_cache: bool = False, cache: Optional[dict] = None,
                ssm_h_states: Optional[torch.Tensor] = None, rope_offset: int = 0):
        residual = hidden_states
        h = self.input_norm(hidden_states)
        ssm_out = ssm_cache = local_h = None
        if self.has_ssm:
            want_h = ((self.is_fusion and (self.use_dsa or self.use_kda_diff or self.use_st_moe))
                      or (not self.has_attention and (self.h_states_needed or self.use_st_moe)))
            ssm_prev = cache.get("ssm") if cache is not None else None
            if want_h:
                ssm_out, ssm_cache, local_h = self.ssm(h, use_cache=use_cache, cache=ssm_prev,
                                                       return_h_states=True)
            else:
                ssm_out, ssm_cache = self.ssm(h, use_cache=use_cache, cache=ssm_prev)

        if not self.has_attention:
            x = self._residual(residual, ssm_out)
            ffn_out, aux = self._ffn(self.post_norm(x), local_h)
            x = x + ffn_out
            new_cache = None
            if use_cache:
                new_cache = {"ssm": ssm_cache}
                if aux is not None:
                    new_cache["moe_aux_info"] = aux
            if local_h is not None:
                new_cache = new_cache if new_cache is not None else {}
                new_cache["ssm_h_states"] = local_h
            if aux is not None and not use_cache:
                new_cache = new_cache if new_cache is not None else {}
                new_cache["moe_aux_info"] = aux
            return x, new_cache

        attn_kw = {}
        if self.is_fusion and local_h is not None:
            attn_kw["h_states"] = local_h
        elif not self.has_ssm and ssm_h_states is not None:
            attn_kw["h_states"] = ssm_h_states
        if rope_offset:
            attn_kw["rope_offset"] = rope_offset
        attn_prev = cache.get("attn") if cache is not None else None
        attn_out, attn_cache = self.attention(h, attention_mask=attention_mask, use_cache=use_cache,
                                              cache=attn_prev, **attn_kw)
        if not self.has_ssm:
            x = self._residual(residual, attn_out)
            st_h = ssm_h_states if self.use_st_moe else None
            ffn_out, aux = self._ffn(self.post_norm(x), st_h)
            x = x + ffn_out
            new_cache = None
            if use_cache:
                new_cache = {"attn": attn_cache}
            if aux is not None:
                new_cache = new_cache if new_cache is not None else {}
                new_cache["moe_aux_info"] = aux
            return x, new_cache

        gate = self.dynamic_gate(h) if self.dynamic_gate is not None else torch.sigmoid(self.gate_alpha)
        gate = gate.to(attn_out.dtype)
        x = self._residual(residual, gate * attn_out + (1.0 - gate) * ssm_out)
        ffn_out, aux = self._ffn(self.post_norm(x), local_h)
        x = x + ffn_out
        new_cache = None
        if use_cache:
            new_cache = {"attn": attn_cache, "ssm": ssm_cache}
        if aux is not None:
            new_cache = new_cache if new_cache is not None else {}
            new_cache["moe_aux_info"] = aux
        return x, new_cache

    def get_gate_values(self) -> Optional[torch.Tensor]:
        return None if self.gate_alpha is None else torch.sigmoid(self.gate_alpha).detach()

    def get_moe_load_statistics(self) -> Optional[dict]:
        if (self.use_moe or self.use_st_moe) and hasattr(self.ffn, "get_load_statistics"):
            return self.ffn.get_load_statistics()
        return None

    def extra_repr(self) -> str:
        mode = "fusion (parallel)" if self.is_fusion else (
            "attention-only (cross-layer)" if self.has_attention else "SSM-only")
        ffn = "ST-MoE" if self.use_st_moe else ("MoE" if self.use_moe else "SwiGLU")
        if hasattr(self, "ffn") and hasattr(self.ffn, "comm_layer"):
            ffn = f"Communicative{ffn}"
        parts = [f"d_model={self.d_model}", f"mode={mode}", f"ffn={ffn}"]
        if self.has_attention:
            parts.append("attn=" + ("KDA-Diff" if self.use_kda_diff else ("DSA" if self.use_dsa else "GQA")))
        if self.ssm is not None:
            parts += [f"d_state={self.ssm.d_state}", f"d_conv={self.ssm.d_conv}"]
        return ", ".join(parts)


def _gqa_rope(rope_kw: dict) -> dict:
    return dict(max_seq_len=rope_kw["max_seq_len"], rope_theta=rope_kw["rope_theta"],
                use_yarn=rope_kw["use_yarn"], yarn_scale=rope_kw["yarn_scale"],
                yarn_original_max_seq_len=rope_kw["yarn_original_max_seq_len"])
