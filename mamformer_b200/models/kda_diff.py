"""KDA-Diff: kernelised differential attention with SSM-driven interleaving.

Reference: ``mamformer/layers/kda_diff.py``.

* ``LinearDiffAttention`` (``kda_diff.py:96-632``): q1, q2, k, v projections; SSM-state
  injection ``k += W_k h[..., :64]``, ``v += W_v h[..., :64]`` (zero-padded when d_state < 64);
  RoPE on q1, q2, k; causal linear attention with phi = elu+1 on the first ``kernel_dim``
  dims and normaliser ``phi(q).z + 1e-8``; ``(o1 - lam o2) / (1 - lam + 1e-8)`` with
  ``lam = min(sigmoid(lambda_raw), 0.99)``; GroupNorm(H groups over hd x S); o_proj.
  Decode keeps the O(1) state ``S (B,H,K,hd)``, ``z (B,H,K,1)``.
* ``FullDiffAttention`` (``kda_diff.py:639-898``): MLA-style ``k = k_expand(k_compress(x))``,
  same for v, injection, RoPE, two softmaxes with a causal (finfo.min) mask, differential
  combine, GroupNorm, o_proj.  The KV cache holds the expanded k, v.
* ``DynamicInterleaveGate`` (``kda_diff.py:905-958``): ``sigmoid(MLP(h_states))``.
* ``KDADiffAttention`` (``kda_diff.py:965-1170``): full attention iff the mean gate > 0.5 when
  h_states is present and dynamic mode is on (a host sync, as in the reference), else iff
  ``(attn_layer_idx + 1) % (linear_ratio + 1) == 0``.

On CUDA the attention cores run in native kernels: the chunked linear scan and the
differential flash-attention kernel; GroupNorm runs in the native two-pass head-norm kernel.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamformer_b200 import ops
from mamformer_b200.models.rope import RotaryEmbedding


def kernel_feature_map(x: torch.Tensor, kernel_dim: int = 128) -> torch.Tensor:
    """phi(x) = elu(x[..., :kernel_dim]) + 1 (always positive)."""
    return F.elu(x[..., :kernel_dim]) + 1.0


def _lambda(lambda_raw: torch.Tensor) -> torch.Tensor:
    return torch.sigmoid(lambda_raw).clamp(max=0.99)


def _logit(p: float) -> float:
    return math.log(p / (1.0 - p)) if 0.0 < p < 1.0 else 0.0


def state_injection_input(h_states: torch.Tensor, dim: int) -> torch.Tensor:
    """Zero-pad or truncate the last dim of h_states to ``dim`` (reference ``kda_diff.py:607-618``)."""
    n = h_states.shape[-1]
    if n < dim:
        return F.pad(h_states, (0, dim - n))
    return h_states[..., :dim]


class _DiffHeadNormMixin:
    def _norm_and_project(self, out_bshd: torch.Tensor) -> torch.Tensor:
        B, S = out_bshd.shape[:2]
        flat = out_bshd.reshape(B, S, -1)
        normed = ops.head_group_norm(flat, self.n_heads, self.group_norm.weight,
                                     self.group_norm.bias, self.group_norm.eps)
        return self.o_proj(normed)


class LinearDiffAttention(_DiffHeadNormMixin, nn.Module):
    def __init__(self, d_model: int, n_heads: int = 32, n_kv_heads: int = 8, head_dim: int = 128,
                 kernel_dim: int = 128, lambda_init: float = 0.8, max_seq_len: int = 8192,
                 rope_theta: float = 10000.0, use_state_injection: bool = True,
                 state_injection_dim: int = 64, dropout: float = 0.0, use_yarn: bool = False,
                 yarn_scale: float = 1.0, yarn_original_max_seq_len: int = 8192,
                 use_triton: bool = True, use_compile: bool = False,
                 scan_chunk_size: int = 256) -> None:
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.kernel_dim = min(kernel_dim, head_dim)
        self.n_head_groups = n_heads // n_kv_heads
        self.use_state_injection = use_state_injection
        self.state_injection_dim = state_injection_dim
        self.scan_chunk_size = scan_chunk_size
        self.q1_proj = nn.Linear(d_model, n_heads * head_dim, bias=False)
        self.q2_proj = nn.Linear(d_model, n_heads * head_dim, bias=False)
        self.k_proj = nn.Linear(d_model, n_kv_heads * head_dim, bias=False)
        self.v_proj = nn.Linear(d_model, n_kv_heads * head_dim, bias=False)
        self.o_proj = nn.Linear(n_heads * head_dim, d_model, bias=False)
        self.lambda_raw = nn.Parameter(torch.full((n_heads,), _logit(lambda_init)))
        if use_state_injection:
            self.h_state_k_proj = nn.Linear(state_injection_dim, n_kv_heads * head_dim, bias=False)
            self.h_state_v_proj = nn.Linear(state_injection_dim, n_kv_heads * head_dim, bias=False)
        self.rope = RotaryEmbedding(head_dim, max_seq_len, rope_theta, use_yarn, yarn_scale,
                                    yarn_original_max_seq_len)
        self.group_norm = nn.GroupNorm(n_heads, n_heads * head_dim, eps=1e-6)
        for p in (self.q1_proj, self.q2_proj, self.k_proj, self.v_proj, self.o_proj):
            nn.init.normal_(p.weight, mean=0.0, std=0.02)
        if use_state_injection:
            nn.init.normal_(self.h_state_k_proj.weight, mean=0.0, std=0.01)
            nn.init.normal_(self.h_state_v_proj.weight, mean=0.0, std=0.01)

    def _project(self, x, h_states, rope_offset):
        B, S, _ = x.shape
        q1 = self.q1_proj(x)
        q2 = self.q2_proj(x)
        k = self.k_proj(x)
        v = self.v_proj(x)
        if self.use_state_injection and h_states is not None:
            hin = state_injection_input(h_states, self.state_injection_dim).to(k.dtype)
            k = k + self.h_state_k_proj(hin)
            v = v + self.h_state_v_proj(hin)
        H, G, hd = self.n_heads, self.n_kv_heads, self.head_dim
        q1, q2 = q1.view(B, S, H, hd), q2.view(B, S, H, hd)
        k, v = k.view(B, S, G, hd), v.view(B, S, G, hd)
        cos, sin = self.rope(S, x.device, rope_offset)
        c, s = cos[0, 0, :, : hd // 2], sin[0, 0, :, : hd // 2]
        return ops.rope(q1, c, s), ops.rope(q2, c, s), ops.rope(k, c, s), v

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                use_cache: bool = False, cache: Optional[dict] = None,
                h_states: Optional[torch.Tensor] = None, rope_offset: int = 0):
        B, S, _ = x.shape
        q1, q2, k, v = self._project(x, h_states, rope_offset)
        lam = _lambda(self.lambda_raw)
        H, K, hd = self.n_heads, self.kernel_dim, self.head_dim
        has_prev = use_cache and cache is not None and cache.get("attn_type") == "linear"
        if has_prev:
            S_prev, z_prev = cache["S"], cache["z"]
        else:
            S_prev = torch.zeros(B, H, K, hd, device=x.device, dtype=x.dtype)
            z_prev = torch.zeros(B, H, K, 1, device=x.device, dtype=x.dtype)
        if S == 1 and use_cache:
            out = self._recurrent(q1, q2, k, v, S_prev, z_prev, lam)
        else:
            out = ops.linear_diff_attention(q1, q2, k, v, lam, K, self.scan_chunk_size)
        new_cache = None
        if use_cache:
            kx = k.repeat_interleave(self.n_head_groups, dim=2) if self.n_head_groups > 1 else k
            vx = v.repeat_interleave(self.n_head_groups, dim=2) if self.n_head_groups > 1 else v
            pk = kernel_feature_map(kx, K).transpose(1, 2)           # (B, H, S, K)
            S_new = torch.matmul(pk.transpose(-2, -1), vx.transpose(1, 2))
            z_new = pk.transpose(-2, -1).sum(-1, keepdim=True)
            new_cache = {"S": S_prev + S_new.to(S_prev.dtype), "z": z_prev + z_new.to(z_prev.dtype),
                         "attn_type": "linear"}
        return self._norm_and_project(out), new_cache

    def _recurrent(self, q1, q2, k, v, S_prev, z_prev, lam):
        """One decode step: update (S, z) with the new token, then read with both queries."""
        g = self.n_head_groups
        kx = k.repeat_interleave(g, dim=2) if g > 1 else k
        vx = v.repeat_interleave(g, dim=2) if g > 1 else v
        K = self.kernel_dim
        pk = kernel_feature_map(kx, K).transpose(1, 2)       # (B, H, 1, K)
        Sx = S_prev + torch.matmul(pk.transpose(-2, -1), vx.transpose(1, 2))
        zx = z_prev + pk.transpose(-2, -1)
        outs = []
        for q in (q1, q2):
            pq = kernel_feature_map(q, K).transpose(1, 2)    # (B, H, 1, K)
            outs.append(torch.matmul(pq, Sx) / (torch.matmul(pq, zx) + 1e-8))
        lam4 = lam.view(1, -1, 1, 1).to(outs[0].dtype)
        return ((outs[0] - lam4 * outs[1]) / (1.0 - lam4 + 1e-8)).transpose(1, 2)

    def _compute_state_injection(self, h_states: torch.Tensor, proj: nn.Linear) -> torch.Tensor:
        return proj(state_injection_input(h_states, self.state_injection_dim))

    def get_lambda_values(self) -> torch.Tensor:
        return torch.sigmoid(self.lambda_raw).detach()

    def extra_repr(self) -> str:
        si = ", state_injection" if self.use_state_injection else ""
        return (f"d_model={self.d_model}, n_heads={self.n_heads}, n_kv_heads={self.n_kv_heads}, "
                f"head_dim={self.head_dim}, kernel_dim={self.kernel_dim}{si}, chunked-scan")


class FullDiffAttention(_DiffHeadNormMixin, nn.Module):
    def __init__(self, d_model: int, n_heads: int = 32, n_kv_heads: int = 8, head_dim: int = 128,
                 latent_dim: int = 512, lambda_init: float = 0.8, max_seq_len: int = 8192,
                 rope_theta: float = 10000.0, use_state_injection: bool = True,
                 state_injection_dim: int = 64, dropout: float = 0.0, sliding_window: int = 0,
                 use_yarn: bool = False, yarn_scale: float = 1.0,
                 yarn_original_max_seq_len: int = 8192, window_mode: str = "reference") -> None:
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.n_head_groups = n_heads // n_kv_heads
        self.latent_dim = latent_dim
        self.sliding_window = sliding_window
        self.window_mode = window_mode
        self.use_state_injection = use_state_injection
        self.state_injection_dim = state_injection_dim
        kv_dim = n_kv_heads * head_dim
        self.q1_proj = nn.Linear(d_model, n_heads * head_dim, bias=False)
        self.q2_proj = nn.Linear(d_model, n_heads * head_dim, bias=False)
        self.k_compress = nn.Linear(d_model, latent_dim, bias=False)
        self.k_expand = nn.Linear(latent_dim, kv_dim, bias=False)
        self.v_compress = nn.Linear(d_model, latent_dim, bias=False)
        self.v_expand = nn.Linear(latent_dim, kv_dim, bias=False)
        self.o_proj = nn.Linear(n_heads * head_dim, d_model, bias=False)
        self.lambda_raw = nn.Parameter(torch.full((n_heads,), _logit(lambda_init)))
        if use_state_injection:
            self.h_state_k_proj = nn.Linear(state_injection_dim, kv_dim, bias=False)
            self.h_state_v_proj = nn.Linear(state_injection_dim, kv_dim, bias=False)
        self.rope = RotaryEmbedding(head_dim, max_seq_len, rope_theta, use_yarn, yarn_scale,
                                    yarn_original_max_seq_len)
        self.group_norm = nn.GroupNorm(n_heads, n_heads * head_dim, eps=1e-6)
        for p in (self.q1_proj, self.q2_proj, self.o_proj):
            nn.init.normal_(p.weight, mean=0.0, std=0.02)
        for p in (self.k_compress, self.k_expand, self.v_compress, self.v_expand):
            nn.init.normal_(p.weight, mean=0.0, std=0.01)
        if use_state_injection:
            nn.init.normal_(self.h_state_k_proj.weight, mean=0.0, std=0.01)
            nn.init.normal_(self.h_state_v_proj.weight, mean=0.0, std=0.01)

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                use_cache: bool = False, cache: Optional[dict] = None,
                h_states: Optional[torch.Tensor] = None, rope_offset: int = 0):
        B, S, _ = x.shape
        H, G, hd = self.n_heads, self.n_kv_heads, self.head_dim
        q1 = self.q1_proj(x).view(B, S, H, hd)
        q2 = self.q2_proj(x).view(B, S, H, hd)
        k = self.k_expand(self.k_compress(x))
        v = self.v_expand(self.v_compress(x))
        if self.use_state_injection and h_states is not None:
            hin = state_injection_input(h_states, self.state_injection_dim).to(k.dtype)
            k = k + self.h_state_k_proj(hin)
            v = v + self.h_state_v_proj(hin)
        k, v = k.view(B, S, G, hd), v.view(B, S, G, hd)
        cos, sin = self.rope(S, x.device, rope_offset)
        c, s = cos[0, 0, :, : hd // 2], sin[0, 0, :, : hd // 2]
        q1, q2, k = ops.rope(q1, c, s), ops.rope(q2, c, s), ops.rope(k, c, s)
        if use_cache and cache is not None and cache.get("attn_type") == "full":
            k = torch.cat([cache["k"], k], dim=1)
            v = torch.cat([cache["v"], v], dim=1)
        new_cache = {"k": k, "v": v, "attn_type": "full"} if use_cache else None
        out = ops.diff_attention(q1, q2, k, v, _lambda(self.lambda_raw), window=self.sliding_window,
                                 window_mode=self.window_mode, attention_mask=attention_mask)
        return self._norm_and_project(out), new_cache

    def get_lambda_values(self) -> torch.Tensor:
        return torch.sigmoid(self.lambda_raw).detach()

    def extra_repr(self) -> str:
        sw = f", sliding_window={self.sliding_window}" if self.sliding_window > 0 else ""
        si = ", state_injection" if self.use_state_injection else ""
        return (f"d_model={self.d_model}, n_heads={self.n_heads}, n_kv_heads={self.n_kv_heads}, "
                f"head_dim={self.head_dim}, latent_dim={self.latent_dim}{sw}{si}")


class DynamicInterleaveGate(nn.Module):
    """ratio = sigmoid(W2 silu(W1 h) + b2) per token; W1: d_state->64 (no bias)."""

    def __init__(self, d_state: int = 128, bottleneck: int = 64):
        super().__init__()
        self.d_state = d_state
        self.mlp = nn.Sequential(nn.Linear(d_state, bottleneck, bias=False), nn.SiLU(),
                                 nn.Linear(bottleneck, 1, bias=True))
        nn.init.normal_(self.mlp[0].weight, mean=0.0, std=0.02)
        nn.init.normal_(self.mlp[2].weight, mean=0.0, std=0.02)
        nn.init.zeros_(self.mlp[2].bias)

    def forward(self, ssm_h_states: torch.Tensor) -> torch.Tensor:
        h = ssm_h_states.to(self.mlp[0].weight.dtype)
        return torch.sigmoid(self.mlp(h))

    def extra_repr(self) -> str:
        return f"d_state={self.d_state}"


class KDADiffAttention(nn.Module):
    def __init__(self, d_model: int, n_heads: int = 32, n_kv_heads: int = 8, head_dim: int = 128,
                 linear_ratio: int = 3, kernel_dim: int = 128, latent_dim: int = 512,
                 lambda_init: float = 0.8, max_seq_len: int = 8192, rope_theta: float = 10000.0,
                 use_state_injection: bool = True, state_injection_dim: int = 64,
                 use_dynamic_ratio: bool = True, d_state: int = 128, dropout: float = 0.0,
                 sliding_window: int = 0, use_yarn: bool = False, yarn_scale: float = 1.0,
                 yarn_original_max_seq_len: int = 8192, use_triton: bool = True,
                 use_compile: bool = False, scan_chunk_size: int = 256,
                 window_mode: str = "reference") -> None:
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.linear_ratio = linear_ratio
        self.use_dynamic_ratio = use_dynamic_ratio
        rope_kw = dict(max_seq_len=max_seq_len, rope_theta=rope_theta, use_yarn=use_yarn,
                       yarn_scale=yarn_scale, yarn_original_max_seq_len=yarn_original_max_seq_len)
        self.linear_attn = LinearDiffAttention(
            d_model, n_heads, n_kv_heads, head_dim, kernel_dim, lambda_init,
            use_state_injection=use_state_injection, state_injection_dim=state_injection_dim,
            dropout=dropout, scan_chunk_size=scan_chunk_size, **rope_kw)
        self.full_attn = FullDiffAttention(
            d_model, n_heads, n_kv_heads, head_dim, latent_dim, lambda_init,
            use_state_injection=use_state_injection, state_injection_dim=state_injection_dim,
            dropout=dropout, sliding_window=sliding_window, window_mode=window_mode, **rope_kw)
        self.interleave_gate = DynamicInterleaveGate(d_state=d_state) if use_dynamic_ratio else None
        self.output_mix = nn.Parameter(torch.zeros(1))
        self.register_buffer("layer_idx", torch.tensor(0, dtype=torch.long))
        self.register_buffer("attn_layer_idx", torch.tensor(-1, dtype=torch.long))
        # Host-side copies of the two indices: the fixed-pattern decision needs no device sync.
        self._layer_idx_host = 0
        self._attn_idx_host = -1
        # Routing decision of the last forward ("linear" | "full"), for logging and tests.
        self.last_choice: Optional[str] = None

    def set_layer_idx(self, idx: int, attn_idx: int = -1) -> None:
        self.layer_idx.fill_(idx)
        self._layer_idx_host = int(idx)
        if attn_idx >= 0:
            self.attn_layer_idx.fill_(attn_idx)
            self._attn_idx_host = int(attn_idx)

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        self._layer_idx_host = int(self.layer_idx.item())
        self._attn_idx_host = int(self.attn_layer_idx.item())

    def _is_full_attention_layer(self) -> bool:
        idx = self._attn_idx_host if self._attn_idx_host >= 0 else self._layer_idx_host
        return (idx + 1) % (self.linear_ratio + 1) == 0

    def choose_full(self, h_states: Optional[torch.Tensor]) -> bool:
        if self.use_dynamic_ratio and h_states is not None:
            return bool(self.interleave_gate(h_states).mean().item() > 0.5)
        return self._is_full_attention_layer()

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                use_cache: bool = False, cache: Optional[dict] = None,
                h_states: Optional[torch.Tensor] = None, rope_offset: int = 0):
        dynamic = self.use_dynamic_ratio and h_states is not None
        full = self.choose_full(h_states)
        self.last_choice = "full" if full else "linear"
        if dynamic:
            want = "full" if full else "linear"
            cache = cache if (cache is None or cache.get("attn_type") == want) else None
        mod = self.full_attn if full else self.linear_attn
        return mod(x, attention_mask=attention_mask, use_cache=use_cache, cache=cache,
                   h_states=h_states, rope_offset=rope_offset)

    def get_lambda_values(self) -> torch.Tensor:
        return (self.linear_attn.get_lambda_values() + self.full_attn.get_lambda_values()) / 2.0

    def extra_repr(self) -> str:
        dyn = ", dynamic_ratio" if self.use_dynamic_ratio else ""
        return (f"d_model={self.d_model}, n_heads={self.n_heads}, n_kv_heads={self.n_kv_heads}, "
                f"head_dim={self.head_dim}, linear_ratio={self.linear_ratio}:1{dyn}")
