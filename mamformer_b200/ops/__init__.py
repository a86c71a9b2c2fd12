"""Hot-op dispatch: native sm_100a kernels for CUDA tensors, PyTorch reference math on CPU.

Every public function here is differentiable.  For CUDA tensors it calls the in-tree
extension ``mamformer_b200._C`` (built by ``setup.py build_ext --inplace`` or
``__graft_entry__.build()``); if that extension is missing on a machine with a GPU the call
raises instead of silently running PyTorch code.  CPU tensors always take the reference path
(``ops.reference``), which is also the numerics oracle in the tests.

``NATIVE`` lists the ops that have a native kernel; ops not listed run composite PyTorch on
CUDA too (each is a documented gap).
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn.functional as F

from mamformer_b200.ops import reference as ref
from mamformer_b200.ops._ext import ext, has_native, require_native

__all__ = [
    "rms_norm", "rope", "swiglu", "causal_conv1d_silu", "selective_scan", "mamba_inner",
    "linear_diff_attention", "diff_attention", "attention", "head_group_norm", "router_topk",
    "expert_histogram", "moe_routed", "moe_expert_outputs", "linear_cross_entropy",
    "fused_ce_available", "token_log_probs", "NATIVE", "has_native", "force_reference",
]

# Native-kernel coverage (op name -> kernel source file).  Filled by ops.native on import.
NATIVE: dict = {}

_FORCE_REF = os.environ.get("MAMF_FORCE_REFERENCE", "0") == "1"


def force_reference() -> bool:
    """True when MAMF_FORCE_REFERENCE=1 sends every CUDA op to its eager PyTorch form (for A/B
    debugging only; benchmarks refuse to run in this mode)."""
    return _FORCE_REF


def _native(t: torch.Tensor) -> bool:
    """True when this call should take the native path (CUDA tensor).  Raises if the
    extension is absent on CUDA, unless MAMF_FORCE_REFERENCE=1 (debug / A-B only)."""
    if not t.is_cuda or _FORCE_REF:
        return False
    require_native()
    return True


def _nat():
    from mamformer_b200.ops import native
    return native


# ---------------------------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    if _native(x) and "rms_norm" in NATIVE:
        return _nat().rms_norm(x, weight, eps)
    return ref.rms_norm(x, weight, eps)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x (B, S, H, hd); cos/sin (S, hd/2) fp32 -> rotated copy."""
    if _native(x) and "rope" in NATIVE:
        return _nat().rope(x, cos, sin)
    return ref.rope(x, cos, sin)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    if _native(gate) and "swiglu" in NATIVE:
        return _nat().swiglu(gate, up)
    return ref.swiglu(gate, up)


def causal_conv1d_silu(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """silu(depthwise causal conv(x)); x (B, S, C) (may be a strided view), weight (C, K)."""
    if _native(x) and "causal_conv1d_silu" in NATIVE:
        return _nat().causal_conv1d_silu(x, weight)
    return F.silu(ref.causal_conv1d(x, weight))


def selective_scan(x, dt, A_log, B, C, D, return_h_states=False, return_final_state=False):
    """Reference-signature scan (dt already positive)."""
    if _native(x) and "selective_scan" in NATIVE:
        return _nat().selective_scan(x, dt, A_log, B, C, D, return_h_states, return_final_state)
    return ref.selective_scan(x, dt, A_log, B, C, D, return_h_states, return_final_state)


def mamba_inner(x_act, dt_raw, A_log, Bm, Cm, D, z, need_h_states: bool,
                return_final: bool = False):
    """softplus(dt_raw) -> scan -> y*silu(z).  Returns (y_gated, h_states|None, final|None)."""
    if _native(x_act) and "mamba_inner" in NATIVE:
        return _nat().mamba_inner(x_act, dt_raw, A_log, Bm, Cm, D, z, need_h_states, return_final)
    return ref.mamba_inner(x_act, dt_raw, A_log, Bm, Cm, D, z, need_h_states, return_final=return_final)


def linear_diff_attention(q1, q2, k, v, lam, kernel_dim: int, chunk: int = 256):
    if _native(q1) and "linear_diff_attention" in NATIVE:
        return _nat().linear_diff_attention(q1, q2, k, v, lam, kernel_dim)
    return ref.linear_diff_attention(q1, q2, k, v, lam, kernel_dim, chunk)


def _window_bounds(window: int, window_mode: str):
    """(lo, hi) on (key - query) for same-length self-attention, causal included."""
    if window <= 0:
        return -(1 << 30), 0
    if window_mode == "reference":
        return 0, 0           # causal AND 0 <= k - q < W  ->  diagonal only
    return -(window - 1), 0   # causal sliding window


def diff_attention(q1, q2, k, v, lam, window: int = 0, window_mode: str = "reference",
                   attention_mask: Optional[torch.Tensor] = None, scale: Optional[float] = None):
    same_len = q1.shape[1] == k.shape[1]
    if _native(q1) and "diff_attention" in NATIVE and attention_mask is None and same_len:
        lo, hi = _window_bounds(window, window_mode)
        return _nat().diff_attention(q1, q2, k, v, lam, lo, hi, scale)
    if window > 0 and window_mode == "causal":
        return _causal_window_diff(q1, q2, k, v, lam, window, attention_mask, scale)
    return ref.diff_attention(q1, q2, k, v, lam, window, True, scale, attention_mask)


def _causal_window_diff(q1, q2, k, v, lam, window, attention_mask, scale):
    S, Skv = q1.shape[1], k.shape[1]
    off = Skv - S
    iq = torch.arange(S, device=q1.device).unsqueeze(1) + off
    ik = torch.arange(Skv, device=q1.device).unsqueeze(0)
    valid = (ik <= iq) & (iq - ik < window)
    m = torch.zeros(S, Skv, device=q1.device, dtype=q1.dtype).masked_fill(~valid, float("-inf"))
    if attention_mask is not None:
        m = m + attention_mask
    return ref.diff_attention(q1, q2, k, v, lam, 0, False, scale, m)


def attention(q, k, v, window: int = 0, window_mode: str = "reference",
              attention_mask: Optional[torch.Tensor] = None, dropout_p: float = 0.0):
    """GQA softmax attention, reference masking semantics (see models.attention)."""
    same_len = q.shape[1] == k.shape[1]
    native_ok = attention_mask is None and same_len and dropout_p == 0.0
    if _native(q) and "attention" in NATIVE and native_ok:
        if window > 0 and window_mode == "reference":
            lo, hi = 0, window - 1          # reference GQA window: 0 <= key - query < W, no causal mask
        else:
            lo, hi = _window_bounds(window, window_mode)
        return _nat().attention(q, k, v, lo, hi)
    if window > 0 and window_mode == "causal":
        S, Skv = q.shape[1], k.shape[1]
        iq = torch.arange(S, device=q.device).unsqueeze(1) + (Skv - S)
        ik = torch.arange(Skv, device=q.device).unsqueeze(0)
        valid = (ik <= iq) & (iq - ik < window)
        m = torch.zeros(S, Skv, device=q.device, dtype=q.dtype).masked_fill(~valid, float("-inf"))
        return ref.sdpa_attention(q, k, v, 0, m if attention_mask is None else m + attention_mask, dropout_p)
    return ref.sdpa_attention(q, k, v, window, attention_mask, dropout_p)


def head_group_norm(x: torch.Tensor, n_heads: int, weight: torch.Tensor, bias: torch.Tensor,
                    eps: float) -> torch.Tensor:
    if _native(x) and "head_group_norm" in NATIVE:
        return _nat().head_group_norm(x, n_heads, weight, bias, eps)
    return ref.head_group_norm(x, n_heads, weight.to(x.dtype) if x.dtype != torch.float32 else weight,
                               bias.to(x.dtype) if x.dtype != torch.float32 else bias, eps)


def router_topk(scores: torch.Tensor, k: int):
    """(softmax over the top-k scores, indices).  scores (T, E) fp32."""
    if _native(scores) and "router_topk" in NATIVE:
        return _nat().router_topk(scores, k)
    return ref.router_topk(scores, k)


def expert_histogram(idx: torch.Tensor, n_experts: int) -> torch.Tensor:
    if _native(idx) and "expert_histogram" in NATIVE:
        return _nat().expert_histogram(idx, n_experts)
    return torch.bincount(idx.flatten().long(), minlength=n_experts)


def moe_routed(x, idx, gates, w_gate, w_up, w_down):
    if _native(x) and "moe_routed" in NATIVE:
        return _nat().moe_routed(x, idx, gates, w_gate, w_up, w_down)
    return ref.moe_routed(x, idx, gates, w_gate, w_up, w_down)


def moe_expert_outputs(x, idx, w_gate, w_up, w_down):
    """Unweighted per-slot expert outputs (T, k, d)."""
    if _native(x) and "moe_expert_outputs" in NATIVE:
        return _nat().moe_expert_outputs(x, idx, w_gate, w_up, w_down)
    return ref.moe_expert_outputs(x, idx, w_gate, w_up, w_down)


def fused_ce_available(h: torch.Tensor) -> bool:
    return h.is_cuda and not _FORCE_REF and has_native() and "linear_cross_entropy" in NATIVE


def linear_cross_entropy(h: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                         ignore_index: int = -100) -> torch.Tensor:
    if _native(h) and "linear_cross_entropy" in NATIVE:
        return _nat().linear_cross_entropy(h, weight, labels, ignore_index)
    return ref.linear_cross_entropy(h, weight, labels, ignore_index)


def token_log_probs(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """log_softmax(logits)[..., target] without materialising the full log-softmax."""
    lf = logits.float()
    return lf.gather(-1, targets.unsqueeze(-1)).squeeze(-1) - torch.logsumexp(lf, dim=-1)


# Register native ops (import has no side effects when the extension is absent).
if has_native():
    from mamformer_b200.ops import native as _native_mod  # noqa: F401
