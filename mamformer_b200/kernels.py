"""Kernel-level API with the names of the reference's ``mamformer.kernels`` package.

Reference: ``mamformer/kernels/__init__.py`` (``triton_ssd_scan``, ``triton_selective_scan_fused``,
``triton_linear_attn_scan``, ``triton_linear_attn_scan_single``, ``flash_attn_gqa``,
``flash_attn_dsa``, ``flash_attn_with_sliding_window``, availability probes, ``benchmark_ssd``).
The names and tensor layouts are kept so callers of the reference work unchanged; every function
runs this repository's sm_100a kernels (no Triton, no flash-attn library) on CUDA tensors and the
PyTorch reference path elsewhere.  Layouts follow the reference: attention inputs are
``(batch, heads, seq, head_dim)``; scan inputs are ``(batch, seq, channels)``.
"""

from __future__ import annotations

import math
import time
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from mamformer_b200 import ops


def is_native_available() -> bool:
    return ops.has_native() and torch.cuda.is_available()


def is_triton_available() -> bool:
    """The reference's probe; this framework's kernels are CUDA C++, so it reports the native
    extension instead of Triton."""
    return is_native_available()


def is_flash_attn_available() -> bool:
    return is_native_available()


# ---- selective scan ---------------------------------------------------------------------------
def triton_ssd_scan(x, dt, A, B, C, D, block_size: int = 64) -> torch.Tensor:
    """y_t = C_t . h_t + D x_t with h_t = exp(-exp(A) dt_t) h_{t-1} + B_t dt_t x_t.
    ``A`` is the log-decay (``A_log``); ``dt`` is already positive (after softplus)."""
    return ops.selective_scan(x, dt, A, B, C, D)


def triton_selective_scan_fused(x, dt_proj, A_log, B_proj, C_proj, D, block_size: int = 64) -> torch.Tensor:
    """dt / B / C projections of ``x`` followed by the scan."""
    dt = F.softplus(dt_proj(x))
    return ops.selective_scan(x, dt, A_log, B_proj(x), C_proj(x), D)


# ---- linear attention ---------------------------------------------------------------------------
def _to_bshd(t):
    return t.transpose(1, 2).contiguous()


def triton_linear_attn_scan(q1, q2, k, v, kernel_dim: int, block_k: int = 128, block_d: int = 128,
                            group_h: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Both causal linear-attention reads (o1, o2) of the KDA-Diff linear branch; inputs
    ``(B, H, S, hd)`` with K/V already expanded to the query heads (as the reference)."""
    z = torch.zeros(q1.shape[1], device=q1.device, dtype=torch.float32)
    k_, v_ = _to_bshd(k), _to_bshd(v)
    o1 = ops.linear_diff_attention(_to_bshd(q1), _to_bshd(q1), k_, v_, z, kernel_dim)
    o2 = ops.linear_diff_attention(_to_bshd(q2), _to_bshd(q2), k_, v_, z, kernel_dim)
    return o1.transpose(1, 2), o2.transpose(1, 2)


def triton_linear_attn_scan_single(q, k, v, kernel_dim: int, block_k: int = 128, block_d: int = 128) -> torch.Tensor:
    z = torch.zeros(q.shape[1], device=q.device, dtype=torch.float32)
    q_ = _to_bshd(q)
    return ops.linear_diff_attention(q_, q_, _to_bshd(k), _to_bshd(v), z, kernel_dim).transpose(1, 2)


# ---- softmax attention ------------------------------------------------------------------------------
def flash_attn_gqa(q, k, v, is_causal: bool = True, attention_mask: Optional[torch.Tensor] = None,
                   sliding_window: int = 0, dropout_p: float = 0.0,
                   softmax_scale: Optional[float] = None) -> torch.Tensor:
    """Causal GQA attention (``(B, H, S, hd)``), optional causal sliding window of
    ``sliding_window`` keys (position i sees [i - W + 1, i])."""
    if softmax_scale is not None and abs(softmax_scale - 1.0 / math.sqrt(q.shape[-1])) > 1e-12:
        q = q * (softmax_scale * math.sqrt(q.shape[-1]))
    if not is_causal and attention_mask is None:
        attention_mask = torch.zeros(q.shape[2], k.shape[2], device=q.device, dtype=q.dtype)
    out = ops.attention(_to_bshd(q), _to_bshd(k), _to_bshd(v), window=sliding_window,
                        window_mode="causal", attention_mask=attention_mask, dropout_p=dropout_p)
    return out.transpose(1, 2)


def flash_attn_dsa(q1, q2, k, v, lam, is_causal: bool = True, attention_mask: Optional[torch.Tensor] = None,
                   sliding_window: int = 0, dropout_p: float = 0.0,
                   softmax_scale: Optional[float] = None) -> torch.Tensor:
    """(softmax(Q1 K^T s) - lam softmax(Q2 K^T s)) V / (1 - lam), ``(B, H, S, hd)`` layout."""
    H = q1.shape[1]
    lam_t = lam if torch.is_tensor(lam) else torch.tensor(float(lam), device=q1.device)
    lam_t = lam_t.float().reshape(-1).expand(H) if lam_t.numel() == 1 else lam_t.float()
    out = ops.diff_attention(_to_bshd(q1), _to_bshd(q2), _to_bshd(k), _to_bshd(v), lam_t,
                             window=sliding_window, window_mode="causal", attention_mask=attention_mask,
                             scale=softmax_scale)
    return out.transpose(1, 2)


def flash_attn_with_sliding_window(q, k, v, window_size: int, is_causal: bool = True, dropout_p: float = 0.0,
                                   softmax_scale: Optional[float] = None) -> torch.Tensor:
    return flash_attn_gqa(q, k, v, is_causal, None, window_size, dropout_p, softmax_scale)


def get_attention_backend_info() -> dict:
    return {"native_sm100a": is_native_available(), "device": torch.cuda.get_device_name(0)
            if torch.cuda.is_available() else "cpu"}


# ---- benchmark ------------------------------------------------------------------------------------
def benchmark_ssd(batch_size: int = 2, seq_len: int = 2048, d_inner: int = 4096, d_state: int = 128,
                  num_warmup: int = 5, num_iters: int = 20, device: str = "cuda") -> dict:
    """Native scan against the sequential PyTorch scan, timed with CUDA events."""
    from mamformer_b200.ops import reference as ref
    g = torch.Generator(device=device).manual_seed(0)
    x = torch.randn(batch_size, seq_len, d_inner, device=device, generator=g)
    dt = F.softplus(torch.randn(batch_size, seq_len, d_inner, device=device, generator=g) - 2)
    A = torch.log(torch.linspace(0.5, 8, d_state, device=device))
    Bm = torch.randn(batch_size, seq_len, d_state, device=device, generator=g)
    Cm = torch.randn(batch_size, seq_len, d_state, device=device, generator=g)
    D = torch.ones(d_inner, device=device)
    res = {}
    for name, fn in (("native", lambda: ops.selective_scan(x, dt, A, Bm, Cm, D)),
                     ("pytorch", lambda: ref.selective_scan(x, dt, A, Bm, Cm, D))):
        for _ in range(num_warmup if name == "native" else 1):
            fn()
        if device == "cuda":
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(num_iters if name == "native" else 1):
                fn()
            b.record()
            torch.cuda.synchronize()
            res[f"{name}_ms"] = a.elapsed_time(b) / (num_iters if name == "native" else 1)
        else:
            t = time.perf_counter()
            fn()
            res[f"{name}_ms"] = (time.perf_counter() - t) * 1000
    res["speedup"] = res["pytorch_ms"] / max(res["native_ms"], 1e-9)
    return res


__all__ = ["triton_ssd_scan", "triton_selective_scan_fused", "triton_linear_attn_scan",
           "triton_linear_attn_scan_single", "is_triton_available", "flash_attn_gqa", "flash_attn_dsa",
           "flash_attn_with_sliding_window", "is_flash_attn_available", "is_native_available",
           "get_attention_backend_info", "benchmark_ssd"]
