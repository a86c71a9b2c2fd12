"""Rotary position embeddings with the reference's YaRN variant.

Semantics (reference ``mamformer/layers/rope.py``):

* inverse frequencies ``theta^(-2j/hd)``; LLaMA half-split rotation
  (``x1*cos - x2*sin, x2*cos + x1*sin`` on the two halves) - ``rope.py:283-339``;
* YaRN (only when ``use_yarn`` and ``yarn_scale > 1``): wavelength ``2*pi/f``, ramp
  ``clamp((wl - beta_slow) / (beta_fast - beta_slow), 0, 1)``, frequencies *multiplied* by
  ``1 + (scale - 1) * ramp`` - ``rope.py:123-162``.  This is not the published YaRN; it is
  kept because checkpoints trained with it depend on it;
* positions start at ``offset``.  The reference's callers always pass offset 0, also while
  decoding with a cache, so decode positions restart at 0 (``attention.py:134``,
  ``kda_diff.py:276,808``).  The layers here default to the same behaviour for checkpoint
  parity (``rope_offset_mode='reference'``) and can use true positions instead
  (``'absolute'``).

Tables are built once per (length, offset, device) and kept in a small LRU; the rotation
itself runs in the native ``rope`` kernel on CUDA (in place on a [B, S, H, hd] tensor).
"""

from __future__ import annotations

import math
from collections import OrderedDict
from typing import Optional, Tuple

import torch
import torch.nn as nn

from mamformer_b200 import ops


def yarn_scale_frequencies(freqs: torch.Tensor, scale: float, beta_fast: float,
                           beta_slow: float) -> torch.Tensor:
    wavelength = 2.0 * math.pi / freqs
    ramp = ((wavelength - beta_slow) / max(1e-6, beta_fast - beta_slow)).clamp(0.0, 1.0)
    return freqs * (1.0 + (scale - 1.0) * ramp)


class RotaryEmbedding(nn.Module):
    def __init__(self, head_dim: int, max_seq_len: int = 8192, theta: float = 10000.0,
                 use_yarn: bool = False, yarn_scale: float = 1.0,
                 yarn_original_max_seq_len: Optional[int] = None, yarn_beta_fast: int = 32,
                 yarn_beta_slow: int = 1) -> None:
        super().__init__()
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.theta = float(theta)
        self.use_yarn = bool(use_yarn)
        self.yarn_scale = float(yarn_scale)
        self.yarn_original_max_seq_len = yarn_original_max_seq_len or max_seq_len
        self.yarn_beta_fast = yarn_beta_fast
        self.yarn_beta_slow = yarn_beta_slow
        inv = 1.0 / (self.theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        self.register_buffer("inv_freqs", inv, persistent=False)
        self._tables: "OrderedDict[tuple, Tuple[torch.Tensor, torch.Tensor]]" = OrderedDict()

    def frequencies(self, device) -> torch.Tensor:
        f = self.inv_freqs.to(device)
        if self.use_yarn and self.yarn_scale > 1.0:
            f = yarn_scale_frequencies(f, self.yarn_scale, self.yarn_beta_fast, self.yarn_beta_slow)
        return f

    def forward(self, seq_len: int, device, offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
        """(cos, sin), each (1, 1, seq_len, head_dim) fp32 (full-width, halves duplicated)."""
        key = (int(seq_len), int(offset), str(device))
        hit = self._tables.get(key)
        if hit is not None:
            self._tables.move_to_end(key)
            return hit
        pos = torch.arange(offset, offset + seq_len, dtype=torch.float32, device=device)
        ang = torch.outer(pos, self.frequencies(device))
        ang = torch.cat([ang, ang], dim=-1)
        out = (ang.cos()[None, None], ang.sin()[None, None])
        if len(self._tables) >= 16:
            self._tables.popitem(last=False)
        self._tables[key] = out
        return out

    def clear_cache(self) -> None:
        self._tables.clear()

    def extra_repr(self) -> str:
        yarn = f", YaRN(scale={self.yarn_scale}, orig={self.yarn_original_max_seq_len})" if self.use_yarn else ""
        return f"head_dim={self.head_dim}, max_seq_len={self.max_seq_len}, theta={self.theta}{yarn}"


class CachedRotaryEmbedding(RotaryEmbedding):
    """Precomputed table up to ``max_seq_len`` (<=128K); longer contexts compute on demand."""

    def __init__(self, head_dim: int, max_seq_len: int = 8192, theta: float = 10000.0,
                 use_yarn: bool = False, yarn_scale: float = 1.0,
                 yarn_original_max_seq_len: Optional[int] = None) -> None:
        super().__init__(head_dim, max_seq_len, theta, use_yarn, yarn_scale, yarn_original_max_seq_len)
        self._use_cached_table = max_seq_len <= 131072
        if self._use_cached_table:
            cos, sin = RotaryEmbedding.forward(self, max_seq_len, torch.device("cpu"))
            self._tables.clear()
            self.register_buffer("cos", cos, persistent=False)
            self.register_buffer("sin", sin, persistent=False)

    def forward(self, seq_len: int, device, offset: int = 0):
        if self._use_cached_table and offset + seq_len <= self.max_seq_len:
            return (self.cos[:, :, offset:offset + seq_len].to(device),
                    self.sin[:, :, offset:offset + seq_len].to(device))
        return super().forward(seq_len, device, offset)


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                     interleaved: bool = False) -> torch.Tensor:
    """Rotate ``x`` (B, H, S, hd) with tables shaped (1, 1, S, hd) or (1, 1, S, hd/2)."""
    hd = x.shape[-1]
    if cos.shape[-1] == hd // 2:
        cos = torch.cat([cos, cos], -1)
        sin = torch.cat([sin, sin], -1)
    if interleaved:
        xe, xo = x[..., 0::2], x[..., 1::2]
        c, s = cos[..., 0::2], sin[..., 0::2]
        out = torch.empty_like(x)
        out[..., 0::2] = xe * c - xo * s
        out[..., 1::2] = xo * c + xe * s
        return out
    half = hd // 2
    x1, x2 = x[..., :half], x[..., half:]
    c, s = cos[..., :half], sin[..., :half]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(x.dtype)


def apply_rope_bshd(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate ``x`` laid out (B, S, H, hd) with (1, 1, S, hd) tables (native kernel on CUDA)."""
    return ops.rope(x, cos[0, 0, :, : x.shape[-1] // 2], sin[0, 0, :, : x.shape[-1] // 2])


def precompute_freqs_cis(head_dim: int, seq_len: int, theta: float = 10000.0,
                         device=torch.device("cpu")) -> torch.Tensor:
    f = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))
    ang = torch.outer(torch.arange(seq_len, dtype=torch.float32, device=device), f)
    return torch.polar(torch.ones_like(ang), ang)


def apply_rotary_emb_complex(x: torch.Tensor, freqs_cis: torch.Tensor) -> torch.Tensor:
    """Adjacent-pair rotation through complex multiplication, x (B, H, S, hd)."""
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xc * freqs_cis[None, None]).flatten(-2).to(x.dtype)
