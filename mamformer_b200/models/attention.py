"""Grouped-query softmax attention (reference ``mamformer/layers/attention.py:26-224``).

q/k/v/o projections without bias, RoPE on q and k, KV cache by concatenation, GQA by index.
Used by dense non-KDA configs and by every MTP depth.  On CUDA the attention runs in the
native flash-attention kernel (single-softmax instantiation of the differential kernel); on
CPU it runs PyTorch SDPA with the reference's masks.

Window semantics: the reference's sliding-window mask keeps keys with
``0 <= key - query < W`` and, for this module, *replaces* the causal mask
(``attention.py:157-166, 193-216``), i.e. each query sees itself and the following W-1 keys.
``window_mode='reference'`` (default) reproduces that; ``'causal'`` uses ``0 <= q - k < W``.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from mamformer_b200 import ops
from mamformer_b200.models.rope import RotaryEmbedding


class GroupedQueryAttention(nn.Module):
    def __init__(self, d_model: int, n_heads: int = 32, n_kv_heads: int = 8, head_dim: int = 128,
                 max_seq_len: int = 8192, rope_theta: float = 10000.0, dropout: float = 0.0,
                 sliding_window: int = 0, use_yarn: bool = False, yarn_scale: float = 1.0,
                 yarn_original_max_seq_len: int = 8192, window_mode: str = "reference") -> None:
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.n_head_groups = n_heads // n_kv_heads
        self.dropout = dropout
        self.sliding_window = sliding_window
        self.window_mode = window_mode
        self.q_proj = nn.Linear(d_model, n_heads * head_dim, bias=False)
        self.k_proj = nn.Linear(d_model, n_kv_heads * head_dim, bias=False)
        self.v_proj = nn.Linear(d_model, n_kv_heads * head_dim, bias=False)
        self.o_proj = nn.Linear(n_heads * head_dim, d_model, bias=False)
        self.rope = RotaryEmbedding(head_dim, max_seq_len, rope_theta, use_yarn, yarn_scale,
                                    yarn_original_max_seq_len)
        for p in (self.q_proj, self.k_proj, self.v_proj, self.o_proj):
            nn.init.normal_(p.weight, mean=0.0, std=0.02)

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                use_cache: bool = False, cache: Optional[dict] = None, **kwargs):
        B, S, _ = x.shape
        q = self.q_proj(x).view(B, S, self.n_heads, self.head_dim)
        k = self.k_proj(x).view(B, S, self.n_kv_heads, self.head_dim)
        v = self.v_proj(x).view(B, S, self.n_kv_heads, self.head_dim)
        offset = kwargs.get("rope_offset", 0)
        cos, sin = self.rope(S, x.device, offset)
        q = ops.rope(q, cos[0, 0, :, : self.head_dim // 2], sin[0, 0, :, : self.head_dim // 2])
        k = ops.rope(k, cos[0, 0, :, : self.head_dim // 2], sin[0, 0, :, : self.head_dim // 2])
        if use_cache and cache is not None:
            k = torch.cat([cache["k"], k], dim=1)
            v = torch.cat([cache["v"], v], dim=1)
        new_cache = {"k": k, "v": v} if use_cache else None
        out = ops.attention(q, k, v, window=self.sliding_window, window_mode=self.window_mode,
                            attention_mask=attention_mask,
                            dropout_p=self.dropout if self.training else 0.0)
        return self.o_proj(out.reshape(B, S, -1)), new_cache

    def extra_repr(self) -> str:
        sw = f", sliding_window={self.sliding_window}" if self.sliding_window > 0 else ""
        return (f"d_model={self.d_model}, n_heads={self.n_heads}, n_kv_heads={self.n_kv_heads}, "
                f"head_dim={self.head_dim}, n_head_groups={self.n_head_groups}{sw}")
