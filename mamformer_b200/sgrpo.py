"""Stochastic GRPO: the policy-gradient loss over a random subset of response tokens.

Reference: ``mamformer/sgrpo.py:1-151`` (``StochasticGRPOConfig``, ``sample_token_mask``; the
method of arXiv:2504.20834).  Selection rule, kept identical so that a seeded mask means the
same thing in both frameworks: the first ``alpha`` positions are always kept, every later
position is kept when a uniform draw is below ``p``, and when more than ``k`` positions survive
(``k > 0``) a random permutation of the non-leading survivors keeps ``k - alpha`` of them.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class StochasticGRPOConfig:
    enabled: bool = False
    p: float = 0.4
    alpha: int = 0
    k: int = 0
    seed: Optional[int] = None

    def validate(self) -> None:
        if not self.enabled:
            return
        if not 0.0 < self.p <= 1.0:
            raise ValueError(f"p must be in (0, 1], got {self.p}")
        if self.alpha < 0:
            raise ValueError(f"alpha must be >= 0, got {self.alpha}")
        if self.k < 0:
            raise ValueError(f"k must be >= 0, got {self.k}")


def sample_token_mask(seq_len: int, config: StochasticGRPOConfig, device=None) -> torch.Tensor:
    """Boolean (seq_len,) mask of the response positions that enter the loss."""
    if not config.enabled or seq_len == 0:
        return torch.ones(seq_len, dtype=torch.bool, device=device)
    lead = min(config.alpha, seq_len)
    keep = torch.zeros(seq_len, dtype=torch.bool, device=device)
    keep[:lead] = True
    rest = seq_len - lead
    if rest > 0:
        gen = None
        if config.seed is not None:
            gen = torch.Generator(device=device)
            gen.manual_seed(config.seed)
        keep[lead:] = torch.rand(rest, device=device, generator=gen) < config.p
    if config.k > 0 and int(keep.sum()) > config.k:
        chosen = keep.nonzero().squeeze(-1)
        tail = chosen[chosen >= lead]
        slots = max(0, config.k - lead)
        if slots < tail.numel():
            tail = tail[torch.randperm(tail.numel(), device=device)[:slots]]
        keep = torch.zeros(seq_len, dtype=torch.bool, device=device)
        keep[:lead] = True
        keep[tail] = True
    return keep


def batch_token_masks(lengths, config: StochasticGRPOConfig, max_len: int, device=None) -> torch.Tensor:
    """(B, max_len) masks for responses of the given lengths (positions past a length False)."""
    out = torch.zeros(len(lengths), max_len, dtype=torch.bool, device=device)
    for i, n in enumerate(lengths):
        n = int(min(n, max_len))
        out[i, :n] = sample_token_mask(n, config, device)
    return out
