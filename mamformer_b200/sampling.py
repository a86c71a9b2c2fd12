"""Token sampling shared by every generation path (reference ``mamformer/sampling.py``).

``sample_one_token``: greedy for temperature <= 0; else temperature, top-k (keep logits >= the
k-th largest), top-p (drop tokens whose preceding cumulative probability already exceeds p;
the top token is always kept), softmax, uniform fallback for an all-masked row, multinomial.
``apply_repetition_penalty``: positive logits of seen tokens are divided by the penalty,
non-positive ones multiplied (vectorised; same result as the reference's per-token loop).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def sample_one_token(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0,
                     top_p: float = 1.0) -> torch.Tensor:
    if temperature <= 0:
        return logits.argmax(dim=-1, keepdim=True)
    V = logits.shape[-1]
    logits = logits.float()
    if temperature != 1.0:
        logits = logits / temperature
    if top_k > 0:
        kth = torch.topk(logits, min(top_k, V), dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    if top_p < 1.0:
        sorted_logits, order = torch.sort(logits, descending=True, dim=-1)
        cum = torch.cumsum(F.softmax(sorted_logits, dim=-1), dim=-1)
        drop = cum > top_p
        drop[:, 1:] = drop[:, :-1].clone()
        drop[:, 0] = False
        logits = logits.masked_fill(drop.scatter(1, order, drop), float("-inf"))
    probs = F.softmax(logits, dim=-1)
    sums = probs.sum(-1, keepdim=True)
    probs = torch.where(sums > 0, probs, torch.full_like(probs, 1.0 / V))
    probs = probs / probs.sum(-1, keepdim=True).clamp(min=1e-12)
    return torch.multinomial(probs, num_samples=1)


def apply_repetition_penalty(logits: torch.Tensor, generated_ids: torch.Tensor,
                             penalty: float) -> torch.Tensor:
    if penalty == 1.0:
        return logits
    seen = torch.zeros_like(logits, dtype=torch.bool)
    ids = generated_ids.clamp(min=0, max=logits.shape[-1] - 1)
    seen.scatter_(1, ids, True)
    penalised = torch.where(logits > 0, logits / penalty, logits * penalty)
    return torch.where(seen, penalised, logits)
