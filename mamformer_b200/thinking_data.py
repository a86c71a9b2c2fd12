"""SFT formatting with thinking control tokens (reference ``mamformer/thinking_data.py``).

``prompt <think_start> response <think_end> <summary_start> response <answer_start> response
<answer_end>``; labels mask the prompt with -100.  (The reference repeats the response three
times as a bootstrap format; kept identical so data prepared by either framework matches.)
"""

from __future__ import annotations

from typing import List, Tuple

import torch

THINK_START, THINK_END, ANSWER_START, ANSWER_END, SUMMARY_START = 3, 4, 5, 6, 7


def format_sequence_with_thinking(prompt_ids: List[int], response_ids: List[int]) -> List[int]:
    r = list(response_ids)
    return list(prompt_ids) + [THINK_START] + r + [THINK_END, SUMMARY_START] + r + [ANSWER_START] + r + [ANSWER_END]


def format_labels_with_thinking(prompt_ids: List[int], response_ids: List[int]) -> List[int]:
    full = format_sequence_with_thinking(prompt_ids, response_ids)
    return [-100] * len(prompt_ids) + full[len(prompt_ids):]


def format_batch_with_thinking(prompt_ids_batch: torch.Tensor,
                               response_ids_batch: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    seqs, labs = [], []
    for p, r in zip(prompt_ids_batch.tolist(), response_ids_batch.tolist()):
        p = [t for t in p if t != 0]
        r = [t for t in r if t != 0]
        seqs.append(format_sequence_with_thinking(p, r))
        labs.append(format_labels_with_thinking(p, r))
    L = max(len(s) for s in seqs)
    ids = torch.zeros(len(seqs), L, dtype=torch.long)
    lab = torch.full((len(seqs), L), -100, dtype=torch.long)
    for i, (s, l) in enumerate(zip(seqs, labs)):
        ids[i, :len(s)] = torch.tensor(s)
        lab[i, :len(l)] = torch.tensor(l)
    return ids, lab


def is_thinking_token(token_id: int) -> bool:
    return token_id in (THINK_START, THINK_END, ANSWER_START, ANSWER_END, SUMMARY_START)
