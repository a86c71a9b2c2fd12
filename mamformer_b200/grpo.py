"""GRPO / S-GRPO reinforcement learning on top of the causal LM.

Reference: ``scripts/train_grpo.py`` (``GRPOPromptDataset`` 99-152, ``collate_prompts`` 154-178,
``compute_grpo_loss`` 180-229, the step of ``train_grpo`` 460-650).  One step:

1. for each prompt, G rollouts with temperatures ``T * (0.9 + 0.2 g / (G - 1))``;
2. rule rewards (``mamformer_b200.rewards``) -> group-normalised advantages
   ``(r - mean_g r) / (std_g r + 1e-8)``;
3. policy and frozen reference mean log-probs over the response tokens (optionally the S-GRPO
   random subset, the same subset for both);
4. loss ``-mean(A * logp) + beta * mean(logp_ref - logp)``; gradient accumulation, clipping and
   the mixed-precision AdamW of the pre-training engine.

Deviation: the S-GRPO mask is placed on the response positions of the shifted label axis (the
reference fills the first ``len(response)`` positions of that axis, i.e. mostly prompt positions
that its label mask then removes).
"""

from __future__ import annotations

import copy
import json
import logging
from dataclasses import dataclass, field
from pathlib import Path
from typing import List, Optional, Tuple

import torch

from mamformer_b200.rewards import RewardCalculator
from mamformer_b200.sgrpo import StochasticGRPOConfig, sample_token_mask

logger = logging.getLogger(__name__)


@dataclass
class GRPOConfig:
    group_size: int = 4
    gen_max_tokens: int = 256
    gen_temperature: float = 0.8
    gen_top_k: int = 50
    gen_top_p: float = 0.95
    kl_beta: float = 0.04
    learning_rate: float = 1e-6
    weight_decay: float = 0.0
    max_grad_norm: float = 1.0
    grad_accum: int = 1
    sub_batch_size: Optional[int] = None
    warmup_steps: int = 10
    max_steps: int = 1000
    sgrpo: StochasticGRPOConfig = field(default_factory=StochasticGRPOConfig)


class PromptDataset(torch.utils.data.Dataset):
    """JSONL prompts ``{"prompt", "answer", "reward_type", "test_cases", "reward_weights"}``; a
    100-item arithmetic stand-in when the file does not exist (as the reference)."""

    def __init__(self, data_path: str, tokenizer, max_prompt_len: int = 2048):
        self.tokenizer = tokenizer
        self.max_prompt_len = max_prompt_len
        p = Path(data_path) if data_path else None
        self.items: List[dict] = []
        self._use_dummy = p is None or not p.exists()
        if self._use_dummy:
            logger.warning("GRPO data %s not found; using dummy prompts", data_path)
            self.items = [{"prompt": f"Question {i}: What is 2+2?", "answer": "4", "reward_type": "math"}
                          for i in range(100)]
        else:
            for line in p.read_text(encoding="utf-8").splitlines():
                line = line.strip()
                if not line:
                    continue
                try:
                    self.items.append(json.loads(line))
                except json.JSONDecodeError:
                    logger.warning("skipping malformed JSONL line: %s", line[:80])

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        it = self.items[i]
        ids = self.tokenizer.encode(it["prompt"], add_bos=True)[: self.max_prompt_len]
        return {"input_ids": torch.tensor(ids, dtype=torch.long), "ground_truth": it.get("answer", ""),
                "reward_type": it.get("reward_type", "format"), "test_cases": it.get("test_cases", []),
                "reward_weights": it.get("reward_weights")}


GRPOPromptDataset = PromptDataset


def collate_prompts(batch: List[dict]) -> dict:
    L = max(b["input_ids"].numel() for b in batch)
    ids = torch.zeros(len(batch), L, dtype=torch.long)
    for i, b in enumerate(batch):
        ids[i, : b["input_ids"].numel()] = b["input_ids"]
    out = {"input_ids": ids}
    for k in ("ground_truth", "reward_type", "test_cases", "reward_weights"):
        out[k] = [b[k] for b in batch]
    return out


def compute_grpo_loss(policy_log_probs: torch.Tensor, reference_log_probs: torch.Tensor,
                      advantages: torch.Tensor, kl_beta: float = 0.04) -> Tuple[torch.Tensor, dict]:
    pg = -(advantages * policy_log_probs).mean()
    kl = (reference_log_probs - policy_log_probs).mean()
    return pg + kl_beta * kl, {"policy_loss": pg.detach(), "kl_div": kl.detach(),
                               "mean_advantage": advantages.mean().detach(),
                               "std_advantage": advantages.std().detach()}


def group_advantages(rewards: torch.Tensor) -> torch.Tensor:
    """(B, G) rewards -> (r - mean) / (std + 1e-8) within each group."""
    return (rewards - rewards.mean(1, keepdim=True)) / (rewards.std(1, keepdim=True) + 1e-8)


def rollout_temperatures(base: float, G: int) -> List[float]:
    return [base * (0.9 + 0.2 * g / max(G - 1, 1)) for g in range(G)]


class GRPOTrainer:
    """Policy + frozen reference + optimizer; ``step(batch)`` runs one GRPO update."""

    def __init__(self, policy, tokenizer, cfg: GRPOConfig, reference=None, compute_dtype=None):
        from mamformer_b200.optim import MixedPrecisionAdamW, create_lr_scheduler, param_groups
        from mamformer_b200.utils.precision import to_compute_dtype
        self.cfg = cfg
        self.policy = policy
        self.tokenizer = tokenizer
        self.reference = reference if reference is not None else copy.deepcopy(policy)
        self.reference.eval()
        for p in self.reference.parameters():
            p.requires_grad_(False)
        if compute_dtype is not None and compute_dtype != torch.float32:
            to_compute_dtype(self.policy, compute_dtype)
            to_compute_dtype(self.reference, compute_dtype)
        self.optimizer = MixedPrecisionAdamW(
            param_groups(policy, cfg.weight_decay, extra_no_decay=("comm_strength",)), lr=cfg.learning_rate,
            weight_decay=cfg.weight_decay, max_grad_norm=cfg.max_grad_norm)
        self.scheduler = create_lr_scheduler(self.optimizer, cfg.warmup_steps, cfg.max_steps, cfg.learning_rate)
        self.rewards = RewardCalculator()
        self.global_step = 0
        self.device = next(policy.parameters()).device

    # -- pieces ---------------------------------------------------------------------------------
    @torch.no_grad()
    def rollouts(self, prompt_ids: torch.Tensor):
        c = self.cfg
        self.policy.eval()
        outs = []
        for t in rollout_temperatures(c.gen_temperature, c.group_size):
            g = self.policy.generate(prompt_ids, max_new_tokens=c.gen_max_tokens, temperature=t, top_k=c.gen_top_k,
                                     top_p=c.gen_top_p)
            outs.append(g[:, prompt_ids.shape[1]:])
        self.policy.train()
        return outs

    def score(self, texts: List[List[str]], batch: dict) -> torch.Tensor:
        B, G = len(texts), len(texts[0])
        r = torch.zeros(B, G)
        for b in range(B):
            kind = batch["reward_type"][b]
            kw = {}
            if kind == "math":
                kw["ground_truth"] = batch["ground_truth"][b]
            elif kind == "code":
                kw["test_cases"] = batch["test_cases"][b]
            elif kind == "combined" and batch["reward_weights"][b] is not None:
                kw["reward_weights"] = batch["reward_weights"][b]
            for g in range(G):
                try:
                    r[b, g] = self.rewards.compute(texts[b][g], reward_type=kind, **kw)
                except (ValueError, KeyError, TypeError) as e:
                    logger.warning("reward failed for prompt %d rollout %d: %s", b, g, e)
        return r

    def build_sequences(self, prompt_ids: torch.Tensor, responses: List[torch.Tensor]):
        """(B*G, P+R) ids and labels with the prompt and each rollout's padding set to -100,
        plus each row's response length."""
        B, P = prompt_ids.shape
        G = len(responses)
        R = max(r.shape[1] for r in responses)
        resp = torch.zeros(B, G, R, dtype=torch.long, device=prompt_ids.device)
        lens = torch.zeros(B, G, dtype=torch.long)
        for g, r in enumerate(responses):
            resp[:, g, : r.shape[1]] = r
            lens[:, g] = r.shape[1]
        ids = torch.cat([prompt_ids.unsqueeze(1).expand(B, G, P), resp], 2).reshape(B * G, P + R)
        labels = ids.clone()
        labels[:, :P] = -100
        flat_len = lens.reshape(-1)
        for i in range(B * G):
            labels[i, P + int(flat_len[i]):] = -100
        return ids, labels, flat_len

    def token_masks(self, labels: torch.Tensor, prompt_len: int, lens: torch.Tensor):
        if not self.cfg.sgrpo.enabled:
            return None
        m = torch.zeros(labels.shape[0], labels.shape[1] - 1, dtype=torch.bool, device=labels.device)
        for i in range(labels.shape[0]):
            n = int(lens[i])
            if n:
                m[i, prompt_len - 1: prompt_len - 1 + n] = sample_token_mask(n, self.cfg.sgrpo, labels.device)
        return m

    # -- step -----------------------------------------------------------------------------------
    def step(self, batch: dict) -> dict:
        c = self.cfg
        prompt = batch["input_ids"].to(self.device)
        B, P = prompt.shape
        responses = self.rollouts(prompt)
        texts = [[self.tokenizer.decode(r[b].tolist()) for r in responses] for b in range(B)]
        rewards = self.score(texts, batch).to(self.device)
        adv = group_advantages(rewards)
        ids, labels, lens = self.build_sequences(prompt, responses)
        tmask = self.token_masks(labels, P, lens)
        N = ids.shape[0]
        sb = c.sub_batch_size or N
        pol = torch.zeros(N, device=self.device)
        ref = torch.zeros(N, device=self.device)
        for s in range(0, N, sb):
            e = min(N, s + sb)
            tm = tmask[s:e] if tmask is not None else None
            pol[s:e] = self.policy.get_log_probs(ids[s:e], labels=labels[s:e], token_mask=tm).float()
            with torch.no_grad():
                ref[s:e] = self.reference.get_log_probs(ids[s:e], labels=labels[s:e], token_mask=tm).float()
        loss, metrics = compute_grpo_loss(pol.view(B, -1), ref.view(B, -1), adv, c.kl_beta)
        if self.global_step % c.grad_accum == 0:
            self.optimizer.zero_grad()
        (loss / c.grad_accum).backward()
        self.global_step += 1
        if self.global_step % c.grad_accum == 0:
            self.optimizer.step()
            self.scheduler.step()
        metrics.update(loss=loss.detach(), mean_reward=rewards.mean(), response_tokens=float(lens.float().mean()))
        return metrics
