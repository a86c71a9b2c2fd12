"""Generation mixin: sampling loop, beam search with cache reordering, token streaming.

Reference: ``mamformer/generation.py``.  ``RuntimeGenerationConfig`` holds runtime sampling
parameters (distinct from the model-level ``config.GenerationConfig``).  Beam search keeps
2*num_beams candidates per step, applies a ``(step+1)^length_penalty`` normalisation from the
second step on, drops EOS candidates and reorders every cache tensor (KV, linear-attention
state, conv and SSM state) along the batch dimension.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Generator, List, Optional

import torch
import torch.nn.functional as F

from mamformer_b200.sampling import apply_repetition_penalty, sample_one_token


@dataclass
class RuntimeGenerationConfig:
    max_new_tokens: int = 256
    temperature: float = 1.0
    top_k: int = 50
    top_p: float = 0.9
    repetition_penalty: float = 1.0
    num_beams: int = 1
    num_beam_groups: int = 1
    diversity_penalty: float = 0.0
    length_penalty: float = 1.0
    early_stopping: bool = False
    eos_token_id: Optional[int] = None
    pad_token_id: Optional[int] = None
    stop_strings: List[str] = field(default_factory=list)
    thinking_enabled: bool = False
    return_full_text: bool = True
    skip_special_tokens: bool = True

    def validate(self) -> None:
        if self.temperature < 0:
            raise ValueError(f"temperature must be >= 0, got {self.temperature}")
        if self.top_k < 0:
            raise ValueError(f"top_k must be >= 0, got {self.top_k}")
        if not (0.0 < self.top_p <= 1.0):
            raise ValueError(f"top_p must be in (0, 1], got {self.top_p}")
        if self.num_beams < 1:
            raise ValueError(f"num_beams must be >= 1, got {self.num_beams}")
        if self.num_beams > 1 and self.temperature > 0:
            raise ValueError("Beam search and sampling cannot be used together")


class GenerationMixin:
    def _step_logits(self, tokens, cache):
        out = self.forward(input_ids=tokens, use_cache=True, cache=cache, return_logits=True)
        return out["logits"][:, -1, :].float(), out.get("cache")

    @staticmethod
    def _merge(config: Optional[RuntimeGenerationConfig], kwargs) -> RuntimeGenerationConfig:
        cfg = config if config is not None else RuntimeGenerationConfig()
        for k, v in kwargs.items():
            if hasattr(cfg, k):
                setattr(cfg, k, v)
        return cfg

    @torch.no_grad()
    def generate_ids(self, input_ids: torch.Tensor,
                     generation_config: Optional[RuntimeGenerationConfig] = None, **kwargs) -> torch.Tensor:
        cfg = self._merge(generation_config, kwargs)
        cfg.validate()
        return self._beam_search(input_ids, cfg) if cfg.num_beams > 1 else self._sample_loop(input_ids, cfg)

    def _sample_token(self, logits, config: RuntimeGenerationConfig) -> torch.Tensor:
        return sample_one_token(logits, config.temperature, config.top_k, config.top_p)

    def _apply_repetition_penalty(self, logits, generated_ids, penalty):
        return apply_repetition_penalty(logits, generated_ids, penalty)

    def _sample_loop(self, input_ids: torch.Tensor, config: RuntimeGenerationConfig) -> torch.Tensor:
        B = input_ids.shape[0]
        generated, cache = input_ids, None
        alive = torch.ones(B, dtype=torch.bool, device=input_ids.device)
        for _ in range(config.max_new_tokens):
            if not bool(alive.any()):
                break
            logits, cache = self._step_logits(generated if cache is None else generated[:, -1:], cache)
            if config.repetition_penalty != 1.0:
                logits = self._apply_repetition_penalty(logits, generated, config.repetition_penalty)
            nxt = self._sample_token(logits, config)
            nxt = nxt.masked_fill(~alive.unsqueeze(-1), config.pad_token_id or 0)
            generated = torch.cat([generated, nxt], dim=-1)
            if config.eos_token_id is not None:
                alive = alive & (nxt.squeeze(-1) != config.eos_token_id)
        return generated

    def _beam_search(self, input_ids: torch.Tensor, config: RuntimeGenerationConfig) -> torch.Tensor:
        B, nb = input_ids.shape[0], config.num_beams
        dev = input_ids.device
        V = self.config.vocab_size
        generated = input_ids.unsqueeze(1).expand(B, nb, -1).reshape(B * nb, -1)
        scores_b = torch.zeros(B * nb, device=dev)
        scores_b.view(B, nb)[:, 1:] = -1e9
        cache = None
        for step in range(config.max_new_tokens):
            logits, cache = self._step_logits(generated if cache is None else generated[:, -1:], cache)
            lp = F.log_softmax(logits, dim=-1)
            if step > 0:
                lp = lp / (step + 1) ** config.length_penalty
            cand = (lp + scores_b.unsqueeze(-1)).view(B, nb * V)
            top_s, top_i = torch.topk(cand, 2 * nb, dim=-1)
            beam_i = (top_i // V).view(-1)
            tok_i = (top_i % V).view(-1)
            base = (torch.arange(B, device=dev).unsqueeze(1) * nb).expand(B, 2 * nb).reshape(-1)
            src = base + beam_i
            scores_b = top_s.view(-1)
            generated = torch.cat([generated[src], tok_i.unsqueeze(-1)], dim=-1)
            cache = self._reorder_cache(cache, src)
            if config.eos_token_id is not None:
                scores_b = scores_b.masked_fill(tok_i == config.eos_token_id, float("-inf"))
            _, best = torch.topk(scores_b.view(B, 2 * nb), nb, dim=-1)
            sel = (best + torch.arange(B, device=dev).unsqueeze(1) * (2 * nb)).view(-1)
            scores_b = scores_b[sel]
            generated = generated[sel]
            cache = self._reorder_cache(cache, sel)
            if config.eos_token_id is not None and bool((tok_i[sel] == config.eos_token_id).all()):
                break
        return generated.view(B, nb, -1)[:, 0, :]

    @staticmethod
    def _reorder_cache(cache, indices):
        if cache is None:
            return None

        def pick(v):
            if isinstance(v, torch.Tensor):
                return v[indices] if v.dim() > 0 else v
            if isinstance(v, dict):
                return {k: pick(x) for k, x in v.items()}
            if isinstance(v, (list, tuple)):
                return type(v)(pick(x) for x in v)
            return v
        return [None if c is None else {k: pick(v) for k, v in c.items()} for c in cache]

    @torch.no_grad()
    def generate_stream(self, input_ids: torch.Tensor,
                        generation_config: Optional[RuntimeGenerationConfig] = None,
                        **kwargs) -> Generator[int, None, None]:
        cfg = self._merge(generation_config, kwargs)
        if input_ids.shape[0] != 1:
            raise ValueError(f"generate_stream only supports batch_size=1, got {input_ids.shape[0]}")
        if cfg.return_full_text:
            for t in input_ids[0].tolist():
                yield t
        generated, cache = input_ids, None
        for _ in range(cfg.max_new_tokens):
            logits, cache = self._step_logits(generated if cache is None else generated[:, -1:], cache)
            if cfg.repetition_penalty != 1.0:
                logits = self._apply_repetition_penalty(logits, generated, cfg.repetition_penalty)
            nxt = self._sample_token(logits, cfg)
            generated = torch.cat([generated, nxt], dim=-1)
            tid = int(nxt[0, 0])
            yield tid
            if cfg.eos_token_id is not None and tid == cfg.eos_token_id:
                break
