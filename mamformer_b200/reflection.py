"""Trainable self-reflection head: critique logits, refined logits and a confidence score.

Reference: ``mamformer/reflection.py`` (``ReflectionModule`` 53-264, ``SelfReflectiveGenerator``
267-374, ``add_reflection_to_model`` 377-396).  Same architecture and parameter names (so the
state dicts load in both frameworks): the response summary is ``RMSNorm(mean_t h_t +
mean_t E_c[token_t])`` through a d -> d/4 -> d SiLU MLP; critique logits project the summary on
``critique_weight``; refined logits project ``MLP([h_t, summary])`` on ``refine_weight``; the
confidence is ``sigmoid(w . summary)``.  Loss: CE(refined) + 0.1 * MSE(confidence, fraction of
tokens whose refined CE beats the original CE).  ``compute_reflection_loss`` returns tensors in
its aux dict (the caller decides when to synchronise).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamformer_b200.models.norm import RMSNorm
from mamformer_b200.sampling import sample_one_token


def _mlp(d_in: int, d_hid: int, d_out: int) -> nn.Sequential:
    return nn.Sequential(nn.Linear(d_in, d_hid, bias=False), nn.SiLU(), nn.Linear(d_hid, d_out, bias=False))


class ReflectionModule(nn.Module):
    def __init__(self, d_model: int, vocab_size: int, max_reflection_tokens: int = 128,
                 embedding_weight: Optional[torch.Tensor] = None):
        super().__init__()
        self.d_model, self.vocab_size = d_model, vocab_size
        self.max_reflection_tokens = max_reflection_tokens
        self.reflection_norm = RMSNorm(d_model)
        self.reflection_proj = _mlp(d_model, d_model // 4, d_model)

        def table():
            if embedding_weight is not None:
                return nn.Parameter(embedding_weight.detach().clone())
            w = nn.Parameter(torch.empty(vocab_size, d_model))
            nn.init.normal_(w, std=0.02)
            return w
        self.critique_weight = table()
        self.refine_adapter = _mlp(2 * d_model, d_model, d_model)
        self.refine_weight = table()
        self.confidence = nn.Sequential(nn.Linear(d_model, 1, bias=False), nn.Sigmoid())
        for seq in (self.reflection_proj, self.refine_adapter):
            for m in seq:
                if isinstance(m, nn.Linear):
                    nn.init.normal_(m.weight, std=0.02)
        nn.init.normal_(self.confidence[0].weight, std=0.02)

    def forward(self, hidden_states: torch.Tensor, generated_tokens: torch.Tensor,
                attention_mask: Optional[torch.Tensor] = None) -> dict:
        S = hidden_states.shape[1]
        tok = F.embedding(generated_tokens, self.critique_weight).mean(1)
        summary = self.reflection_proj(self.reflection_norm(hidden_states.mean(1) + tok))
        critique = F.linear(summary.unsqueeze(1), self.critique_weight)
        joint = torch.cat([hidden_states, summary.unsqueeze(1).expand(-1, S, -1)], -1)
        refined = F.linear(self.refine_adapter(joint), self.refine_weight)
        return {"refined_logits": refined, "critique_logits": critique,
                "confidence": self.confidence(summary), "reflection_summary": summary}

    def compute_reflection_loss(self, original_logits: torch.Tensor, refined_logits: torch.Tensor,
                                labels: torch.Tensor, confidence: torch.Tensor) -> Tuple[torch.Tensor, dict]:
        B = labels.shape[0]
        V = self.vocab_size
        lab = labels[..., 1:].reshape(-1)
        ref_rows = refined_logits[..., :-1, :].reshape(-1, V)
        refine_loss = F.cross_entropy(ref_rows, lab, ignore_index=-100)
        with torch.no_grad():
            orig = F.cross_entropy(original_logits[..., :-1, :].reshape(-1, V), lab, ignore_index=-100,
                                   reduction="none")
            new = F.cross_entropy(ref_rows, lab, ignore_index=-100, reduction="none")
            valid = (lab != -100).float()
            better = ((new < orig).float() * valid).view(B, -1).sum(1) / valid.view(B, -1).sum(1).clamp(min=1)
        conf_loss = F.mse_loss(confidence.squeeze(-1), better)
        return refine_loss + 0.1 * conf_loss, {
            "refine_loss": refine_loss.detach(), "conf_loss": conf_loss.detach(),
            "avg_confidence": confidence.detach().mean(), "improvement_rate": better.mean()}


class SelfReflectiveGenerator:
    """generate -> reflect -> keep the refined continuation when the confidence clears a threshold."""

    def __init__(self, model, reflection_module: ReflectionModule, tokenizer):
        self.model, self.reflection, self.tokenizer = model, reflection_module, tokenizer

    @torch.no_grad()
    def generate_with_reflection(self, input_ids: torch.Tensor, max_new_tokens: int = 256, temperature: float = 0.7,
                                 top_k: int = 50, top_p: float = 0.9, reflection_threshold: float = 0.3):
        first = self.model.generate(input_ids=input_ids, max_new_tokens=max_new_tokens, temperature=temperature,
                                    top_k=top_k, top_p=top_p, eos_token_id=self.tokenizer.eos_token_id)
        h = self.model.model(input_ids=first, use_cache=False)["last_hidden_state"]
        p = input_ids.shape[1]
        gen_h = h[:, p:] if h.shape[1] > p else h
        out = self.reflection(hidden_states=gen_h.to(self.reflection.critique_weight.dtype),
                              generated_tokens=first[:, p:])
        conf = float(out["confidence"].mean())
        use = conf > reflection_threshold
        if use:
            lg = out["refined_logits"]
            ids = sample_one_token(lg.reshape(-1, lg.shape[-1]), temperature=temperature, top_k=top_k,
                                   top_p=1.0).view(lg.shape[0], -1)
            final = torch.cat([input_ids, ids], -1)
        else:
            final = first
        return final, {"used_reflection": use, "confidence": conf, "threshold": reflection_threshold,
                       "initial_length": first.shape[1] - p, "final_length": final.shape[1] - p}


def add_reflection_to_model(model, vocab_size: int, max_reflection_tokens: int = 128):
    emb = model.model.embed_tokens.weight if model.config.tie_word_embeddings else None
    model.reflection = ReflectionModule(model.config.d_model, vocab_size, max_reflection_tokens, emb)
    return model
