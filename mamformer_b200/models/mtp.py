"""Multi-token prediction heads (reference ``mamformer/layers/mtp.py``).

For depth k = 0..D-1 (training only):

* ``prev = input_ids`` for k = 0, else ``labels`` shifted left by k and zero-padded; positions
  equal to -100 get a zero embedding (own ``token_embedding``);
* ``h_k = fuse_k([h_cur, emb(prev)])``; ``h_k = h_k + GQA(n1 h_k) + Mamba(n1 h_k)`` (no gate);
  ``h_k = h_k + SwiGLU_{d_ff/8}(n2 h_k)``;
* logits through the main embedding (tied) or an own head; loss
  ``CE(logits[:, :-(k+1)], labels[:, k+1:])``; the MTP loss is the mean over depths.

Differences from the reference, both deliberate:

* the tied output weight is the live main embedding parameter.  The reference registers it as
  a non-persistent *buffer*, which ``Module.to()`` replaces by a copy, so on a GPU its MTP
  heads read a frozen copy of the initial embedding and send it no gradient;
* on CUDA the logits are never materialised during training: the loss runs in the fused
  linear-cross-entropy kernel path (``ops.linear_cross_entropy``).  ``return_logits=True``
  restores the reference's ``mtp_logits`` output.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamformer_b200 import ops
from mamformer_b200.models.attention import GroupedQueryAttention
from mamformer_b200.models.ffn import SwiGLUFFN
from mamformer_b200.models.mamba2 import Mamba2Block
from mamformer_b200.models.norm import RMSNorm


class MultiTokenPredictor(nn.Module):
    def __init__(self, d_model: int, vocab_size: int, depth: int = 2, n_heads: int = 32,
                 n_kv_heads: int = 8, head_dim: int = 128, d_ff: int = 1152, d_state: int = 128,
                 d_conv: int = 4, max_seq_len: int = 8192, rope_theta: float = 10000.0,
                 dropout: float = 0.0, rms_norm_eps: float = 1e-6,
                 embedding_weight: Optional[torch.Tensor] = None,
                 embedding_module: Optional[nn.Embedding] = None) -> None:
        super().__init__()
        self.d_model = d_model
        self.vocab_size = vocab_size
        self.depth = depth
        self.token_embedding = nn.Embedding(vocab_size, d_model)
        self.mtp_norms_1 = nn.ModuleList([RMSNorm(d_model, eps=rms_norm_eps) for _ in range(depth)])
        self.mtp_attentions = nn.ModuleList([
            GroupedQueryAttention(d_model, n_heads, n_kv_heads, head_dim, max_seq_len, rope_theta,
                                  dropout) for _ in range(depth)])
        self.mtp_ssms = nn.ModuleList([Mamba2Block(d_model, d_state, d_conv, expand=1)
                                       for _ in range(depth)])
        self.mtp_norms_2 = nn.ModuleList([RMSNorm(d_model, eps=rms_norm_eps) for _ in range(depth)])
        self.mtp_ffns = nn.ModuleList([SwiGLUFFN(d_model, d_ff, dropout) for _ in range(depth)])
        tied = embedding_weight is not None or embedding_module is not None
        # The tied embedding is looked up through the owner (not registered as a submodule, so it
        # is neither saved twice nor re-initialised here).
        object.__setattr__(self, "_tied_embedding", embedding_module)
        object.__setattr__(self, "_tied_weight", embedding_weight if embedding_module is None else None)
        self.output_heads = None if tied else nn.ModuleList(
            [nn.Linear(d_model, vocab_size, bias=False) for _ in range(depth)])
        self.fusion_projections = nn.ModuleList([nn.Linear(2 * d_model, d_model, bias=False)
                                                 for _ in range(depth)])
        nn.init.normal_(self.token_embedding.weight, mean=0.0, std=0.02)
        for p in self.fusion_projections:
            nn.init.normal_(p.weight, mean=0.0, std=0.02)
        if self.output_heads is not None:
            for h in self.output_heads:
                nn.init.normal_(h.weight, mean=0.0, std=0.02)
        self.return_logits = False

    def _head_weight(self, k: int) -> torch.Tensor:
        if self.output_heads is not None:
            return self.output_heads[k].weight
        if self._tied_embedding is not None:
            return self._tied_embedding.weight
        return self._tied_weight

    @property
    def _shared_embedding(self) -> torch.Tensor:
        return self._head_weight(0)

    def _block(self, k: int, h_k: torch.Tensor, attention_mask) -> torch.Tensor:
        n1 = self.mtp_norms_1[k](h_k)
        attn, _ = self.mtp_attentions[k](n1, attention_mask=attention_mask, use_cache=False)
        ssm, _ = self.mtp_ssms[k](n1, use_cache=False)
        h_k = h_k + attn + ssm
        return h_k + self.mtp_ffns[k](self.mtp_norms_2[k](h_k))

    def forward(self, hidden_states: torch.Tensor, input_ids: torch.Tensor,
                labels: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                return_logits: Optional[bool] = None) -> Tuple[List[torch.Tensor], Optional[torch.Tensor]]:
        want_logits = self.return_logits if return_logits is None else return_logits
        B, S, d = hidden_states.shape
        logits_list: List[torch.Tensor] = []
        losses: List[torch.Tensor] = []
        h_cur = hidden_states
        for k in range(self.depth):
            if labels is not None and k > 0:
                prev = torch.cat([labels[:, k:], labels.new_zeros(B, k)], dim=1)
            else:
                prev = input_ids
            emb = self.token_embedding(prev.clamp(min=0))
            emb = emb * (prev != -100).unsqueeze(-1).to(emb.dtype)
            fused = torch.cat([h_cur, emb.to(h_cur.dtype)], dim=-1)
            h_k = self._block(k, self.fusion_projections[k](fused), attention_mask)
            W = self._head_weight(k)
            shift = k + 1
            need_loss = labels is not None and S > shift
            if want_logits or labels is None or not ops.fused_ce_available(h_k):
                logits = F.linear(h_k, W.to(h_k.dtype))
                logits_list.append(logits)
                if need_loss:
                    losses.append(F.cross_entropy(
                        logits[:, :-shift].reshape(-1, W.shape[0]).float()
                        if logits.dtype != torch.float32 else logits[:, :-shift].reshape(-1, W.shape[0]),
                        labels[:, shift:].reshape(-1), ignore_index=-100))
            elif need_loss:
                losses.append(ops.linear_cross_entropy(
                    h_k[:, :-shift].reshape(-1, d), W, labels[:, shift:].reshape(-1)))
            h_cur = h_k
        loss = torch.stack(losses).mean() if losses else None
        return logits_list, loss

    def generate_mtp_tokens(self, hidden_states, input_ids, attention_mask=None,
                            temperature: float = 1.0) -> List[torch.Tensor]:
        logits_list, _ = self.forward(hidden_states, input_ids, None, attention_mask, return_logits=True)
        out = []
        for logits in logits_list:
            last = logits[:, -1, :]
            if temperature == 0:
                out.append(last.argmax(-1, keepdim=True))
            else:
                probs = F.softmax(last.float() / temperature, dim=-1)
                out.append(torch.multinomial(probs, 1))
        return out

    def extra_repr(self) -> str:
        return f"d_model={self.d_model}, vocab_size={self.vocab_size}, depth={self.depth}"
