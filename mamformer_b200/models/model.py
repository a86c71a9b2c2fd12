"""MamformerModel (trunk) and MamformerForCausalLM (LM head, losses, generation, GRPO scoring).

Reference: ``mamformer/model.py``.

Trunk (``model.py:74-315``): embedding -> N hybrid blocks -> RMSNorm.  Cross-layer SSM state:
an SSM-only layer's ``h_states`` is held as ``pending`` and handed to the next attention-only
layer, which clears it; fusion layers neither read nor clear it.  Selective activation
checkpointing recomputes only full-attention layers.  Weights: every Linear/Embedding of the
trunk is re-drawn from N(0, initializer_range) after construction, in the reference's module
order, so a seeded build reproduces the reference's initial weights.

Causal LM (``model.py:387-1137``): tied head ``h E^T`` (or an own ``lm_head``), shifted CE,
``loss = main + loss_weight * mtp`` in training, ``generate`` (temperature / top-k / top-p,
repetition penalty, EOS, multi-path thinking), ``get_log_probs`` for GRPO with S-GRPO token
masks, ``_extend_embeddings`` for thinking control tokens.

B200 path: with ``return_logits=False`` (what the training engine uses) the main and MTP losses
run through the fused linear-cross-entropy kernel and the (B, S, V) logits are never
materialised.
"""

from __future__ import annotations

from typing import List, Optional, Union

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as activation_checkpoint

from mamformer_b200.utils.nvtx import rng as nvtx_rng
from mamformer_b200 import ops
from mamformer_b200.config import MamformerConfig
from mamformer_b200.generation import GenerationMixin
from mamformer_b200.models.hybrid import MamformerBlock
from mamformer_b200.models.moe import DeepSeekMoE
from mamformer_b200.models.mtp import MultiTokenPredictor
from mamformer_b200.models.norm import RMSNorm
from mamformer_b200.sampling import apply_repetition_penalty, sample_one_token


def _checkpointed_layer(layer: MamformerBlock, h, attention_mask, kw):
    """Run one layer under non-reentrant activation checkpointing, keeping the cross-layer SSM
    state it emits (a tensor output of the checkpointed function) and its MoE statistics.  The
    recomputation in the backward pass replays the routing of the original forward (the MoE
    layers stash their router bias per call) and does not update routing statistics again."""
    from mamformer_b200.models.moe import routing_replay
    calls = {"n": 0}
    aux: dict = {}
    pend = kw.get("ssm_h_states")
    rest = {k: v for k, v in kw.items() if k != "ssm_h_states"}

    def run(hs, am, ph):
        replay = calls["n"] > 0
        calls["n"] += 1
        extra = dict(rest)
        if ph is not None:
            extra["ssm_h_states"] = ph
        with routing_replay(replay):
            out, entry = layer(hs, attention_mask=am, use_cache=False, cache=None, **extra)
        if not replay and entry is not None and "moe_aux_info" in entry:
            aux["moe_aux_info"] = entry["moe_aux_info"]
        hst = entry.get("ssm_h_states") if entry is not None else None
        return (out, hst) if hst is not None else (out,)

    outs = activation_checkpoint(run, h, attention_mask, pend, use_reentrant=False)
    entry = dict(aux)
    if len(outs) > 1:
        entry["ssm_h_states"] = outs[1]
    return outs[0], (entry or None)


def _is_full_attention_checkpointable(layer: MamformerBlock) -> bool:
    attn = getattr(layer, "attention", None)
    if attn is None:
        return False
    if hasattr(attn, "_is_full_attention_layer"):
        return attn._is_full_attention_layer()
    return True


def reinit_like_reference(root: nn.Module, std: float) -> None:
    """N(0, std) for every Linear/Embedding weight (zero biases), in module order; MoE modules
    re-draw their stacked experts in the order of the reference's per-expert modules."""
    def visit(m: nn.Module):
        if hasattr(m, "reinit_in_reference_order"):
            m.reinit_in_reference_order(std)
            return
        for child in m.children():
            visit(child)
        if isinstance(m, nn.Linear):
            nn.init.normal_(m.weight, mean=0.0, std=std)
            if m.bias is not None:
                nn.init.zeros_(m.bias)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, mean=0.0, std=std)
    with torch.no_grad():
        visit(root)


def block_kwargs(config: MamformerConfig, lt: dict, i: int) -> dict:
    c = config
    return dict(
        d_model=c.d_model, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads, head_dim=c.head_dim,
        d_ff=c.d_ff, d_state=c.mamba.d_state, d_conv=c.mamba.d_conv, mamba_expand=c.mamba.expand,
        max_seq_len=c.max_seq_len, rope_theta=c.rope.theta, dropout=c.dropout,
        rms_norm_eps=c.rms_norm_eps,
        sliding_window=c.sliding_window if c.use_sliding_window else 0,
        has_attention=lt["has_attention"], has_ssm=lt["has_ssm"], layer_idx=i,
        use_dsa=c.dsa.enabled and not c.kda_diff.enabled, dsa_lambda_init=c.dsa.lambda_init,
        dsa_state_injection=c.dsa.use_state_injection,
        use_kda_diff=c.kda_diff.enabled, kda_linear_ratio=c.kda_diff.linear_ratio,
        kda_kernel_dim=c.kda_diff.kernel_dim, kda_latent_dim=c.kda_diff.latent_dim,
        kda_use_dynamic_ratio=c.kda_diff.use_dynamic_ratio,
        rope_use_yarn=c.rope.use_yarn, rope_yarn_scale=c.rope.yarn_scale,
        rope_yarn_original_max_seq_len=c.rope.yarn_original_max_seq_len,
        use_moe=c.moe.enabled and not c.st_moe.enabled, moe_n_shared=c.moe.n_shared_experts,
        moe_n_routed=c.moe.n_routed_experts, moe_top_k=c.moe.top_k,
        moe_shared_dim=c.moe.shared_expert_intermediate_dim,
        moe_routed_dim=c.moe.routed_expert_intermediate_dim,
        moe_aux_loss_free=c.moe.aux_loss_free, moe_bias_speed=c.moe.bias_update_speed,
        use_st_moe=c.st_moe.enabled, st_moe_lambda_init=c.st_moe.lambda_init,
        st_moe_lambda_max=c.st_moe.lambda_max, st_moe_learnable_lambda=c.st_moe.learnable_lambda,
        st_moe_use_balance_lock=c.st_moe.use_balance_lock,
        st_moe_balance_lock_threshold=c.st_moe.balance_lock_threshold,
        use_communicative_moe=c.communicative_moe.enabled,
        comm_moe_n_heads=c.communicative_moe.n_comm_heads,
        comm_moe_depth=c.communicative_moe.comm_depth,
        comm_moe_dropout=c.communicative_moe.comm_dropout,
        window_mode=getattr(c, "window_mode", "reference"),
    )


def _h_states_consumers(layer_types: List[dict]) -> List[bool]:
    """For each SSM-only layer: will a later attention-only layer read its h_states?"""
    needed = [False] * len(layer_types)
    for i, lt in enumerate(layer_types):
        if lt["has_attention"] or not lt["has_ssm"]:
            continue
        for j in range(i + 1, len(layer_types)):
            lj = layer_types[j]
            if lj["has_attention"] and not lj["has_ssm"]:
                needed[i] = True
                break
            if not lj["has_attention"] and lj["has_ssm"]:
                break
    return needed


class MamformerModel(nn.Module):
    def __init__(self, config: MamformerConfig) -> None:
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.d_model)
        layer_types = config.layer_types()
        self.layers = nn.ModuleList()
        attn_counter = 0
        consumed = _h_states_consumers(layer_types)
        for i, lt in enumerate(layer_types):
            layer = MamformerBlock(**block_kwargs(config, lt, i))
            layer.h_states_needed = consumed[i]
            self.layers.append(layer)
            if lt["has_attention"] and config.kda_diff.enabled:
                if hasattr(layer.attention, "set_layer_idx"):
                    layer.attention.set_layer_idx(i, attn_counter)
                attn_counter += 1
        self.norm = RMSNorm(config.d_model, eps=config.rms_norm_eps)
        self.gradient_checkpointing = False
        self.checkpoint_all = False
        reinit_like_reference(self, config.initializer_range)

    def _init_weights(self, module: nn.Module) -> None:
        std = self.config.initializer_range
        if isinstance(module, DeepSeekMoE):
            module.reinit_in_reference_order(std)
        elif isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=std)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=std)

    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                use_cache: bool = False, cache: Optional[List[dict]] = None,
                rope_offset: int = 0) -> dict:
        h = self.embed_tokens(input_ids)
        if attention_mask is not None and attention_mask.dim() == 2:
            m = attention_mask[:, None, None, :].to(h.dtype)
            attention_mask = (1.0 - m) * torch.finfo(h.dtype).min
        h, _, new_caches, aux_list = self.run_layers(h, attention_mask, 0, len(self.layers), None,
                                                     use_cache, cache, rope_offset)
        h = self.norm(h)
        out = {"last_hidden_state": h}
        if use_cache:
            out["cache"] = new_caches
        if aux_list:
            out["moe_aux_info"] = aux_list
        return out

    def run_layers(self, h: torch.Tensor, attention_mask: Optional[torch.Tensor], start: int, end: int,
                   pending: Optional[torch.Tensor] = None, use_cache: bool = False,
                   cache: Optional[List[dict]] = None, rope_offset: int = 0):
        """Layers [start, end) with cross-layer SSM-state passing (``model.py:237-297``): an
        SSM-only layer's per-step state is handed to the next attention-only layer.  Returns
        (hidden, pending state, caches, MoE aux list); the pipeline stages call this on their
        slice and ship ``pending`` with the activations."""
        per_layer = cache if cache is not None else [None] * len(self.layers)
        new_caches: List[dict] = []
        aux_list: List[dict] = []
        for idx in range(start, end):
            layer = self.layers[idx]
            lc = per_layer[idx] if idx < len(per_layer) else None
            kw: dict = {}
            attn_only = layer.has_attention and not layer.has_ssm
            if attn_only and pending is not None:
                kw["ssm_h_states"] = pending
            if rope_offset:
                kw["rope_offset"] = rope_offset
            with nvtx_rng(f"layer{idx}"):
                if self.gradient_checkpointing and self.training and self.checkpoint_all and not use_cache:
                    h, entry = _checkpointed_layer(layer, h, attention_mask, kw)
                elif (self.gradient_checkpointing and self.training and layer.has_attention
                        and _is_full_attention_checkpointable(layer)):
                    def run(hs, am, _layer=layer, _kw=kw):
                        return _layer(hs, attention_mask=am, use_cache=False, cache=None, **_kw)[0]
                    h = activation_checkpoint(run, h, attention_mask, use_reentrant=False)
                    entry = None
                else:
                    h, entry = layer(h, attention_mask=attention_mask, use_cache=use_cache, cache=lc, **kw)
            if not layer.has_attention and layer.has_ssm and entry is not None and "ssm_h_states" in entry:
                pending = entry["ssm_h_states"]
            if attn_only and kw.get("ssm_h_states") is not None:
                pending = None
            if use_cache:
                new_caches.append(entry)
            if entry is not None and "moe_aux_info" in entry:
                aux_list.append(entry["moe_aux_info"])
        return h, pending, new_caches, aux_list

    def enable_gradient_checkpointing(self, all_layers: bool = False) -> None:
        """Recompute activations in the backward pass.  Default: the reference's selective form
        (full-attention layers only, ``model.py:252-277``).  ``all_layers=True``: every layer
        keeps only its input and recomputes the rest, the form that lets the full 32-layer MoE
        models fit; MoE layers then replay their original routing during the recomputation."""
        self.gradient_checkpointing = True
        self.checkpoint_all = bool(all_layers)

    def disable_gradient_checkpointing(self) -> None:
        self.gradient_checkpointing = False

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def print_parameter_summary(self) -> None:
        total = self.num_parameters()
        emb = self.embed_tokens.weight.numel()
        layer_p = sum(p.numel() for l in self.layers for p in l.parameters())
        n_f = sum(1 for l in self.layers if l.is_fusion)
        n_a = sum(1 for l in self.layers if l.has_attention and not l.has_ssm)
        n_s = sum(1 for l in self.layers if l.has_ssm and not l.has_attention)
        attn = sum(p.numel() for l in self.layers if l.attention is not None for p in l.attention.parameters())
        ssm = sum(p.numel() for l in self.layers if l.ssm is not None for p in l.ssm.parameters())
        ffn = sum(p.numel() for l in self.layers for p in l.ffn.parameters())
        bar = "=" * 55
        print(bar)
        print("  Mamformer Model Parameter Summary")
        print(bar)
        print(f"  Embedding:     {emb:>15,}")
        print(f"  Layers: {n_f} fusion, {n_a} attn-only, {n_s} SSM-only (x{len(self.layers)} total)")
        print(f"    Attention:   {attn // max(1, n_f + n_a):>15,}")
        print(f"    SSM:         {ssm // max(1, n_f + n_s):>15,}")
        print(f"    FFN:         {ffn // max(1, len(self.layers)):>15,}")
        print(f"  Layers (x{len(self.layers)}):  {layer_p:>15,}")
        print(bar)
        print(f"  Total:         {total:>15,}")
        print(f"  Total (B):     {total / 1e9:>14.2f}B")
        print(bar)


class MamformerForCausalLM(GenerationMixin, nn.Module):
    def __init__(self, config: MamformerConfig) -> None:
        super().__init__()
        self.config = config
        self.model = MamformerModel(config)
        if config.tie_word_embeddings:
            self.lm_head = None
        else:
            self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False)
            nn.init.normal_(self.lm_head.weight, mean=0.0, std=config.initializer_range)
        self.mtp = None
        if config.mtp.enabled:
            mtp_dim = config.mtp.mtp_d_model or config.d_model
            self.mtp = MultiTokenPredictor(
                d_model=mtp_dim, vocab_size=config.vocab_size, depth=config.mtp.depth,
                n_heads=config.n_heads, n_kv_heads=config.n_kv_heads, head_dim=config.head_dim,
                d_ff=config.d_ff // 8, d_state=config.mamba.d_state, d_conv=config.mamba.d_conv,
                max_seq_len=config.max_seq_len, rope_theta=config.rope.theta, dropout=config.dropout,
                rms_norm_eps=config.rms_norm_eps,
                embedding_module=self.model.embed_tokens if config.tie_word_embeddings else None)
        self._embeddings_extended = False
        # True: return (B, S, V) logits like the reference.  False: losses via the fused
        # linear-cross-entropy path and no logits (the training engine's setting).
        self.return_logits = True

    # -- head ------------------------------------------------------------------------------
    @property
    def output_weight(self) -> torch.Tensor:
        return self.lm_head.weight if self.lm_head is not None else self.model.embed_tokens.weight

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        W = self.output_weight
        return F.linear(hidden, W.to(hidden.dtype))

    def _extend_embeddings(self, new_vocab_size: int) -> None:
        cur = self.config.vocab_size
        if new_vocab_size <= cur:
            return
        n_new, d = new_vocab_size - cur, self.config.d_model
        old = self.model.embed_tokens.weight.data
        mean = old.float().mean(0, keepdim=True)
        rows = (mean.repeat(n_new, 1) + torch.randn(n_new, d, device=old.device) * 0.02).to(old.dtype)
        emb = nn.Embedding(new_vocab_size, d, device=old.device, dtype=old.dtype)
        emb.weight.data.copy_(torch.cat([old, rows], 0))
        self.model.embed_tokens = emb
        if self.lm_head is not None:
            oh = self.lm_head.weight.data
            rows_h = (mean.repeat(n_new, 1) + torch.randn(n_new, d, device=oh.device) * 0.02).to(oh.dtype)
            head = nn.Linear(d, new_vocab_size, bias=False, device=oh.device, dtype=oh.dtype)
            head.weight.data.copy_(torch.cat([oh, rows_h], 0))
            self.lm_head = head
        if self.mtp is not None and self.mtp.output_heads is None:
            object.__setattr__(self.mtp, "_tied_embedding", self.model.embed_tokens)
        self.config.vocab_size = new_vocab_size
        self._embeddings_extended = True

    def _ensure_thinking_tokens(self) -> None:
        from mamformer_b200.tokenizer import MamformerTokenizer
        need = MamformerTokenizer.SUMMARY_START_ID + 1
        if self.config.vocab_size < need:
            self._extend_embeddings(need)

    # -- forward ---------------------------------------------------------------------------
    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                labels: Optional[torch.Tensor] = None, use_cache: bool = False,
                cache: Optional[List[dict]] = None, return_logits: Optional[bool] = None,
                rope_offset: int = 0) -> dict:
        want_logits = self.return_logits if return_logits is None else return_logits
        out = self.model(input_ids=input_ids, attention_mask=attention_mask, use_cache=use_cache,
                         cache=cache, rope_offset=rope_offset)
        h = out["last_hidden_state"]
        result: dict = {}
        if use_cache:
            result["cache"] = out.get("cache")
        if "moe_aux_info" in out:
            result["moe_aux_info"] = out["moe_aux_info"]
        return self.compute_head(h, input_ids, labels, attention_mask, want_logits, result)

    def compute_head(self, h: torch.Tensor, input_ids: torch.Tensor, labels: Optional[torch.Tensor],
                     attention_mask: Optional[torch.Tensor], want_logits: bool, result: dict) -> dict:
        """Tied LM head, shifted CE and the MTP loss on the final hidden state (also the last
        pipeline stage's head)."""
        fused = (labels is not None and not want_logits and ops.fused_ce_available(h))
        main_loss = None
        if fused:
            V = self.output_weight.shape[0]
            hs = h[:, :-1].reshape(-1, h.shape[-1])
            main_loss = ops.linear_cross_entropy(hs, self.output_weight, labels[:, 1:].reshape(-1))
            result["logits"] = None
        else:
            logits = self.compute_logits(h)
            result["logits"] = logits
            if labels is not None:
                V = logits.shape[-1]
                sl = logits[..., :-1, :].reshape(-1, V)
                main_loss = F.cross_entropy(sl if sl.dtype == torch.float32 else sl.float(),
                                            labels[..., 1:].reshape(-1), ignore_index=-100)
        mtp_loss = None
        if self.mtp is not None and self.training:
            mtp_logits, mtp_loss = self.mtp(h, input_ids, labels, attention_mask,
                                            return_logits=want_logits or labels is None)
            if mtp_logits:
                result["mtp_logits"] = mtp_logits
        if main_loss is not None:
            if mtp_loss is not None:
                result["loss"] = main_loss + self.config.mtp.loss_weight * mtp_loss
                result["main_loss"] = main_loss.detach()
                result["mtp_loss"] = mtp_loss.detach()
            else:
                result["loss"] = main_loss
        return result

    # -- generation ------------------------------------------------------------------------
    def _sample_from_logits(self, logits, temperature, top_k, top_p) -> torch.Tensor:
        return sample_one_token(logits, temperature=temperature, top_k=top_k, top_p=top_p)

    def _gen_defaults(self, max_new_tokens, temperature, top_k, top_p):
        g = self.config.generation
        return (g.max_output_tokens if max_new_tokens is None else max_new_tokens,
                g.default_temperature if temperature is None else temperature,
                g.default_top_k if top_k is None else top_k,
                g.default_top_p if top_p is None else top_p)

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: Optional[int] = None,
                 temperature: Optional[float] = None, top_k: Optional[int] = None,
                 top_p: Optional[float] = None, eos_token_id: Optional[int] = None,
                 pad_token_id: Optional[int] = None,
                 thinking_config: Optional[object] = None) -> Union[torch.Tensor, dict]:
        if (thinking_config is not None and getattr(thinking_config, "enabled", False)
                and getattr(thinking_config, "is_active", False)):
            self._ensure_thinking_tokens()
            return self._generate_with_thinking(input_ids, max_new_tokens, temperature, top_k,
                                                top_p, eos_token_id, pad_token_id, thinking_config)
        max_new_tokens, temperature, top_k, top_p = self._gen_defaults(
            max_new_tokens, temperature, top_k, top_p)
        rep = self.config.generation.repetition_penalty
        B = input_ids.shape[0]
        generated = input_ids.clone()
        cache = None
        alive = torch.ones(B, dtype=torch.bool, device=input_ids.device)
        for _ in range(max_new_tokens):
            if not bool(alive.any()):
                break
            cur = generated if cache is None else generated[:, -1:]
            out = self.forward(cur, use_cache=True, cache=cache, return_logits=True)
            logits = out["logits"][:, -1, :].float()
            cache = out.get("cache")
            if rep != 1.0:
                logits = apply_repetition_penalty(logits, generated, rep)
            nxt = self._sample_from_logits(logits, temperature, top_k, top_p)
            nxt = nxt.masked_fill(~alive.unsqueeze(-1), 0 if pad_token_id is None else pad_token_id)
            generated = torch.cat([generated, nxt], dim=-1)
            if eos_token_id is not None:
                alive = alive & (nxt.squeeze(-1) != eos_token_id)
        return generated

    @torch.no_grad()
    def _expand_cache_batch(self, cache: Optional[List[dict]], n: int) -> Optional[List[dict]]:
        if cache is None:
            return None

        def grow(v):
            if isinstance(v, torch.Tensor) and v.dim() > 0 and v.shape[0] == 1:
                return v.expand(n, *v.shape[1:]).clone()
            if isinstance(v, dict):
                return {k: grow(x) for k, x in v.items()}
            return v
        return [None if c is None else {k: grow(v) for k, v in c.items()} for c in cache]

    @torch.no_grad()
    def _generate_thinking_paths_batched(self, prompt_cache, base_sequence, think_start_id,
                                         think_end_id, think_budget, temperature, top_k, top_p,
                                         rep_penalty, num_paths, device):
        caches = self._expand_cache_batch(prompt_cache, num_paths)
        tokens: List[List[int]] = [[] for _ in range(num_paths)]
        done = [False] * num_paths
        hit_end = [False] * num_paths
        for step in range(think_budget):
            if all(done):
                break
            if step == 0:
                cur = torch.full((num_paths, 1), think_start_id, dtype=torch.long, device=device)
            else:
                cur = torch.tensor([[t[-1]] for t in tokens], dtype=torch.long, device=device)
            out = self.forward(cur, use_cache=True, cache=caches, return_logits=True)
            logits = out["logits"][:, -1, :].float()
            caches = out.get("cache")
            if rep_penalty != 1.0:
                for p in range(num_paths):
                    if not done[p] and tokens[p]:
                        ids = torch.tensor(sorted(set(tokens[p])), device=device)
                        row = logits[p, ids]
                        logits[p, ids] = torch.where(row > 0, row / rep_penalty, row * rep_penalty)
            nxt = self._sample_from_logits(logits, temperature, top_k, top_p)
            for p in range(num_paths):
                if done[p]:
                    continue
                tid = int(nxt[p, 0])
                tokens[p].append(tid)
                if tid == think_end_id:
                    hit_end[p] = done[p] = True
                elif step >= think_budget - 1:
                    done[p] = True
        for p in range(num_paths):
            if not hit_end[p]:
                tokens[p].append(think_end_id)
        seq = base_sequence.clone()
        for p in range(num_paths):
            seq = torch.cat([seq, torch.tensor([[think_start_id] + tokens[p]], dtype=torch.long,
                                               device=device)], dim=-1)
        return tokens, seq

    @torch.no_grad()
    def _generate_with_thinking(self, input_ids, max_new_tokens, temperature, top_k, top_p,
                                eos_token_id, pad_token_id, thinking_config) -> dict:
        from mamformer_b200.thinking import MultiPathController
        max_new_tokens, temperature, top_k, top_p = self._gen_defaults(
            max_new_tokens, temperature, top_k, top_p)
        tc = thinking_config
        B = input_ids.shape[0]
        dev = input_ids.device
        rep = self.config.generation.repetition_penalty
        budget, summary_budget, n_paths = tc.effective_budget, tc.effective_summary_budget, tc.effective_num_paths
        ctl = MultiPathController(tc)
        generated = input_ids.clone()
        prompt_cache = self.forward(generated, use_cache=True, return_logits=True).get("cache")
        paths, generated = self._generate_thinking_paths_batched(
            prompt_cache, generated, tc.think_start_token_id, tc.think_end_token_id, budget,
            temperature, top_k, top_p, rep, n_paths, dev)
        total_think = sum(len(t) for t in paths)
        for p in range(n_paths):
            ctl.start_path(p)
            for tid in paths[p]:
                ctl.record_path_token(p, tid)
        generated = torch.cat([generated, torch.full((B, 1), tc.summary_start_token_id,
                                                     dtype=torch.long, device=dev)], -1)
        ctl.start_summary()
        recent = generated[:, -(n_paths * 2 + 1):] if generated.shape[1] > n_paths * 2 else generated
        cache = self.forward(recent, use_cache=True, cache=prompt_cache, return_logits=True).get("cache")
        for _ in range(summary_budget):
            out = self.forward(generated[:, -1:], use_cache=True, cache=cache, return_logits=True)
            logits = out["logits"][:, -1, :].float()
            cache = out.get("cache")
            if rep != 1.0:
                logits = apply_repetition_penalty(logits, generated, rep)
            nxt = self._sample_from_logits(logits, temperature, top_k, top_p)
            ev = ctl.record_summary_token(int(nxt[0, 0]))
            generated = torch.cat([generated, nxt], -1)
            if ev == "end_summary":
                break
        generated = torch.cat([generated, torch.full((B, 1), tc.answer_start_token_id,
                                                     dtype=torch.long, device=dev)], -1)
        ctl.start_answer()
        remaining = max_new_tokens - total_think - summary_budget - (n_paths * 2 + 3)
        alive = torch.ones(B, dtype=torch.bool, device=dev)
        for _ in range(max(remaining, 1)):
            if not bool(alive.any()):
                break
            out = self.forward(generated[:, -1:], use_cache=True, cache=cache, return_logits=True)
            logits = out["logits"][:, -1, :].float()
            cache = out.get("cache")
            if rep != 1.0:
                logits = apply_repetition_penalty(logits, generated, rep)
            nxt = self._sample_from_logits(logits, temperature, top_k, top_p)
            ev = ctl.record_answer_token(int(nxt[0, 0]))
            nxt = nxt.masked_fill(~alive.unsqueeze(-1), 0 if pad_token_id is None else pad_token_id)
            generated = torch.cat([generated, nxt], -1)
            if eos_token_id is not None:
                alive = alive & (nxt.squeeze(-1) != eos_token_id)
            if ev == "end_answer":
                break
        info = ctl.finalize()
        t = lambda xs: torch.tensor([xs], dtype=torch.long, device=dev)  # noqa: E731
        return {"generated_ids": generated, "all_paths": [t(x) for x in info["all_paths"]],
                "path_counts": info["path_counts"], "summary_ids": t(info["summary_tokens"]),
                "answer_ids": t(info["answer_tokens"]), "total_think_tokens": info["total_think_tokens"],
                "num_paths": n_paths, "budget_forced": any(info["path_budget_forced"])}

    # -- GRPO scoring ----------------------------------------------------------------------
    def get_log_probs(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None,
                      attention_mask: Optional[torch.Tensor] = None,
                      token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Per-token log p(input_ids[t+1] | <= t); with labels, the mean over response tokens
        (labels != -100, optionally AND token_mask) per sequence."""
        out = self.forward(input_ids, attention_mask=attention_mask, use_cache=False, return_logits=True)
        logits = out["logits"][:, :-1, :]
        tgt = input_ids[:, 1:]
        tok_lp = ops.token_log_probs(logits, tgt.clamp(min=0))
        tok_lp = tok_lp.masked_fill(tgt == -100, 0.0)
        if labels is None:
            return tok_lp
        mask = (labels[:, 1:] != -100).float()
        if token_mask is not None:
            mask = mask * token_mask.float()
        return (tok_lp * mask).sum(1) / mask.sum(1).clamp(min=1)

    # -- info ------------------------------------------------------------------------------
    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def num_parameters_billions(self) -> float:
        return self.num_parameters() / 1e9

    def print_parameter_summary(self) -> None:
        total = self.num_parameters()
        bar = "=" * 55
        emb = self.model.embed_tokens.weight.numel()
        layer_p = sum(p.numel() for l in self.model.layers for p in l.parameters())
        print(bar)
        print("  Mamformer Model Parameter Summary")
        print(bar)
        print(f"  Embedding:     {emb:>15,}")
        print(f"  Layers (x{self.config.n_layers}): {layer_p:>15,}")
        if self.lm_head is not None:
            print(f"  LM Head:       {self.lm_head.weight.numel():>15,}")
        if self.mtp is not None:
            print(f"  MTP Heads:     {sum(p.numel() for p in self.mtp.parameters()):>15,}")
        print(bar)
        print(f"  Total:         {total:>15,}")
        print(f"  Total (B):     {total / 1e9:>14.2f}B")
        print(bar)
