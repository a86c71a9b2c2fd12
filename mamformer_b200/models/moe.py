"""DeepSeek-style MoE: shared SwiGLU experts + routed top-k SwiGLU experts.

Reference: ``mamformer/layers/moe.py``.  Semantics kept:

* router ``Linear(d, E, bias=False)`` (init std ``0.02/sqrt(E)``), optional temperature;
* in training with ``aux_loss_free``, the load-balancing bias is added to the scores *before*
  top-k and the gates are the softmax of the biased top-k scores (``moe.py:171-183``);
* output ``sum(shared(x)) + sum_k gate_k * expert_{idx_k}(x)``;
* after each training forward: ``bias -= speed * sign(count/(T k) - 1/E)`` and
  ``ema = 0.99 ema + 0.01 load`` (``moe.py:335-347``); ``_expert_counts`` and
  ``_total_tokens`` accumulate.

B200 design: the routed experts are stored *stacked* - ``routed_gate_proj`` (E, I, d),
``routed_up_proj`` (E, I, d), ``routed_down_proj`` (E, d, I) - so that one grouped GEMM serves
all experts (native kernel on CUDA) and one optimizer launch updates them.  State-dict hooks
write and read the reference's per-expert keys ``routed_experts.{e}.{gate,up,down}_proj.weight``
so checkpoints are interchangeable.  When expert parallelism shards the experts, a module
holds the global range ``[expert_offset, expert_offset + n_local)`` and its state dict uses
global expert indices.

Deviation: ``aux_info`` values are 0-dim tensors instead of Python floats (the reference calls
``.item()`` twice per MoE layer per forward, which blocks the host).
"""

from __future__ import annotations

import collections
import contextlib
import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamformer_b200 import ops
from mamformer_b200.ops.linear import linear as _native_linear


class _SwiGLUExpert(nn.Module):
    """One SwiGLU expert (used for shared experts)."""

    def __init__(self, d_model: int, intermediate_dim: int, dropout: float = 0.0) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(d_model, intermediate_dim, bias=False)
        self.up_proj = nn.Linear(d_model, intermediate_dim, bias=False)
        self.down_proj = nn.Linear(intermediate_dim, d_model, bias=False)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        for p in (self.gate_proj, self.up_proj, self.down_proj):
            nn.init.normal_(p.weight, mean=0.0, std=0.02)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(self.dropout(ops.swiglu(self.gate_proj(x), self.up_proj(x))))


class _RoutedExpertView(nn.Module):
    """Read-only per-expert view (``moe.routed_experts[e](x)``) over the stacked weights."""

    def __init__(self, owner: "DeepSeekMoE", e: int):
        super().__init__()
        object.__setattr__(self, "_owner", owner)
        self.e = e

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        o = self._owner
        i = self.e - o.expert_offset
        g = F.linear(x, o.routed_gate_proj[i].to(x.dtype))
        u = F.linear(x, o.routed_up_proj[i].to(x.dtype))
        return F.linear(ops.swiglu(g, u), o.routed_down_proj[i].to(x.dtype))


class _RoutedExpertList:
    def __init__(self, owner: "DeepSeekMoE"):
        self._owner = owner

    def __len__(self):
        return self._owner.n_local_experts

    def __getitem__(self, e: int) -> _RoutedExpertView:
        return _RoutedExpertView(self._owner, e)

    def __iter__(self):
        o = self._owner
        return (self[e] for e in range(o.expert_offset, o.expert_offset + o.n_local_experts))


# Routing replay for activation checkpointing of whole layers: the original forward ("record")
# stashes the routing state it used (router bias, and any other state a subclass names) in
# first-in first-out order per module; the recomputation in the backward pass ("replay") routes
# with the stashed state and leaves the routing statistics alone, so it reproduces the original
# top-k choice exactly even if other micro-batches moved the bias in between.
_ROUTING_MODE: list = [None]


@contextlib.contextmanager
def routing_replay(replay: bool):
    _ROUTING_MODE.append("replay" if replay else "record")
    try:
        yield
    finally:
        _ROUTING_MODE.pop()


def _routing_mode():
    return _ROUTING_MODE[-1]


# Expert slice to allocate at construction (expert-parallel models too large to build whole):
# inside ``build_expert_slice(rank, size)`` every DeepSeekMoE allocates and initialises only the
# routed experts [rank * E/size, (rank + 1) * E/size).
_BUILD_SLICE: list = [None]


@contextlib.contextmanager
def build_expert_slice(rank: int, size: int):
    _BUILD_SLICE.append((int(rank), int(size)))
    try:
        yield
    finally:
        _BUILD_SLICE.pop()


class DeepSeekMoE(nn.Module):
    def __init__(self, d_model: int, n_shared_experts: int = 2, shared_expert_dim: int = 2304,
                 n_routed_experts: int = 64, top_k: int = 8, routed_expert_dim: int = 576,
                 router_temperature: float = 1.0, aux_loss_free: bool = True,
                 bias_update_speed: float = 0.001, dropout: float = 0.0) -> None:
        super().__init__()
        self.d_model = d_model
        self.n_shared_experts = n_shared_experts
        self.shared_expert_dim = shared_expert_dim
        self.n_routed_experts = n_routed_experts
        self.top_k = top_k
        self.routed_expert_dim = routed_expert_dim
        self.router_temperature = router_temperature
        self.aux_loss_free = aux_loss_free
        self.bias_update_speed = bias_update_speed
        self.dropout_rate = dropout
        self.expert_offset = 0
        self.n_local_experts = n_routed_experts
        sl = _BUILD_SLICE[-1]
        if sl is not None:
            if n_routed_experts % sl[1]:
                raise ValueError(f"{n_routed_experts} routed experts do not split over {sl[1]} ranks")
            self.n_local_experts = n_routed_experts // sl[1]
            self.expert_offset = sl[0] * self.n_local_experts
        # Optional expert-parallel engine (set by parallel.expert_parallel.shard_experts_ep).
        self.ep_engine = None

        self.shared_experts = nn.ModuleList(
            [_SwiGLUExpert(d_model, shared_expert_dim, dropout) for _ in range(n_shared_experts)])
        I = routed_expert_dim
        El = self.n_local_experts
        self.routed_gate_proj = nn.Parameter(torch.empty(El, I, d_model))
        self.routed_up_proj = nn.Parameter(torch.empty(El, I, d_model))
        self.routed_down_proj = nn.Parameter(torch.empty(El, d_model, I))
        self._init_routed_like_reference(construct=True)
        self.router = nn.Linear(d_model, n_routed_experts, bias=False)
        if aux_loss_free:
            self.register_buffer("expert_bias", torch.zeros(n_routed_experts))
            self.register_buffer("expert_load_ema", torch.ones(n_routed_experts) / n_routed_experts)
        self.register_buffer("_total_tokens", torch.zeros(1, dtype=torch.long))
        self.register_buffer("_expert_counts", torch.zeros(n_routed_experts, dtype=torch.long))
        nn.init.normal_(self.router.weight, mean=0.0, std=0.02 / n_routed_experts ** 0.5)
        self.register_state_dict_post_hook(DeepSeekMoE._split_routed_state)
        self.register_load_state_dict_pre_hook(DeepSeekMoE._stack_routed_state)

    # -- initialisation in the reference's RNG order ---------------------------------------
    def _init_routed_like_reference(self, construct: bool, std: float = 0.02) -> None:
        """Consume the CPU RNG exactly like E separately-constructed ``_SwiGLUExpert`` s.

        ``construct=True``: per expert, three ``nn.Linear`` default inits (kaiming-uniform)
        then three ``normal_(0, 0.02)``.  ``construct=False``: per expert, the three
        ``normal_(0, std)`` of a model-wide re-initialisation."""
        with torch.no_grad():
            for e in range(self.routed_gate_proj.shape[0]):
                mats = (self.routed_gate_proj[e], self.routed_up_proj[e], self.routed_down_proj[e])
                if construct:
                    for m in mats:
                        nn.init.kaiming_uniform_(m, a=math.sqrt(5))
                    for m in mats:
                        nn.init.normal_(m, mean=0.0, std=0.02)
                else:
                    for m in mats:
                        nn.init.normal_(m, mean=0.0, std=std)

    def reinit_in_reference_order(self, std: float) -> None:
        """Model-wide ``normal_(0, std)`` re-init in the reference's module-traversal order."""
        with torch.no_grad():
            for ex in self.shared_experts:
                for p in (ex.gate_proj, ex.up_proj, ex.down_proj):
                    nn.init.normal_(p.weight, mean=0.0, std=std)
            self._init_routed_like_reference(construct=False, std=std)
            nn.init.normal_(self.router.weight, mean=0.0, std=std)

    # -- checkpoint format hooks --------------------------------------------------------------
    @staticmethod
    def _split_routed_state(module, state_dict, prefix, local_metadata):
        names = (("routed_gate_proj", "gate_proj"), ("routed_up_proj", "up_proj"),
                 ("routed_down_proj", "down_proj"))
        for stacked, short in names:
            t = state_dict.pop(prefix + stacked, None)
            if t is None:
                continue
            for i in range(t.shape[0]):
                e = module.expert_offset + i
                state_dict[f"{prefix}routed_experts.{e}.{short}.weight"] = t[i]

    @staticmethod
    def _stack_routed_state(module, state_dict, prefix, local_metadata, strict, missing_keys,
                            unexpected_keys, error_msgs):
        names = (("routed_gate_proj", "gate_proj"), ("routed_up_proj", "up_proj"),
                 ("routed_down_proj", "down_proj"))
        for stacked, short in names:
            if prefix + stacked in state_dict:
                continue
            rows = []
            for i in range(module.n_local_experts):
                key = f"{prefix}routed_experts.{module.expert_offset + i}.{short}.weight"
                if key not in state_dict:
                    rows = None
                    break
                rows.append(state_dict[key])
            if rows is not None:
                state_dict[prefix + stacked] = torch.stack(rows, 0)
            # drop per-expert keys of this module (including other ranks' experts)
            for key in [k for k in state_dict if k.startswith(f"{prefix}routed_experts.")
                        and k.endswith(f".{short}.weight")]:
                del state_dict[key]

    @property
    def routed_experts(self) -> _RoutedExpertList:
        return _RoutedExpertList(self)

    # -- forward --------------------------------------------------------------------------
    def _shared(self, xf: torch.Tensor) -> torch.Tensor:
        out = None
        for ex in self.shared_experts:
            y = ex(xf)
            out = y if out is None else out + y
        return out if out is not None else torch.zeros_like(xf)

    def _router_logits(self, xf: torch.Tensor) -> torch.Tensor:
        logits = _native_linear(xf, self.router.weight.to(xf.dtype)).float()
        if self.router_temperature != 1.0:
            logits = logits / self.router_temperature
        return logits

    def _replayed(self, name: str, value: torch.Tensor) -> torch.Tensor:
        """``value`` in normal operation; under activation checkpointing, the value stashed by
        the original forward (record mode stashes a copy, replay mode takes it back)."""
        mode = _routing_mode()
        if mode is None:
            return value
        stash = self.__dict__.setdefault("_replay_stash", collections.defaultdict(collections.deque))
        if mode == "record":
            stash[name].append(value.detach().clone())
            return value
        return stash[name].popleft()

    def _select(self, logits: torch.Tensor):
        if self.aux_loss_free and self.training:
            scores = logits + self._replayed("expert_bias", self.expert_bias).float()
        else:
            scores = logits
        return ops.router_topk(scores, self.top_k)

    def _routed(self, xf: torch.Tensor, idx: torch.Tensor, gates: torch.Tensor) -> torch.Tensor:
        if self.ep_engine is not None:
            return self.ep_engine.routed(self, xf, idx, gates)
        return ops.moe_routed(xf, idx, gates, self.routed_gate_proj, self.routed_up_proj,
                              self.routed_down_proj)

    def _after_routing(self, idx: torch.Tensor, n_tokens: int, aux: dict) -> None:
        if not self.training or _routing_mode() == "replay":
            return
        counts = ops.expert_histogram(idx, self.n_routed_experts)
        if self.ep_engine is not None:
            counts = self.ep_engine.global_counts(counts)
        if self.aux_loss_free:
            _update_expert_bias(counts, n_tokens * (self.ep_engine.dp_factor if self.ep_engine else 1),
                                self.n_routed_experts, self.top_k, self.bias_update_speed,
                                self.expert_bias, self.expert_load_ema)
            aux["expert_bias_mean"] = self.expert_bias.mean()
            aux["expert_bias_std"] = self.expert_bias.std()
        with torch.no_grad():
            self._total_tokens += n_tokens
            self._expert_counts += counts.to(self._expert_counts.dtype)

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, dict]:
        B, S, d = x.shape
        xf = x.reshape(-1, d)
        aux: dict = {}
        shared = self._shared(xf)
        gates, idx = self._select(self._router_logits(xf))
        routed = self._routed(xf, idx, gates)
        self._after_routing(idx, B * S, aux)
        aux["routed_expert_count"] = self.n_routed_experts
        aux["active_experts"] = self.top_k
        return (shared + routed.to(shared.dtype)).view(B, S, d), aux

    # -- statistics -----------------------------------------------------------------------
    def get_load_statistics(self) -> dict:
        if int(self._total_tokens.item()) == 0:
            return {"per_expert_load": None, "load_entropy": 0.0}
        counts = self._expert_counts.double()
        total = counts.sum()
        if total == 0:
            return {"per_expert_load": None, "load_entropy": 0.0}
        p = counts / total
        nz = p[p > 0]
        ent = float(-(nz * nz.log()).sum())
        max_ent = math.log(self.n_routed_experts)
        avg = 1.0 / self.n_routed_experts
        return {
            "per_expert_load": p.tolist(),
            "load_entropy": ent / max_ent if max_ent > 0 else 0.0,
            "max_load_ratio": float(p.max()) / avg,
            "bias_values": self.expert_bias.tolist() if self.aux_loss_free else None,
        }

    def reset_load_statistics(self) -> None:
        self._expert_counts.zero_()
        self._total_tokens.zero_()

    @property
    def total_expert_params(self) -> int:
        shared = sum(p.numel() for ex in self.shared_experts for p in ex.parameters())
        routed = self.n_routed_experts * 3 * self.d_model * self.routed_expert_dim
        return shared + routed + self.router.weight.numel()

    @property
    def active_params_per_token(self) -> int:
        shared = sum(p.numel() for ex in self.shared_experts for p in ex.parameters())
        return shared + self.top_k * 3 * self.d_model * self.routed_expert_dim + self.router.weight.numel()

    def extra_repr(self) -> str:
        return (f"d_model={self.d_model}, n_shared={self.n_shared_experts} (dim {self.shared_expert_dim}), "
                f"n_routed={self.n_routed_experts} (dim {self.routed_expert_dim}), top_k={self.top_k}, "
                f"load_balance={'aux-loss-free' if self.aux_loss_free else 'aux_loss'}")


def _update_expert_bias(counts: torch.Tensor, n_tokens: int, n_experts: int, top_k: int,
                        speed: float, expert_bias: torch.Tensor, load_ema: torch.Tensor) -> None:
    """bias -= speed * sign(load - 1/E), load EMA; one native kernel on CUDA (bitwise equal to
    the eager float32 ops below, which are the CPU path)."""
    if counts.is_cuda and expert_bias.dtype == torch.float32 and load_ema.dtype == torch.float32 \
            and expert_bias.is_contiguous() and load_ema.is_contiguous():
        from mamformer_b200.ops._ext import ext
        C = ext()
        if C is not None and not ops.force_reference():
            C.moe_bias_update(counts.long().contiguous(), float(n_tokens * top_k), n_experts, float(speed),
                              expert_bias, load_ema)
            return
    with torch.no_grad():
        load = counts.float() / (n_tokens * top_k + 1e-8)
        expert_bias -= speed * torch.sign(load - 1.0 / n_experts)
        load_ema.mul_(0.99).add_(0.01 * load)


def _moe_update_expert_bias(top_k_indices, total_tokens, n_routed_experts, top_k,
                            bias_update_speed, expert_bias, expert_load_ema) -> None:
    """Reference-signature helper (``moe.py:335-347``)."""
    counts = torch.bincount(top_k_indices.flatten().long(), minlength=n_routed_experts)
    _update_expert_bias(counts, total_tokens, n_routed_experts, top_k, bias_update_speed,
                        expert_bias, expert_load_ema)


class MoERouter(nn.Module):
    """Stand-alone top-k router returning (softmaxed top-k gates, indices)."""

    def __init__(self, d_model: int, n_experts: int, top_k: int = 8, temperature: float = 1.0):
        super().__init__()
        self.d_model = d_model
        self.n_experts = n_experts
        self.top_k = top_k
        self.temperature = temperature
        self.weight = nn.Parameter(torch.empty(n_experts, d_model))
        nn.init.normal_(self.weight, mean=0.0, std=0.02 / n_experts ** 0.5)

    def forward(self, x: torch.Tensor, expert_bias: Optional[torch.Tensor] = None):
        logits = _native_linear(x, self.weight.to(x.dtype)).float()
        if self.temperature != 1.0:
            logits = logits / self.temperature
        if expert_bias is not None:
            logits = logits + expert_bias
        return ops.router_topk(logits.reshape(-1, self.n_experts), self.top_k) if logits.dim() == 2 else \
            tuple(t.view(*logits.shape[:-1], self.top_k)
                  for t in ops.router_topk(logits.reshape(-1, self.n_experts), self.top_k))
