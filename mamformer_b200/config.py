"""Model configuration: dataclasses, YAML I/O (nested and flat schema) and presets.

Parity with the reference configuration system (``mamformer/config.py``):

* the same dataclass names and field names (``MamformerConfig`` with the sub-configs
  ``mamba``, ``rope``, ``moe``, ``dsa``, ``mtp``, ``kda_diff``, ``st_moe``,
  ``communicative_moe``, ``interleave``, ``generation``), reference ``config.py:27-419``;
* the same two YAML layouts: nested under ``model:`` (``configs/ultra-7b.yaml``) and the flat
  ``<prefix>_<field>`` layout written by ``to_yaml`` (``configs/_arch_verify.yaml``), with the
  same flat key names (reference ``config.py:732-810``) so files round-trip between the two
  frameworks;
* the same layer-type resolution for the interleave patterns ``attn_every_k``, ``cross_layer``
  and ``custom`` (reference ``config.py:197-314``);
* the same presets (reference ``config.py:828-945``) and parameter-count formulas
  (reference ``config.py:451-534``).

Deliberate difference: every numeric field is coerced to its declared type on load.  PyYAML
reads ``1e-6`` (no dot) as the *string* ``'1e-6'``; the reference passes that string on to
``RMSNorm`` and fails on the first forward for ``ultra-7b.yaml``, ``7b.yaml``, ``pro-7b.yaml``
and ``ultra-7b-dense.yaml``.  Here those files load with ``rms_norm_eps == 1e-6``.
"""

from __future__ import annotations

import dataclasses
import math
import typing
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import yaml

__all__ = [
    "MambaConfig", "RopeConfig", "MoEConfig", "DSAConfig", "MTPConfig", "STMoEConfig",
    "KDADiffConfig", "CommunicativeMoEConfig", "InterleaveConfig", "GenerationConfig",
    "MamformerConfig", "PRESETS",
]


# ---------------------------------------------------------------------------------------------
# type coercion for values read from YAML / dicts
# ---------------------------------------------------------------------------------------------

def _coerce(value: Any, annotation: Any) -> Any:
    """Convert ``value`` to the type named by a dataclass annotation (string annotations)."""
    if value is None:
        return None
    ann = annotation if isinstance(annotation, str) else getattr(annotation, "__name__", str(annotation))
    ann = ann.replace(" ", "")
    if ann == "bool":
        if isinstance(value, str):
            low = value.strip().lower()
            if low in ("true", "yes", "on", "1"):
                return True
            if low in ("false", "no", "off", "0"):
                return False
            raise ValueError(f"cannot read {value!r} as a boolean")
        return bool(value)
    if ann == "int":
        if isinstance(value, bool):
            return int(value)
        if isinstance(value, str):
            return int(float(value))
        if isinstance(value, float) and value.is_integer():
            return int(value)
        return value
    if ann == "float":
        if isinstance(value, (str, int)) and not isinstance(value, bool):
            return float(value)
        return value
    if ann in ("str|int", "int|str"):
        if isinstance(value, str) and value.strip().lower() != "auto":
            try:
                return int(float(value))
            except ValueError:
                return value
        return value
    if ann.startswith("list[int]") or ann.startswith("List[int]"):
        return [int(v) for v in value]
    return value


def _field_types(cls) -> Dict[str, Any]:
    return {f.name: f.type for f in dataclasses.fields(cls)}


def _build(cls, values: Dict[str, Any]):
    """Instantiate dataclass ``cls`` from ``values`` (unknown keys ignored, types coerced)."""
    types = _field_types(cls)
    kwargs = {k: _coerce(v, types[k]) for k, v in values.items() if k in types}
    return cls(**kwargs)


# ---------------------------------------------------------------------------------------------
# sub-configs
# ---------------------------------------------------------------------------------------------

@dataclass
class MambaConfig:
    """Selective-SSM block settings.  ``dt_rank='auto'`` resolves to ceil(d_model/32).

    Note: the layer itself always uses ceil(d_model/32) (reference ``mamba2.py:191``); the
    resolved value here is informational, as in the reference."""
    expand: int = 1
    d_state: int = 128
    d_conv: int = 4
    dt_rank: str | int = "auto"


@dataclass
class RopeConfig:
    """Rotary embedding settings, with the reference's YaRN variant (``rope.py:123-162``)."""
    theta: float = 10000.0
    use_yarn: bool = False
    yarn_scale: float = 1.0
    yarn_original_max_seq_len: int = 8192
    yarn_beta_fast: int = 32
    yarn_beta_slow: int = 1


@dataclass
class MoEConfig:
    """DeepSeek-style MoE: shared experts + routed top-k experts, aux-loss-free bias."""
    enabled: bool = False
    n_shared_experts: int = 2
    shared_expert_intermediate_dim: int = 2304
    n_routed_experts: int = 64
    top_k: int = 8
    expert_intermediate_dim: int = 576
    routed_expert_intermediate_dim: int = 0
    router_temperature: float = 1.0
    aux_loss_free: bool = True
    bias_update_speed: float = 0.001
    target_expert_load: float = 1.0
    expert_dropout: float = 0.0

    def __post_init__(self):
        if not self.routed_expert_intermediate_dim:
            self.routed_expert_intermediate_dim = self.expert_intermediate_dim


@dataclass
class DSAConfig:
    """Legacy differential state-aware attention (superseded by KDA-Diff when both set)."""
    enabled: bool = False
    lambda_init: float = 0.8
    use_state_injection: bool = True
    state_injection_dim: int = 64
    num_attn_groups: int = 2


@dataclass
class MTPConfig:
    """Multi-token prediction heads (training-only auxiliary loss)."""
    enabled: bool = False
    depth: int = 2
    loss_weight: float = 0.3
    mtp_d_model: int = 0


@dataclass
class STMoEConfig:
    """Space-time MoE: temporal routing term lambda*W_h*h_t plus the balance lock."""
    enabled: bool = False
    lambda_init: float = 0.2
    lambda_max: float = 0.3
    learnable_lambda: bool = True
    use_balance_lock: bool = True
    balance_lock_threshold: int = 50


@dataclass
class KDADiffConfig:
    """Kernelised differential attention: linear (elu+1) and full (softmax) variants."""
    enabled: bool = False
    linear_ratio: int = 3
    kernel_dim: int = 128
    latent_dim: int = 512
    use_dynamic_ratio: bool = True


@dataclass
class CommunicativeMoEConfig:
    """Attention among the k selected expert outputs before the gate-weighted sum."""
    enabled: bool = False
    n_comm_heads: int = 4
    comm_depth: int = 1
    comm_dropout: float = 0.0


@dataclass
class InterleaveConfig:
    """Which layers run attention, SSM, or both (fusion).

    Patterns (reference ``config.py:159-314``):
      * ``attn_every_k``: attention every k layers (+ last ``last_layers_dense``); every
        attention layer is a fusion layer and every layer has an SSM.
      * ``cross_layer``: attention layers as above plus ``fusion_layers``; non-fusion attention
        layers are attention-only and take the SSM state of the preceding SSM-only layers.
      * ``custom``: explicit ``attention_layers`` (hybrid, like ``attn_every_k``).
    """
    enabled: bool = False
    pattern: str = "attn_every_k"
    attn_every_k: int = 4
    first_layer_attn: bool = True
    last_layers_dense: int = 2
    attention_layers: list[int] = field(default_factory=list)
    fusion_layers: list[int] = field(default_factory=list)

    def _periodic(self, n_layers: int) -> set:
        first = 0 if self.first_layer_attn else self.attn_every_k
        out = set(range(first, n_layers, max(1, self.attn_every_k)))
        if self.last_layers_dense > 0:
            out.update(range(max(0, n_layers - self.last_layers_dense), n_layers))
        return out

    def resolve_attention_layers(self, n_layers: int) -> list[int]:
        if self.pattern == "custom":
            chosen = {i for i in self.attention_layers if 0 <= i < n_layers}
            if not chosen:
                raise ValueError(
                    f"interleave pattern 'custom' needs attention_layers inside [0, {n_layers})")
            return sorted(chosen)
        chosen = self._periodic(n_layers)
        if self.pattern == "cross_layer":
            chosen.update(i for i in self.fusion_layers if 0 <= i < n_layers)
        return sorted(chosen)

    def resolve_fusion_layers(self, n_layers: int) -> set[int]:
        if self.pattern == "cross_layer":
            return {i for i in self.fusion_layers if 0 <= i < n_layers}
        return set(self.resolve_attention_layers(n_layers))

    def resolve_layer_types(self, n_layers: int) -> list[dict]:
        attn = set(self.resolve_attention_layers(n_layers))
        fusion = self.resolve_fusion_layers(n_layers)
        types = []
        for i in range(n_layers):
            has_attn = i in attn
            is_fusion = i in fusion
            has_ssm = ((not has_attn) or is_fusion) if self.pattern == "cross_layer" else True
            types.append({"has_attention": has_attn, "has_ssm": has_ssm, "is_fusion": is_fusion})
        return types

    def layout_string(self, n_layers: int) -> str:
        """Compact layer map: A = attention-only, S = SSM-only, F = fusion."""
        out = []
        for t in self.resolve_layer_types(n_layers):
            if t["has_attention"] and t["has_ssm"]:
                out.append("F")
            elif t["has_attention"]:
                out.append("A")
            else:
                out.append("S")
        return "".join(out)


@dataclass
class GenerationConfig:
    """Model-level generation limits and defaults (thinking-mode defaults included)."""
    max_context: int = 8192
    max_output_tokens: int = 4096
    default_temperature: float = 0.7
    default_top_k: int = 50
    default_top_p: float = 0.9
    repetition_penalty: float = 1.0
    thinking_enabled: bool = False
    thinking_mode: str = "NoThink"
    thinking_budget: int = 0
    thinking_num_paths: int = 0
    thinking_summary_budget: int = 0


# (attribute, flat-key prefix, sub-config class, {field: flat key}).  The flat key names are
# part of the on-disk format shared with the reference (reference ``config.py:732-810``); the
# mapping is the identity "<prefix>_<field>" except where listed explicitly.
_FLAT_EXCEPTIONS = {
    ("communicative_moe", "n_comm_heads"): "comm_moe_n_heads",
    ("communicative_moe", "comm_depth"): "comm_moe_depth",
    ("communicative_moe", "comm_dropout"): "comm_moe_dropout",
    ("mtp", "mtp_d_model"): "mtp_d_model",
}
_SUBCONFIGS = [
    ("mamba", "mamba", MambaConfig, ["expand", "d_state", "d_conv", "dt_rank"]),
    ("rope", "rope", RopeConfig, ["theta", "use_yarn", "yarn_scale", "yarn_original_max_seq_len",
                                  "yarn_beta_fast", "yarn_beta_slow"]),
    ("moe", "moe", MoEConfig, ["enabled", "n_shared_experts", "shared_expert_intermediate_dim",
                               "n_routed_experts", "top_k", "expert_intermediate_dim",
                               "router_temperature", "aux_loss_free", "bias_update_speed",
                               "expert_dropout", "target_expert_load"]),
    ("dsa", "dsa", DSAConfig, ["enabled", "lambda_init", "use_state_injection",
                               "state_injection_dim", "num_attn_groups"]),
    ("kda_diff", "kda_diff", KDADiffConfig, ["enabled", "linear_ratio", "kernel_dim",
                                             "latent_dim", "use_dynamic_ratio"]),
    ("mtp", "mtp", MTPConfig, ["enabled", "depth", "loss_weight", "mtp_d_model"]),
    ("st_moe", "st_moe", STMoEConfig, ["enabled", "lambda_init", "lambda_max",
                                       "learnable_lambda", "use_balance_lock",
                                       "balance_lock_threshold"]),
    ("communicative_moe", "comm_moe", CommunicativeMoEConfig,
     ["enabled", "n_comm_heads", "comm_depth", "comm_dropout"]),
    ("interleave", "interleave", InterleaveConfig,
     ["enabled", "pattern", "attn_every_k", "first_layer_attn", "last_layers_dense",
      "attention_layers", "fusion_layers"]),
    ("generation", "gen", GenerationConfig,
     ["max_context", "max_output_tokens", "default_temperature", "default_top_k",
      "default_top_p", "repetition_penalty", "thinking_enabled", "thinking_mode",
      "thinking_budget", "thinking_num_paths", "thinking_summary_budget"]),
]
_TOP_LEVEL = ["name", "model_type", "description", "d_model", "n_layers", "n_heads",
              "n_kv_heads", "head_dim", "d_ff", "vocab_size", "max_seq_len",
              "tie_word_embeddings", "use_sliding_window", "sliding_window", "dropout",
              "rms_norm_eps", "initializer_range"]


def _flat_key(attr: str, prefix: str, name: str) -> str:
    return _FLAT_EXCEPTIONS.get((attr, name), f"{prefix}_{name}")


@dataclass
class MamformerConfig:
    """Top-level model configuration (reference ``config.py:346-719``)."""

    d_model: int = 4096
    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    d_ff: int = 9216
    vocab_size: int = 128000
    max_seq_len: int = 8192
    tie_word_embeddings: bool = True
    use_sliding_window: bool = False
    sliding_window: int = 4096
    mamba: MambaConfig = field(default_factory=MambaConfig)
    rope: RopeConfig = field(default_factory=RopeConfig)
    moe: MoEConfig = field(default_factory=MoEConfig)
    dsa: DSAConfig = field(default_factory=DSAConfig)
    mtp: MTPConfig = field(default_factory=MTPConfig)
    kda_diff: KDADiffConfig = field(default_factory=KDADiffConfig)
    st_moe: STMoEConfig = field(default_factory=STMoEConfig)
    communicative_moe: CommunicativeMoEConfig = field(default_factory=CommunicativeMoEConfig)
    interleave: InterleaveConfig = field(default_factory=InterleaveConfig)
    generation: GenerationConfig = field(default_factory=GenerationConfig)
    dropout: float = 0.0
    rms_norm_eps: float = 1e-6
    initializer_range: float = 0.02
    name: str = "Mamformer"
    model_type: str = "Mamformer"
    description: str = ""

    def __post_init__(self):
        types = _field_types(MamformerConfig)
        for key in _TOP_LEVEL:
            setattr(self, key, _coerce(getattr(self, key), types[key]))
        if self.d_model % self.n_heads:
            raise ValueError(f"d_model ({self.d_model}) must be divisible by n_heads ({self.n_heads})")
        if self.n_heads % self.n_kv_heads:
            raise ValueError(f"n_heads ({self.n_heads}) must be divisible by n_kv_heads ({self.n_kv_heads})")
        if self.head_dim != self.d_model // self.n_heads:
            raise ValueError(f"head_dim ({self.head_dim}) must equal d_model//n_heads "
                             f"({self.d_model // self.n_heads})")
        if self.d_ff <= 0:
            raise ValueError(f"d_ff ({self.d_ff}) must be positive")
        if self.mamba.dt_rank == "auto":
            self.mamba.dt_rank = math.ceil(self.d_model / 32)
        if self.generation.max_context == 8192 and self.max_seq_len != 8192:
            self.generation.max_context = self.max_seq_len
        if self.communicative_moe.enabled and not (self.moe.enabled or self.st_moe.enabled):
            raise ValueError("communicative_moe needs moe.enabled or st_moe.enabled")

    # -- derived -------------------------------------------------------------------------
    @property
    def n_head_groups(self) -> int:
        return self.n_heads // self.n_kv_heads

    @property
    def d_inner(self) -> int:
        return self.d_model * self.mamba.expand

    @property
    def total_context_length(self) -> int:
        if self.rope.use_yarn:
            return int(self.rope.yarn_original_max_seq_len * self.rope.yarn_scale)
        return self.max_seq_len

    @property
    def max_output_tokens(self) -> int:
        return self.generation.max_output_tokens

    def layer_types(self) -> list[dict]:
        """Per-layer {has_attention, has_ssm, is_fusion} (all fusion when interleave is off)."""
        if self.interleave.enabled:
            return self.interleave.resolve_layer_types(self.n_layers)
        return [{"has_attention": True, "has_ssm": True, "is_fusion": True}
                for _ in range(self.n_layers)]

    def layout_string(self) -> str:
        return "".join("F" if t["has_attention"] and t["has_ssm"] else
                       ("A" if t["has_attention"] else "S") for t in self.layer_types())

    # -- analytic parameter counts (same formulas as reference config.py:451-534) ---------
    def _attn_params(self) -> int:
        d, h, kv, hd = self.d_model, self.n_heads, self.n_kv_heads, self.head_dim
        if self.dsa.enabled:
            p = 2 * d * h * hd + 2 * d * kv * hd + d * h * hd
            if self.dsa.use_state_injection:
                s = self.dsa.state_injection_dim
                p += 2 * d * s + 2 * s * kv * hd
            return p
        return d * h * hd + 2 * d * kv * hd + d * h * hd

    def _ssm_params(self) -> int:
        d, di, n = self.d_model, self.d_inner, self.mamba.d_state
        return 4 * d * di + di * d + di * self.mamba.d_conv + d * n + 2 * d * n + n + di

    def _ffn_params(self, active: bool) -> int:
        d = self.d_model
        if self.moe.enabled or (active and self.st_moe.enabled):
            m = self.moe
            n_routed = m.top_k if active else m.n_routed_experts
            return (m.n_shared_experts * 3 * d * m.shared_expert_intermediate_dim
                    + n_routed * 3 * d * m.routed_expert_intermediate_dim
                    + d * m.n_routed_experts + m.n_routed_experts)
        return 3 * d * self.d_ff

    def _ffn_total_params(self) -> int:
        return self._ffn_params(active=False)

    def _ffn_active_params(self) -> int:
        return self._ffn_params(active=True)

    def _mtp_params(self) -> int:
        if not self.mtp.enabled:
            return 0
        md = self.mtp.mtp_d_model or self.d_model
        per_depth = (md + self._attn_params() + self._ssm_params() + 3 * md * (self.d_ff // 8)
                     + self.d_model * md + self.d_model)
        return self.mtp.depth * per_depth

    def _per_layer(self, active: bool) -> int:
        return (self._attn_params() + self._ssm_params() + self._ffn_params(active)
                + self.d_model + 4 * self.d_model)

    @property
    def num_parameters(self) -> int:
        total = self.n_layers * self._per_layer(False) + self.vocab_size * self.d_model + self.d_model
        if not self.tie_word_embeddings:
            total += self.vocab_size * self.d_model
        return total + self._mtp_params()

    @property
    def num_active_parameters(self) -> int:
        return self.n_layers * self._per_layer(True) + self.vocab_size * self.d_model + self.d_model

    @property
    def num_parameters_billions(self) -> float:
        return self.num_parameters / 1e9

    @property
    def num_active_parameters_billions(self) -> float:
        return self.num_active_parameters / 1e9

    # -- serialisation --------------------------------------------------------------------
    def to_dict(self) -> dict:
        """Flat dict with the shared ``<prefix>_<field>`` key names."""
        out = {k: getattr(self, k) for k in ["name", "model_type", "description"]}
        out.update({k: getattr(self, k) for k in _TOP_LEVEL if k not in out})
        for attr, prefix, _cls, names in _SUBCONFIGS:
            sub = getattr(self, attr)
            for n in names:
                value = getattr(sub, n)
                out[_flat_key(attr, prefix, n)] = list(value) if isinstance(value, list) else value
        return out

    def to_nested_dict(self) -> dict:
        """Nested layout (``model:`` block with sub-config sections)."""
        out = {k: getattr(self, k) for k in _TOP_LEVEL}
        for attr, _prefix, _cls, names in _SUBCONFIGS:
            sub = getattr(self, attr)
            out[attr] = {n: getattr(sub, n) for n in names}
        return {"model": out}

    def to_yaml(self, path: str, nested: bool = False) -> None:
        data = self.to_nested_dict() if nested else self.to_dict()
        with open(path, "w") as fh:
            yaml.safe_dump(data, fh, default_flow_style=False, sort_keys=False)

    @classmethod
    def from_dict(cls, d: dict) -> "MamformerConfig":
        """Build from a flat dict, a nested dict, or a mixture (nested sections win)."""
        d = dict(d.get("model", d)) if isinstance(d.get("model"), dict) else dict(d)
        subs = {}
        for attr, prefix, sub_cls, names in _SUBCONFIGS:
            values = {}
            for n in names:
                key = _flat_key(attr, prefix, n)
                if key in d:
                    values[n] = d[key]
            nested = d.get(attr)
            if isinstance(nested, dict):
                values.update({k: v for k, v in nested.items() if k in names or
                               k in _field_types(sub_cls)})
            subs[attr] = _build(sub_cls, values)
        types = _field_types(cls)
        top = {k: _coerce(d[k], types[k]) for k in _TOP_LEVEL if k in d}
        return cls(**top, **subs)

    @classmethod
    def from_yaml(cls, path: str) -> "MamformerConfig":
        with open(path) as fh:
            raw = yaml.safe_load(fh) or {}
        return cls.from_dict(raw)

    @classmethod
    def from_preset(cls, name: str = "7b") -> "MamformerConfig":
        if name not in PRESETS:
            raise ValueError(f"Unknown preset '{name}'. Available: {', '.join(PRESETS)}")
        return PRESETS[name]()

    @classmethod
    def load(cls, spec: str) -> "MamformerConfig":
        """A YAML path or a preset name (the ``--config`` argument of the training scripts)."""
        if spec in PRESETS:
            return cls.from_preset(spec)
        return cls.from_yaml(spec)

    def replace(self, **changes) -> "MamformerConfig":
        """Copy with top-level fields changed (sub-configs are deep-copied)."""
        d = self.to_dict()
        new = MamformerConfig.from_dict(d)
        for k, v in changes.items():
            setattr(new, k, v)
        return new

    def summary(self) -> str:
        bar = "=" * 60
        title = f"  {self.name} - {self.description}" if self.description else f"  {self.name}"
        rows = [bar, title, bar,
                f"  d_model:         {self.d_model}",
                f"  n_layers:        {self.n_layers}",
                f"  n_heads:         {self.n_heads} (GQA, kv={self.n_kv_heads})",
                f"  head_dim:        {self.head_dim}",
                f"  d_ff (base):     {self.d_ff}",
                f"  vocab_size:      {self.vocab_size}",
                bar,
                f"  Context:         {self.total_context_length:,} tokens",
                f"  Max Output:      {self.max_output_tokens:,} tokens",
                bar]
        if self.moe.enabled:
            m = self.moe
            rows += ["  MoE:             ENABLED",
                     f"    Shared:        {m.n_shared_experts} x dim {m.shared_expert_intermediate_dim}",
                     f"    Routed:        {m.n_routed_experts} experts x dim {m.routed_expert_intermediate_dim}",
                     f"    Active:        top-{m.top_k}",
                     f"    Load balance:  {'aux-loss-free' if m.aux_loss_free else 'auxiliary loss'}"]
        if self.dsa.enabled:
            rows.append(f"  DSA:             ENABLED (lambda={self.dsa.lambda_init})")
        if self.kda_diff.enabled:
            k = self.kda_diff
            rows.append(f"  KDA-Diff:        ENABLED ({k.linear_ratio}:1 linear:full, kernel={k.kernel_dim}, "
                        f"latent={k.latent_dim}, dynamic={'on' if k.use_dynamic_ratio else 'off'})")
        if self.mtp.enabled:
            rows.append(f"  MTP:             ENABLED (depth={self.mtp.depth})")
        if self.st_moe.enabled:
            rows.append(f"  ST-MoE:          ENABLED (lambda={self.st_moe.lambda_init}, max={self.st_moe.lambda_max})")
        if self.communicative_moe.enabled:
            c = self.communicative_moe
            rows.append(f"  CommunicativeMoE:ENABLED ({c.n_comm_heads} heads, depth={c.comm_depth})")
        if self.interleave.enabled:
            rows.append(f"  Interleave:      ENABLED pattern={self.interleave.pattern} "
                        f"layout={self.layout_string()}")
        if self.rope.use_yarn:
            rows.append(f"  YaRN:            scale={self.rope.yarn_scale}x, theta={self.rope.theta}")
        rows += [bar,
                 f"  Total params:    {self.num_parameters_billions:.1f}B",
                 f"  Active params:   {self.num_active_parameters_billions:.1f}B",
                 f"  Expansion ratio: {self.num_parameters / max(1, self.num_active_parameters):.1f}x",
                 bar]
        return "\n".join(rows)


# ---------------------------------------------------------------------------------------------
# presets (values match reference config.py:828-945)
# ---------------------------------------------------------------------------------------------

def _dense(name: str, **dims) -> MamformerConfig:
    return MamformerConfig(
        name=f"Mamformer-{name}",
        mamba=MambaConfig(expand=1, d_state=32 if name == "debug" else 128, d_conv=4),
        generation=GenerationConfig(max_context=dims["max_seq_len"],
                                    max_output_tokens=dims["max_seq_len"] // 2),
        **dims)


def _ultra(name, desc, d_model, n_layers, n_heads, d_ff, max_seq_len, window, theta,
           yarn_scale, n_routed, shared_dim, routed_dim, fusion, max_out, beta=False):
    rope = RopeConfig(theta=theta, use_yarn=True, yarn_scale=yarn_scale)
    if yarn_scale > 1.0:
        rope.yarn_original_max_seq_len = 8192
    return MamformerConfig(
        name=name, description=desc, d_model=d_model, n_layers=n_layers, n_heads=n_heads,
        n_kv_heads=8, head_dim=128, d_ff=d_ff, vocab_size=128000, max_seq_len=max_seq_len,
        use_sliding_window=True, sliding_window=window,
        mamba=MambaConfig(expand=1, d_state=128, d_conv=4), rope=rope,
        moe=MoEConfig(enabled=True, n_shared_experts=2, shared_expert_intermediate_dim=shared_dim,
                      n_routed_experts=n_routed, top_k=8, expert_intermediate_dim=routed_dim,
                      aux_loss_free=True, bias_update_speed=0.001),
        dsa=DSAConfig(enabled=False, lambda_init=0.8, use_state_injection=True, state_injection_dim=64),
        kda_diff=KDADiffConfig(enabled=True, linear_ratio=3, kernel_dim=128, latent_dim=512,
                               use_dynamic_ratio=True),
        mtp=MTPConfig(enabled=True, depth=2, loss_weight=0.3),
        interleave=InterleaveConfig(enabled=True, pattern="cross_layer", attn_every_k=4,
                                    first_layer_attn=True, last_layers_dense=2, fusion_layers=fusion),
        generation=GenerationConfig(max_context=max_seq_len, max_output_tokens=max_out,
                                    default_temperature=0.7, default_top_k=50, default_top_p=0.9))


PRESETS = {
    "7b": lambda: _dense("7b", d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128,
                         d_ff=9216, vocab_size=128000, max_seq_len=8192),
    "1b": lambda: _dense("1b", d_model=2048, n_layers=24, n_heads=16, n_kv_heads=4, head_dim=128,
                         d_ff=5632, vocab_size=64000, max_seq_len=4096),
    "300m": lambda: _dense("300m", d_model=1024, n_layers=24, n_heads=16, n_kv_heads=4, head_dim=64,
                           d_ff=2816, vocab_size=32000, max_seq_len=2048),
    "debug": lambda: _dense("debug", d_model=256, n_layers=4, n_heads=4, n_kv_heads=2, head_dim=64,
                            d_ff=512, vocab_size=1000, max_seq_len=128),
    "ultra-7b": lambda: _ultra("Mamformer-Ultra-7B", "~39B total / ~7.5B active | 8K context | 4K output",
                               4096, 32, 32, 9216, 8192, 4096, 1.0e6, 1.0, 128, 2304, 576, [30, 31], 4096),
    "ultra-37b": lambda: _ultra("Mamformer-Ultra-37B", "~200B total / ~37B active | 128K context | 32K output",
                                6144, 40, 48, 12288, 131072, 16384, 1.0e7, 16.0, 256, 3072, 768, [38, 39], 32768),
    "ultra-371b": lambda: _ultra("Mamformer-Ultra-371B", "371B total / 28B active | 256K context | 65K output",
                                 7168, 46, 56, 14336, 262144, 16384, 2.0e7, 32.0, 384, 3584, 896, [44, 45], 65536),
    "ultra-671b": lambda: _ultra("Mamformer-Ultra-671B", "671B total / 37B active | 1M context | 163K output [MAX]",
                                 7168, 52, 56, 14336, 1048576, 32768, 5.0e7, 128.0, 640, 3584, 896,
                                 [48, 49, 50, 51], 163800),
}
