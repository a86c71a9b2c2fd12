"""Training metrics: the reference's log line plus device-timed throughput, MFU and JSONL.

Reference fields (``scripts/train.py:466-516``): step, loss (average over the log window), main
and MTP loss, learning rate, tokens/s; log format ``%(asctime)s | %(levelname)s | %(message)s``.
Added: the step time measured with CUDA events on the training stream, tokens/s per rank and
for the job, model FLOPs utilisation against a peak (``MAMF_PEAK_TFLOPS``, default the dense
bf16 figure of one B200) and one JSON object per logged step in ``metrics.jsonl``.
"""

from __future__ import annotations

import json
import logging
import os
import time
from typing import Optional

import torch

LOG_FORMAT = "%(asctime)s | %(levelname)s | %(message)s"


def setup_logging(rank: int = 0, level=logging.INFO) -> logging.Logger:
    logging.basicConfig(level=level if rank == 0 else logging.WARNING, format=LOG_FORMAT)
    return logging.getLogger("mamformer_b200")


def train_flops_per_token(config, seq_len: int) -> float:
    """6 x active parameters + the quadratic attention term of the softmax-attention layers."""
    n_active = config.num_active_parameters
    attn_layers = sum(1 for lt in config.layer_types() if lt["has_attention"])
    quad = 12 * attn_layers * seq_len * config.n_heads * config.head_dim / 2   # causal half
    return 6.0 * n_active + quad


def matmul_params_per_token(model) -> int:
    """Weights that take part in a matmul for one token of a training forward.

    Counts every 2-D projection weight once, the routed experts at top-k of their number (the
    stacked (E, out, in) tensors, local slice included under expert parallelism), the attention
    module each KDA-Diff layer actually ran last (``last_choice``; linear when none has run yet)
    and the tied vocabulary head once per loss head (main + every MTP depth).  Token embedding
    lookups, depthwise convolutions, norms and the scan are not matmuls and are left out."""
    from mamformer_b200.models.kda_diff import KDADiffAttention
    from mamformer_b200.models.moe import DeepSeekMoE
    skip_ids = set()
    total = 0
    for mod in model.modules():
        if isinstance(mod, KDADiffAttention):
            unused = mod.full_attn if (mod.last_choice or "linear") == "linear" else mod.linear_attn
            skip_ids.update(id(p) for p in unused.parameters())
        elif isinstance(mod, DeepSeekMoE):
            for name in ("routed_gate_proj", "routed_up_proj", "routed_down_proj"):
                w = getattr(mod, name)
                skip_ids.add(id(w))
                total += w.numel() // max(1, w.shape[0]) * mod.top_k
    vocab_heads = 1
    for name, p in model.named_parameters():
        if id(p) in skip_ids or p.dim() != 2:
            continue
        if "embed" in name:
            continue
        total += p.numel()
    mtp = getattr(model, "mtp", None)
    if mtp is not None and getattr(mtp, "output_heads", None) is None:
        vocab_heads += int(getattr(mtp, "depth", 0))      # MTP depths reuse the tied embedding
    emb = getattr(getattr(model, "model", None), "embed_tokens", None)
    if emb is not None:
        total += vocab_heads * emb.weight.numel()
    return total


class MetricsLogger:
    def __init__(self, out_dir: Optional[str], rank: int = 0, world: int = 1, flops_per_token: float = 0.0,
                 peak_tflops: Optional[float] = None):
        self.rank, self.world = rank, world
        self.flops_per_token = flops_per_token
        self.peak = float(peak_tflops or os.environ.get("MAMF_PEAK_TFLOPS", 2250.0)) * 1e12
        self.path = os.path.join(out_dir, "metrics.jsonl") if (out_dir and rank == 0) else None
        if self.path:
            os.makedirs(out_dir, exist_ok=True)
        self.log = logging.getLogger("mamformer_b200")
        self._t0 = None
        self._ev = None
        self._window = []

    def step_start(self) -> None:
        self._t0 = time.perf_counter()
        if torch.cuda.is_available():
            self._ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self._ev[0].record()

    def step_end(self, step: int, loss: float, tokens_per_rank: int, lr: float, extra: Optional[dict] = None,
                 emit: bool = True) -> dict:
        dev_ms = None
        if self._ev is not None:
            self._ev[1].record()
            self._ev[1].synchronize()
            dev_ms = self._ev[0].elapsed_time(self._ev[1])
        wall = time.perf_counter() - (self._t0 or time.perf_counter())
        t = (dev_ms / 1000.0) if dev_ms else wall
        tps = tokens_per_rank / t if t > 0 else 0.0
        rec = {"step": step, "loss": loss, "lr": lr, "step_ms": t * 1000.0, "wall_ms": wall * 1000.0,
               "tokens_per_s_rank": tps, "tokens_per_s_job": tps * self.world,
               "mfu": (tps * self.flops_per_token / self.peak) if self.flops_per_token else None}
        if extra:
            rec.update({k: (float(v) if torch.is_tensor(v) else v) for k, v in extra.items()})
        if emit and self.rank == 0:
            msg = f"step {step} | loss {loss:.4f} | lr {lr:.2e} | {rec['step_ms']:.0f} ms | {rec['tokens_per_s_job']:.0f} tok/s"
            if rec["mfu"] is not None:
                msg += f" | MFU {100 * rec['mfu']:.1f}%"
            for k in ("main_loss", "mtp_loss", "grad_norm"):
                if k in rec and rec[k] is not None:
                    msg += f" | {k} {rec[k]:.4f}"
            self.log.info(msg)
            if self.path:
                with open(self.path, "a") as f:
                    f.write(json.dumps(rec) + "\n")
        return rec
