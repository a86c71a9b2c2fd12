#!/usr/bin/env python
"""Analytic memory / compute budget of a config under a 4-D layout on B200s.

Reference: ``scripts/profile_model.py`` (34-136: estimates for an 8 x A100 FSDP split).  Here the
budget follows this framework's storage: bf16 weights plus fp32 master, gradient and two Adam
moments (18 bytes per parameter held), routed experts divided by EP, dense weights by TP and PP,
activations per micro-batch estimated per layer type, against 180 GB per GPU.
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402

GB = 1e9


def budget(cfg, seq_len, batch, dp=1, tp=1, pp=1, ep=1, checkpointing=False):
    total = cfg.num_parameters
    active = cfg.num_active_parameters
    routed = 0
    if cfg.moe.enabled:
        moe_layers = sum(1 for i in range(cfg.n_layers))
        routed = moe_layers * cfg.moe.n_routed_experts * 3 * cfg.d_model * cfg.moe.expert_intermediate_dim
    dense = total - routed
    per_gpu_params = dense / (tp * pp) + routed / (ep * pp)
    weights = per_gpu_params * 18
    d, S, L = cfg.d_model, seq_len, cfg.n_layers / pp
    per_layer_act = batch * S * d * 2 * (34 if not checkpointing else 4)       # bf16 activations kept
    per_layer_act += batch * S * cfg.d_model * cfg.mamba.expand * 2 * 6         # SSM branch
    if cfg.moe.enabled:
        per_layer_act += batch * S * cfg.moe.top_k * (d + 3 * cfg.moe.expert_intermediate_dim) * 2
    acts = per_layer_act * L / tp
    logits = batch * min(S, 8192) * 2 * 2 * (1 << 30) / (1 << 30) * 0 + (1 << 30) * 1.5   # fused CE chunk
    flops_per_token = 6 * active
    return {"params_b": total / 1e9, "active_b": active / 1e9, "params_per_gpu_b": per_gpu_params / 1e9,
            "weights_optimizer_gb": weights / GB, "activations_gb": acts / GB, "ce_chunk_gb": logits / GB,
            "total_gb": (weights + acts + logits) / GB, "fits_180gb": (weights + acts + logits) / GB < 170,
            "train_gflops_per_token": flops_per_token / 1e9}


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", required=True)
    p.add_argument("--seq_len", type=int, default=8192)
    p.add_argument("--batch_size", type=int, default=1)
    for k in ("dp", "tp", "pp", "ep"):
        p.add_argument(f"--{k}", type=int, default=1)
    p.add_argument("--gradient_checkpointing", action="store_true")
    a = p.parse_args(argv)
    cfg = _common.load_config(a.config)
    print(cfg.summary() if hasattr(cfg, "summary") else cfg)
    for k, v in budget(cfg, a.seq_len, a.batch_size, a.dp, a.tp, a.pp, a.ep, a.gradient_checkpointing).items():
        print(f"{k:26s} {v:.3f}" if isinstance(v, float) else f"{k:26s} {v}")


if __name__ == "__main__":
    main()
