#!/usr/bin/env python
"""Per-op profile of a training step with ablations (KDA-Diff, interleave, Mamba).

Reference: ``scripts/profile_kda.py`` (49-345): torch.profiler top-20 CUDA ops, chrome trace,
ablations ``no_kda_diff`` / ``no_interleave`` / ``no_mamba``, peak memory.  Times come from the
profiler's device events (not wall clock); the chrome trace is written when ``--trace`` is given.
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402

ABLATIONS = ("full", "no_kda_diff", "no_interleave", "no_mamba")


def ablate(cfg, name):
    """Ablated copies of a config (reference ``scripts/profile_kda.py:49-78``):

    * ``no_kda_diff``: KDA-Diff off, the differential state attention (DSA) takes its place;
    * ``no_interleave``: interleaving off, every layer runs attention and SSM in fusion;
    * ``no_mamba``: every layer attention-only (``cross_layer`` with attention in every layer
      and no fusion layer, so no layer builds an SSM).  The reference's version of this
      ablation only switches interleaving off and so still runs the SSM everywhere."""
    if name == "no_kda_diff":
        cfg.kda_diff.enabled = False
        cfg.dsa.enabled = True
    elif name == "no_interleave":
        cfg.interleave.enabled = False
    elif name == "no_mamba":
        cfg.interleave.enabled = True
        cfg.interleave.pattern = "cross_layer"
        cfg.interleave.attn_every_k = 1
        cfg.interleave.first_layer_attn = True
        cfg.interleave.fusion_layers = []
        assert not any(t["has_ssm"] for t in cfg.layer_types()), "no_mamba ablation left an SSM layer"
    return cfg


def profile(cfg, seq_len, batch, steps, trace=None, top=20):
    import torch
    from torch.profiler import ProfilerActivity, profile as tprof
    from mamformer_b200 import MamformerForCausalLM
    from mamformer_b200.engine import TrainConfig, Trainer
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    torch.manual_seed(0)
    tr = Trainer(MamformerForCausalLM(cfg).to(dev),
                 TrainConfig(micro_batch=batch, compute_dtype=torch.bfloat16 if dev == "cuda" else torch.float32))
    ids = torch.randint(0, cfg.vocab_size, (batch, seq_len), device=dev)
    tr.train_step(ids)
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if dev == "cuda" else [])
    with tprof(activities=acts, acc_events=True) as prof:
        for _ in range(steps):
            tr.train_step(ids)
        if dev == "cuda":
            torch.cuda.synchronize()
    key = "self_cuda_time_total" if dev == "cuda" else "self_cpu_time_total"
    print(prof.key_averages().table(sort_by=key, row_limit=top))
    if trace:
        prof.export_chrome_trace(trace)
    if dev == "cuda":
        print(f"peak memory {torch.cuda.max_memory_allocated() / 2**30:.1f} GiB")


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", default="configs/_arch_verify.yaml")
    p.add_argument("--seq_len", type=int, default=2048)
    p.add_argument("--batch_size", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--ablation", default="full", choices=ABLATIONS + ("all",))
    p.add_argument("--trace", default=None, help="chrome trace output path")
    p.add_argument("--top", type=int, default=20)
    a = p.parse_args(argv)
    for name in (ABLATIONS if a.ablation == "all" else (a.ablation,)):
        print(f"==== {name}")
        profile(ablate(_common.load_config(a.config), name), a.seq_len, a.batch_size, a.steps, a.trace, a.top)


if __name__ == "__main__":
    main()
