#!/usr/bin/env python
"""Headline benchmark: training tokens/s for the ultra-7b MoE architecture on N B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mamformer_b200|reference]

For N > 1 launch with torchrun (one process per GPU, NCCL over NVLink); every rank runs the
same steps and rank 0 prints one JSON line.

Workload: ``configs/ultra-7b.yaml`` (d_model 4096, 32 heads / 8 KV heads, Mamba expand 2 with
d_state 128, KDA-Diff, 2 shared + 128 routed experts top-8, MTP depth 2, vocab 128000) with
the depth truncated to ``--layers`` (default 4: layout A S S F - attention-only, two SSM-only,
one fusion layer, the same per-layer shapes as the full model); sequence length 4096;
uniform-random token ids; random-init weights; bf16 compute with fp32 master weights and
AdamW; per-GPU batch = micro_batch x grad_accum sequences (weak scaling).  A step is one full
optimizer step (forward, backward, gradient reduction, clipping, AdamW).

Timing: W untimed warm-up steps, then K steps between a barrier + device synchronisation,
measured with CUDA events on the launching stream; the time is the max over ranks.  The
working set (11+ GB of bf16 weights, GBs of activations) is far larger than the 126 MB L2.
SM clocks and throttle reasons are sampled with nvidia-smi during the timed region.

End-to-end number (``e2e``): the same metric through the public ``Trainer.train_step`` API
with each step's token ids copied from pinned host memory and the loss read back to the host
every step, timed on the host (max over ranks).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "train tokens/s per box, ultra-7b MoE bf16 @1/2/4/8 B200, max over ranks"
# The reference publishes no throughput for this model or hardware, so vs_baseline stays null.
BASELINE_TOKS = None


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mamformer_b200", choices=["mamformer_b200", "reference"])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--micro-batch", type=int, default=4)
    ap.add_argument("--grad-accum", type=int, default=4)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile-launches", type=int, default=1)
    ap.add_argument("--dp-transport", default="p2p", choices=["p2p", "nccl"],
                    help="N > 1: dense-gradient all-reduce by this repository's peer-memory path (default: "
                         "copy-engine pulls of symmetric-memory gradient buckets, overlapped with the last "
                         "backward; run at 2 and 8 GPUs) or by NCCL")
    ap.add_argument("--profile-table", type=int, default=0,
                    help="print the top-N kernels of one extra step by device time (torch profiler, for "
                         "ranking only; never a timed number) to stderr")
    ap.add_argument("--breakdown", type=int, default=1,
                    help="after the timed steps, one extra step with CUDA-event marks: forward, backward, "
                         "exposed gradient reduction, optimizer and the expert-parallel phases (max over ranks)")
    ap.add_argument("--workload", default="ultra7b", choices=["ultra7b", "7b-tp"],
                    help="ultra7b: the headline MoE benchmark; 7b-tp: configs/7b.yaml (dense hybrid, all "
                         "layers) tensor-parallel over the N GPUs at seq 8192, global batch 64 sequences "
                         "(tokens/s of the job; strong scaling)")
    ap.add_argument("--window-mode", default="reference", choices=["reference", "causal"],
                    help="sliding-window masks: the reference's (0 <= key - query < W, which with the causal "
                         "mask leaves only the diagonal in full differential attention and looks ahead in "
                         "GQA) or the causal window (0 <= query - key < W)")
    ap.add_argument("--checkpoint", default="none", choices=["none", "attention", "all"],
                    help="activation recomputation: none, the reference's selective form (full-attention "
                         "layers), or every layer (needed by the full 32-layer model)")
    ap.add_argument("--zero", type=int, default=0, choices=[0, 1],
                    help="1: shard the dense weights' fp32 masters and Adam moments over the data-parallel group")
    ap.add_argument("--build", default="auto", choices=["auto", "host", "device"],
                    help="device: construct on the GPU, each rank allocating only its routed-expert slice "
                         "(auto: device when the model has more than 8 layers)")
    ap.add_argument("--parallel", default="ep", choices=["ep", "dp"],
                    help="N > 1: ep = routed experts sharded over all N GPUs (EP=N x dense DP=N, the "
                         "ultra-7b benchmark layout, EP=8 x DP on 8 GPUs); dp = every GPU holds every expert")
    return ap.parse_args()


def bench_config(layers: int, root: str = ROOT) -> dict:
    sys.path.insert(0, root)
    from mamformer_b200.config import MamformerConfig
    d = MamformerConfig.from_yaml(os.path.join(root, "configs", "ultra-7b.yaml")).to_dict()
    d.update(n_layers=layers, interleave_fusion_layers=[layers - 1], interleave_last_layers_dense=1)
    return d


def _dist_init():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def _max_over_ranks(x: float, world: int) -> float:
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _peak_tflops():
    """bf16 peak used for MFU: the measured sustained cuBLAS figure of this pool when the
    measurement file is present, else the same figure recorded earlier."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured sustained cuBLAS bf16"
    except (OSError, KeyError, ValueError):
        return 1390.2, "sustained cuBLAS bf16 measured on this pool (file absent)"


def _breakdown(trainer, model, batch, world):
    """One extra (untimed) step with CUDA-event marks; milliseconds per phase, max over ranks.
    The expert-parallel phases are also contained in forward / backward."""
    import torch
    eng = getattr(model, "_mamf_ep_engine", None)
    trainer.timer.enabled = True
    trainer.timer.reset()
    if eng is not None:
        eng.timer.enabled = True
        eng.timer.reset()
    _barrier(world)
    trainer.train_step(batch)
    torch.cuda.synchronize()
    out = trainer.timer.summary()
    if eng is not None:
        out.update({"ep." + k: v for k, v in eng.timer.summary().items()})
        eng.timer.enabled = False
    trainer.timer.enabled = False
    keys = sorted(out)
    vals = [_max_over_ranks(out[k], world) for k in keys]
    return {k: round(v, 2) for k, v in zip(keys, vals)}


def _kernel_table(step_fn, top):
    """Device time per kernel name over one step (torch profiler; ranking only)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    agg = {}
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            a = agg.setdefault(ev.name, [0.0, 0])
            a[0] += ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
            a[1] += 1
    total = sum(v[0] for v in agg.values()) or 1.0
    rows = sorted(agg.items(), key=lambda kv: -kv[1][0])[:top]
    print(f"# kernel device time over one step (total {total / 1e3:.1f} ms, profiler)", file=sys.stderr)
    for name, (us, n) in rows:
        print(f"{us / 1e3:9.2f} ms {100 * us / total:5.1f}% {n:6d}x  {name[:140]}", file=sys.stderr)


def _emit(obj, rank):
    if rank == 0:
        print(json.dumps(obj), flush=True)


def _count_launches(step_fn, prefix=("mamf::",)):
    """Run one step under the profiler; return (our kernel launches, all kernel launches)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA], acc_events=True) as prof:
        step_fn()
        torch.cuda.synchronize()
    ours = total = 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA and not ev.name.startswith("Memcpy") \
                and not ev.name.startswith("Memset"):
            total += 1
            if any(p in ev.name for p in prefix):
                ours += 1
    return ours, total


def run_ours(args, rank, world):
    import torch
    import torch.distributed as dist
    from mamformer_b200 import ops
    from mamformer_b200.config import MamformerConfig
    from mamformer_b200.engine import TrainConfig, Trainer
    from mamformer_b200.models.model import MamformerForCausalLM
    from mamformer_b200.utils.clocks import ClockSampler

    if not ops.has_native():
        raise RuntimeError("native extension missing: run python setup.py build_ext --inplace")
    if ops.force_reference():
        raise RuntimeError("MAMF_FORCE_REFERENCE=1 routes every op to eager PyTorch; bench.py refuses to "
                           "time that path (unset it)")
    cfg = MamformerConfig.from_dict(bench_config(args.layers))
    per_gpu = args.micro_batch * args.grad_accum
    tcfg = TrainConfig(learning_rate=2e-4, warmup_steps=10, max_steps=1000, micro_batch=args.micro_batch,
                       grad_accum=args.grad_accum)
    torch.manual_seed(0)
    on_device = args.build == "device" or (args.build == "auto" and args.layers > 8)
    if on_device:
        import contextlib
        from mamformer_b200.models.moe import build_expert_slice
        sl = build_expert_slice(rank, world) if (world > 1 and args.parallel == "ep") else contextlib.nullcontext()
        with torch.device("cuda"), sl:
            model = MamformerForCausalLM(cfg)
    else:
        model = MamformerForCausalLM(cfg).cuda()
    if args.checkpoint != "none":
        model.model.enable_gradient_checkpointing(all_layers=args.checkpoint == "all")
    if args.window_mode != "reference":
        for m in model.modules():
            if hasattr(m, "window_mode"):
                m.window_mode = args.window_mode
    if world > 1 and args.parallel == "ep":
        from mamformer_b200.parallel import DistributedCoordinator, ParallelConfig
        coord = DistributedCoordinator(ParallelConfig(ep_size=world)).initialize()
        model = coord.shard_model(model)
        torch.cuda.empty_cache()
        trainer = Trainer(model, tcfg, dp_group=coord.get_group("dense_dp"),
                          expert_dp_group=coord.get_group("expert_dp"), ep_group=coord.get_group("ep"),
                          dp_transport=args.dp_transport, zero_stage=args.zero)
        parallelism = f"ep{world} (routed experts sharded over {world} GPUs; dense weights data-parallel)"
    else:
        trainer = Trainer(model, tcfg, dp_group=dist.group.WORLD if world > 1 else None,
                          dp_transport=args.dp_transport, zero_stage=args.zero)
        parallelism = f"dp{world}"
    n_batches = 2
    g = torch.Generator().manual_seed(1234 + rank)
    host = [torch.randint(0, cfg.vocab_size, (per_gpu, args.seq), generator=g).pin_memory()
            for _ in range(n_batches)]
    dev = [h.cuda() for h in host]

    for i in range(args.warmup):
        trainer.train_step(dev[i % n_batches])
    _barrier(world)
    clocks = ClockSampler(gpu_index=torch.cuda.current_device()).start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        trainer.train_step(dev[i % n_batches])
    end.record()
    torch.cuda.synchronize()
    _barrier(world)
    clk = clocks.stop()
    ms = _max_over_ranks(start.elapsed_time(end), world) / args.steps
    tokens_per_step = world * per_gpu * args.seq
    value = tokens_per_step / (ms / 1000.0)

    e2e = None
    if not args.no_e2e and args.e2e_steps > 0:
        _barrier(world)
        t0 = time.perf_counter()
        loss = None
        for i in range(args.e2e_steps):
            loss = trainer.train_step(host[i % n_batches], sync_loss=True)   # H2D ids, D2H loss
        torch.cuda.synchronize()
        el = _max_over_ranks(time.perf_counter() - t0, world) / args.e2e_steps
        e2e = {"value": tokens_per_step / el, "unit": "tokens/s",
               "h2d_bytes_per_step": host[0].numel() * host[0].element_size(),
               "d2h_bytes_per_step": 4, "last_loss": loss}

    breakdown = _breakdown(trainer, model, dev[0], world) if args.breakdown else None
    if args.profile_table and rank == 0:
        _kernel_table(lambda: trainer.train_step(dev[0]), args.profile_table)
    elif args.profile_table:
        trainer.train_step(dev[0])                 # every rank takes the same collective steps
    launches = all_kernels = None
    if args.profile_launches:
        ours, total = _count_launches(lambda: trainer.train_step(dev[0]))
        launches = ours * args.steps
        all_kernels = total * args.steps
    mem = torch.cuda.max_memory_allocated() / 2 ** 30
    from mamformer_b200.utils.metrics import matmul_params_per_token
    n_mm = matmul_params_per_token(model)
    peak_tf, peak_src = _peak_tflops()
    mfu = {"value": round(value / world * 6.0 * n_mm / (peak_tf * 1e12), 4),
           "flops_per_token": 6.0 * n_mm, "matmul_params_per_token": n_mm, "peak_tflops_per_gpu": peak_tf,
           "peak": peak_src,
           "counts": "6 x matmul weights active per token (top-k experts, 1 + MTP-depth vocab heads); "
                     "attention scores, scans and recomputation not counted"}
    out = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / BASELINE_TOKS) if BASELINE_TOKS else None, "dtype": "bf16",
        "data": "synthetic uniform-random token ids, random-init weights",
        "impl": "mamformer_b200",
        "config": {"model": f"ultra-7b (configs/ultra-7b.yaml) depth-truncated to {args.layers} layers "
                            f"({cfg.layout_string()}), same per-layer shapes",
                   "global_batch": world * per_gpu, "seq_len": args.seq,
                   "micro_batch": args.micro_batch, "grad_accum": args.grad_accum,
                   "parallelism": parallelism, "checkpoint": args.checkpoint, "zero": args.zero,
                   "window_mode": args.window_mode,
                   "dp_transport": args.dp_transport if world > 1 else None,
                   "params_b": round(sum(p.numel() for p in model.parameters()) / 1e9, 3),
                   "l2": "working set >> L2 (inputs larger than L2)"},
        "clocks": clk, "e2e": e2e, "gpu_launches": launches, "all_kernel_launches": all_kernels,
        "peak_mem_gib": round(mem, 1), "mfu": mfu, "breakdown_ms": breakdown,
    }
    _emit(out, rank)


def run_reference(args, rank, world):
    """The unmodified reference (installed under baseline/_ref) through its public API: the
    same model config, fp32 weights + bf16 autocast + AdamW, the loop of its scripts/train.py
    (FSDP FULL_SHARD for N > 1, as that script does)."""
    import torch
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "mamformer")):
        _emit({"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}, rank)
        return
    sys.path.insert(0, ref_dir)
    from mamformer.config import MamformerConfig as RefConfig
    from mamformer.model import MamformerForCausalLM as RefModel
    cfg = RefConfig.from_dict(bench_config(args.layers))
    per_gpu = args.micro_batch * args.grad_accum
    try:
        torch.manual_seed(0)
        model = RefModel(cfg).cuda()
        if world > 1:
            from torch.distributed.fsdp import FullyShardedDataParallel as FSDP, MixedPrecision, ShardingStrategy
            from torch.distributed.fsdp.wrap import ModuleWrapPolicy
            from mamformer.layers.hybrid import MamformerBlock
            model = FSDP(model, sharding_strategy=ShardingStrategy.FULL_SHARD,
                         auto_wrap_policy=ModuleWrapPolicy({MamformerBlock}),
                         mixed_precision=MixedPrecision(param_dtype=torch.bfloat16, reduce_dtype=torch.bfloat16,
                                                        buffer_dtype=torch.bfloat16),
                         device_id=torch.cuda.current_device(), use_orig_params=True)
        decay, no_decay = [], []
        for n, p in model.named_parameters():
            (no_decay if any(k in n for k in ("norm", "bias", "gate", "alpha", "lambda_log", "A_log")) else decay).append(p)
        opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1}, {"params": no_decay, "weight_decay": 0.0}],
                                lr=2e-4, betas=(0.9, 0.95), eps=1e-8)
        model.train()
        g = torch.Generator().manual_seed(1234 + rank)
        batch = torch.randint(0, cfg.vocab_size, (per_gpu, args.seq), generator=g).cuda()

        def step():
            opt.zero_grad()
            for i in range(args.grad_accum):
                mb = batch[i * args.micro_batch:(i + 1) * args.micro_batch]
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    loss = model(mb, labels=mb)["loss"]
                (loss / args.grad_accum).backward()
            torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
            opt.step()

        for _ in range(args.warmup):
            step()
        _barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        torch.cuda.synchronize()
        ms = _max_over_ranks(s.elapsed_time(e), world) / args.steps
        value = world * per_gpu * args.seq / (ms / 1000.0)
        _emit({"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
               "config": {"model": f"ultra-7b truncated to {args.layers} layers", "global_batch": world * per_gpu,
                          "seq_len": args.seq, "parallelism": f"fsdp{world}" if world > 1 else "single"}}, rank)
    except torch.cuda.OutOfMemoryError as exc:
        msg = str(exc).split("\n")[0][:160]
        _emit({"impl": "reference", "unavailable": f"CUDA out of memory on a 180 GB B200 at seq {args.seq}, "
                                                   f"micro-batch {args.micro_batch}: {msg}"}, rank)
    except Exception as exc:   # e.g. the reference's own Triton kernel failing to compile
        import traceback
        traceback.print_exc(file=sys.stderr)
        _emit({"impl": "reference", "unavailable": "reference fails on its stock GPU path: "
                                                   + _exception_summary(exc)}, rank)


def _exception_summary(exc: BaseException) -> str:
    """One line: the exception's module-qualified type, the first and the last non-empty line
    of its message, and the innermost frame of the reference's own code that raised it."""
    import traceback
    lines = [ln.strip() for ln in str(exc).splitlines() if ln.strip()]
    msg = lines[0] if lines else ""
    if len(lines) > 1 and lines[-1] != msg:
        msg += " ... " + lines[-1]
    where = ""
    for fr in traceback.extract_tb(exc.__traceback__):
        if os.sep + "mamformer" + os.sep in fr.filename and "_ref" in fr.filename:
            where = f" [raised under {os.path.relpath(fr.filename, ROOT)}:{fr.lineno} in {fr.name}]"
    kind = type(exc)
    return f"{kind.__module__}.{kind.__qualname__}: {msg[:300]}{where}"


def run_tp(args, rank, world):
    """configs/7b.yaml tensor-parallel over every GPU: the sharded model computes the unsharded
    function, every rank sees the same token batch; the all-reduces after row-parallel GEMMs run
    as this repository's GEMM -> reduce-scatter + all-gather paths."""
    import torch
    from mamformer_b200 import ops
    from mamformer_b200.config import MamformerConfig
    from mamformer_b200.engine import TrainConfig, Trainer
    from mamformer_b200.models.model import MamformerForCausalLM
    from mamformer_b200.parallel import DistributedCoordinator, ParallelConfig
    from mamformer_b200.utils.clocks import ClockSampler
    if not ops.has_native():
        raise RuntimeError("native extension missing")
    cfg = MamformerConfig.from_yaml(os.path.join(ROOT, "configs", "7b.yaml"))
    seq = args.seq if args.seq != 4096 else 8192
    global_batch = 64
    mb = 1
    tcfg = TrainConfig(learning_rate=2e-4, warmup_steps=10, max_steps=1000, micro_batch=mb,
                       grad_accum=global_batch // mb)
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = MamformerForCausalLM(cfg)
    if args.checkpoint != "none":
        model.model.enable_gradient_checkpointing(all_layers=args.checkpoint == "all")
    if world > 1:
        coord = DistributedCoordinator(ParallelConfig(tp_size=world)).initialize()
        model = coord.shard_model(model)
    torch.cuda.empty_cache()
    trainer = Trainer(model, tcfg)
    g = torch.Generator().manual_seed(1234)                   # identical batch on every TP rank
    host = torch.randint(0, cfg.vocab_size, (global_batch, seq), generator=g).pin_memory()
    dev = host.cuda()
    for _ in range(args.warmup):
        trainer.train_step(dev)
    _barrier(world)
    clocks = ClockSampler(gpu_index=torch.cuda.current_device()).start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        trainer.train_step(dev)
    e.record()
    torch.cuda.synchronize()
    _barrier(world)
    clk = clocks.stop()
    ms = _max_over_ranks(s.elapsed_time(e), world) / args.steps
    value = global_batch * seq / (ms / 1000.0)
    e2e = None
    if not args.no_e2e and args.e2e_steps > 0:
        _barrier(world)
        t0 = time.perf_counter()
        loss = None
        for _ in range(args.e2e_steps):
            loss = trainer.train_step(host, sync_loss=True)
        torch.cuda.synchronize()
        el = _max_over_ranks(time.perf_counter() - t0, world) / args.e2e_steps
        e2e = {"value": global_batch * seq / el, "unit": "tokens/s",
               "h2d_bytes_per_step": host.numel() * host.element_size(), "d2h_bytes_per_step": 4,
               "last_loss": loss}
    from mamformer_b200.utils.metrics import matmul_params_per_token
    n_mm = matmul_params_per_token(model) * world              # the shards add up to the model
    peak_tf, peak_src = _peak_tflops()
    _emit({"metric": "train tokens/s per box, configs/7b.yaml dense hybrid bf16 TP over N B200, max over ranks",
           "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic uniform-random token ids, random-init weights", "impl": "mamformer_b200",
           "config": {"model": f"7b (configs/7b.yaml, {cfg.n_layers} layers, {cfg.layout_string()})",
                      "global_batch": global_batch, "seq_len": seq, "micro_batch": mb,
                      "grad_accum": global_batch // mb, "parallelism": f"tp{world}", "checkpoint": args.checkpoint,
                      "l2": "working set >> L2 (inputs larger than L2)"},
           "clocks": clk, "e2e": e2e, "peak_mem_gib": round(torch.cuda.max_memory_allocated() / 2 ** 30, 1),
           "mfu": {"value": round(value / world * 6.0 * n_mm / (peak_tf * 1e12), 4), "peak": peak_src,
                   "counts": "6 x matmul weights per token, approximate under TP (per-rank shards x N)"}}, rank)


def main():
    args = _args()
    rank, world, _ = _dist_init()
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.workload == "7b-tp":
            run_tp(args, rank, world)
        else:
            run_ours(args, rank, world)
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
