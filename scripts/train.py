#!/usr/bin/env python
"""Pre-training entry point (one GPU, or data-parallel over torchrun ranks).

Reference: ``scripts/train.py`` (CLI 579-649, loop 363-462, checkpoints 535-576).  Same flags;
``--bf16``/``--fp16`` select the compute dtype of the mixed-precision engine (fp32 masters);
``--ep N`` additionally shards the routed experts over N ranks (the rest stays data-parallel).
Without ``.bin`` shards in ``--data`` it trains on synthetic uniform-random tokens.

    torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node 8 scripts/train.py \\
        --config configs/ultra-7b.yaml --bf16 --ep 8
"""
import argparse
import logging
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402


def build_parser():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", required=True, help="model config YAML or preset name")
    p.add_argument("--data", default="./data", help="directory of pre-tokenised .bin shards")
    p.add_argument("--batch_size", type=int, default=1, help="micro-batch per GPU")
    p.add_argument("--gradient_accumulation_steps", type=int, default=8)
    p.add_argument("--learning_rate", type=float, default=3e-4)
    p.add_argument("--weight_decay", type=float, default=0.1)
    p.add_argument("--warmup_steps", type=int, default=2000)
    p.add_argument("--max_steps", type=int, default=100000)
    p.add_argument("--max_seq_len", type=int, default=8192)
    p.add_argument("--bf16", action="store_true")
    p.add_argument("--fp16", action="store_true")
    p.add_argument("--gradient_checkpointing", action="store_true", default=False)
    p.add_argument("--no_gradient_checkpointing", action="store_false", dest="gradient_checkpointing")
    p.add_argument("--output_dir", default="./checkpoints")
    p.add_argument("--save_every", type=int, default=5000)
    p.add_argument("--log_every", type=int, default=10)
    p.add_argument("--use_wandb", action="store_true", help="accepted for compatibility (metrics go to JSONL)")
    p.add_argument("--wandb_project", default="Mamformer")
    p.add_argument("--wandb_run_name", default=None)
    p.add_argument("--num_workers", type=int, default=0)
    p.add_argument("--resume", default=None, help="checkpoint file to resume from")
    p.add_argument("--comm_moe", action="store_true", help="enable CommunicativeMoE")
    p.add_argument("--thinking_format", action="store_true", help="accepted for compatibility")
    p.add_argument("--ep", type=int, default=1, help="expert-parallel size (routed experts sharded)")
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--zero", type=int, default=0, choices=[0, 1],
                   help="1: shard fp32 master weights and Adam moments over the data-parallel ranks")
    p.add_argument("--dp-transport", default="nccl", choices=["nccl", "p2p"],
                   help="data-parallel gradient sums: NCCL, or this repository's NVLink peer-memory kernels")
    return p


def train(args, parallel=None):
    import torch
    import torch.distributed as dist
    from mamformer_b200 import MamformerForCausalLM
    from mamformer_b200.checkpoint import load_checkpoint, save_checkpoint, save_sharded
    from mamformer_b200.data import PinnedBatchLoader, TokenShardDataset
    from mamformer_b200.engine import TrainConfig, Trainer
    from mamformer_b200.parallel import DistributedCoordinator, ParallelConfig
    from mamformer_b200.utils.metrics import MetricsLogger, setup_logging, train_flops_per_token

    rank, world, local, device = _common.init_distributed()
    log = setup_logging(rank)
    cfg = _common.load_config(args.config)
    if args.comm_moe:
        cfg.comm_moe.enabled = True
    seq = min(args.max_seq_len, cfg.max_seq_len)
    dtype = torch.bfloat16 if args.bf16 else (torch.float16 if args.fp16 else torch.float32)
    pc = parallel or ParallelConfig(dp_size=world // max(1, args.ep), ep_size=max(1, args.ep))
    coord = DistributedCoordinator(pc).initialize()
    torch.manual_seed(args.seed)
    model = MamformerForCausalLM(cfg).to(device)
    model = coord.shard_model(model)
    tcfg = TrainConfig(learning_rate=args.learning_rate, weight_decay=args.weight_decay,
                       warmup_steps=args.warmup_steps, max_steps=args.max_steps, micro_batch=args.batch_size,
                       grad_accum=args.gradient_accumulation_steps, compute_dtype=dtype,
                       gradient_checkpointing=args.gradient_checkpointing)
    trainer = Trainer(model, tcfg, dp_group=coord.get_group("dense_dp") if world > 1 else None,
                      expert_dp_group=coord.get_group("expert_dp"), ep_group=coord.get_group("ep"),
                      zero_stage=args.zero, dp_transport=args.dp_transport)
    start = 0
    if args.resume:
        start = load_checkpoint(args.resume, trainer.model, trainer.optimizer, trainer.scheduler)
        log.info("resumed from %s at step %d", args.resume, start)
    dp_rank = coord.get_rank("dp") * coord.get_size("ep") + coord.get_rank("ep")
    ds = TokenShardDataset(args.data, seq, seed=args.seed, rank=dp_rank, world=coord.get_size("dense_dp"),
                           vocab_size=cfg.vocab_size)
    if ds.synthetic:
        log.warning("no .bin shards in %s: training on synthetic uniform-random tokens", args.data)
    per_step = args.batch_size * args.gradient_accumulation_steps
    loader = PinnedBatchLoader(ds, per_step, device)
    metrics = MetricsLogger(args.output_dir, rank, world, train_flops_per_token(cfg, seq))
    log.info("config %s | %.2fB params (%.2fB active) | world %d | %s", args.config,
             cfg.num_parameters / 1e9, cfg.num_active_parameters / 1e9, world, pc)
    sharded = world > 1 and (pc.ep_size > 1 or pc.tp_size > 1 or pc.pp_size > 1)
    for step in range(start, args.max_steps):
        ids = next(loader)
        metrics.step_start()
        loss = trainer.train_step(ids, sync_loss=(step + 1) % args.log_every == 0)
        if (step + 1) % args.log_every == 0:
            metrics.step_end(step + 1, float(loss), per_step * seq, trainer.scheduler.get_last_lr()[0],
                             {"grad_norm": trainer.optimizer.grad_norm()})
        if args.save_every and (step + 1) % args.save_every == 0:
            _save(args, trainer, step + 1, sharded, rank)
    _save(args, trainer, args.max_steps, sharded, rank, final=True)
    loader.close()
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def _save(args, trainer, step, sharded, rank, final=False):
    from mamformer_b200.checkpoint import save_checkpoint, save_sharded
    name = "checkpoint_final" if final else f"checkpoint_step_{step}"
    if sharded:
        save_sharded(os.path.join(args.output_dir, name), trainer.model, trainer.optimizer, trainer.scheduler, step)
    else:   # every rank takes part (ZeRO gathers the fp32 weights); rank 0 writes
        save_checkpoint(os.path.join(args.output_dir, name + ".pt"), trainer.model, trainer.optimizer,
                        trainer.scheduler, step, write=rank == 0)


def main(argv=None):
    train(build_parser().parse_args(argv))


if __name__ == "__main__":
    main()
