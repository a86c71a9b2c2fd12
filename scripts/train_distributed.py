#!/usr/bin/env python
"""4-D parallel pre-training (DP x TP x PP x EP) over torchrun ranks.

Reference: ``scripts/train_distributed.py`` (loop 124-353, CLI 384-432).  ``--dp/--tp/--pp/--ep``
define the layout (product = world size, rank order [DP][TP][PP][EP]).  PP > 1 runs the 1F1B
schedule with NCCL p2p between stages (micro-batches = ``--gradient_accumulation_steps``);
otherwise the loop of ``scripts/train.py`` runs on the sharded model.

    torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node 8 scripts/train_distributed.py \\
        --config configs/7b.yaml --bf16 --tp 8
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402
import train as _train  # noqa: E402


def build_parser():
    p = _train.build_parser()
    p.add_argument("--dp", type=int, default=1)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--pp", type=int, default=1)
    p.set_defaults(gradient_checkpointing=True)
    return p


def train_pipeline(args, pc):
    import torch
    import torch.distributed as dist
    from mamformer_b200 import MamformerForCausalLM
    from mamformer_b200.checkpoint import save_sharded
    from mamformer_b200.data import PinnedBatchLoader, TokenShardDataset
    from mamformer_b200.optim import MixedPrecisionAdamW, create_lr_scheduler, param_groups
    from mamformer_b200.parallel import DistributedCoordinator, PipelineScheduler1F1B
    from mamformer_b200.utils.metrics import MetricsLogger, setup_logging, train_flops_per_token
    from mamformer_b200.utils.precision import to_compute_dtype

    rank, world, local, device = _common.init_distributed()
    log = setup_logging(rank)
    cfg = _common.load_config(args.config)
    seq = min(args.max_seq_len, cfg.max_seq_len)
    dtype = torch.bfloat16 if args.bf16 else torch.float32
    coord = DistributedCoordinator(pc).initialize()
    torch.manual_seed(args.seed)
    stage = coord.shard_model(MamformerForCausalLM(cfg).to(device))
    if dtype != torch.float32:
        to_compute_dtype(stage, dtype)
    stage.model.return_logits = False
    stage.model.train()
    if args.gradient_checkpointing:
        stage.enable_gradient_checkpointing()
    expert = [p for p in stage.parameters() if getattr(p, "_mamf_expert", False)] or None
    opt = MixedPrecisionAdamW(param_groups(stage, args.weight_decay), lr=args.learning_rate,
                              weight_decay=args.weight_decay, dp_group=coord.get_group("dense_dp"),
                              no_dp_reduce=expert, expert_dp_group=coord.get_group("expert_dp"),
                              ep_group=coord.get_group("ep"))
    sched = create_lr_scheduler(opt, args.warmup_steps, args.max_steps, args.learning_rate)
    m = args.gradient_accumulation_steps
    pipe = PipelineScheduler1F1B(stage, m, cfg.d_model, dtype=dtype)
    emb = dist.new_group(stage.embedding_group_members()) if pc.pp_size > 1 else None
    dp_rank = coord.get_rank("dp") * coord.get_size("ep") + coord.get_rank("ep")
    ds = TokenShardDataset(args.data, seq, seed=args.seed, rank=dp_rank, world=coord.get_size("dense_dp"),
                           vocab_size=cfg.vocab_size)
    loader = PinnedBatchLoader(ds, args.batch_size * m, device)
    metrics = MetricsLogger(args.output_dir, rank, world, train_flops_per_token(cfg, seq))
    for step in range(args.max_steps):
        ids = next(loader)
        metrics.step_start()
        opt.zero_grad()
        loss = pipe.run_forward_backward(ids)
        pipe.sync_tied_embedding_grads(emb)
        opt.step()
        sched.step()
        if (step + 1) % args.log_every == 0:
            lv = torch.zeros(1, device=device) if loss is None else loss.detach().reshape(1).float()
            if stage.is_last is False:
                lv.zero_()
            dist.all_reduce(lv, group=coord.get_group("pp")) if coord.get_group("pp") is not None else None
            metrics.step_end(step + 1, float(lv), args.batch_size * m * seq, sched.get_last_lr()[0])
        if args.save_every and (step + 1) % args.save_every == 0:
            save_sharded(os.path.join(args.output_dir, f"checkpoint_step_{step + 1}"), stage.model, opt, sched, step + 1)
    loader.close()
    dist.barrier()
    dist.destroy_process_group()


def main(argv=None):
    from mamformer_b200.parallel import ParallelConfig
    args = build_parser().parse_args(argv)
    pc = ParallelConfig(dp_size=args.dp, tp_size=args.tp, pp_size=args.pp, ep_size=args.ep)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if pc.world_size != world:
        raise SystemExit(f"dp*tp*pp*ep = {pc.world_size} but WORLD_SIZE = {world}")
    if pc.pp_size > 1:
        train_pipeline(args, pc)
    else:
        _train.train(args, parallel=pc)


if __name__ == "__main__":
    main()
