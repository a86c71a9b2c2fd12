#!/usr/bin/env python
"""GRPO / S-GRPO reinforcement learning from an SFT checkpoint.

Reference: ``scripts/train_grpo.py`` (CLI 812-930, loop 250-715).  Rollouts, rule rewards,
group-normalised advantages, policy / frozen-reference log-probs and the KL-penalised loss run
in ``mamformer_b200.grpo.GRPOTrainer``; prompts come from a JSONL file (a dummy arithmetic set
when it is missing).
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402


def build_parser():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", required=True)
    p.add_argument("--checkpoint", required=True, help="SFT checkpoint ('none' = random init)")
    p.add_argument("--data", default="./data/grpo_prompts.jsonl")
    p.add_argument("--reward_type", default="math", help="default reward when a prompt names none")
    p.add_argument("--group_size", type=int, default=8)
    p.add_argument("--kl_beta", type=float, default=0.04)
    p.add_argument("--gen_max_tokens", type=int, default=1024)
    p.add_argument("--gen_temperature", type=float, default=1.0)
    p.add_argument("--gen_top_p", type=float, default=0.95)
    p.add_argument("--gen_top_k", type=int, default=50)
    p.add_argument("--batch_size", type=int, default=4)
    p.add_argument("--gradient_accumulation_steps", type=int, default=1)
    p.add_argument("--learning_rate", type=float, default=1e-6)
    p.add_argument("--weight_decay", type=float, default=0.1)
    p.add_argument("--warmup_steps", type=int, default=100)
    p.add_argument("--max_steps", type=int, default=10000)
    p.add_argument("--max_prompt_len", type=int, default=2048)
    p.add_argument("--sub_batch_size", type=int, default=0)
    p.add_argument("--bf16", action="store_true")
    p.add_argument("--fp16", action="store_true")
    p.add_argument("--gradient_checkpointing", action="store_true")
    p.add_argument("--max_grad_norm", type=float, default=1.0)
    p.add_argument("--output_dir", default="./grpo_checkpoints")
    p.add_argument("--save_every", type=int, default=500)
    p.add_argument("--log_every", type=int, default=10)
    p.add_argument("--eval_every", type=int, default=100)
    p.add_argument("--num_workers", type=int, default=2)
    p.add_argument("--resume", default=None)
    p.add_argument("--sgrpo", action="store_true")
    p.add_argument("--sgrpo_p", type=float, default=0.4)
    p.add_argument("--sgrpo_alpha", type=int, default=0)
    p.add_argument("--sgrpo_k", type=int, default=0)
    p.add_argument("--use_wandb", action="store_true")
    p.add_argument("--wandb_project", default="Mamformer-GRPO")
    p.add_argument("--wandb_run_name", default=None)
    return p


def main(argv=None):
    import torch
    from mamformer_b200.checkpoint import load_checkpoint, save_checkpoint
    from mamformer_b200.grpo import GRPOConfig, GRPOTrainer, PromptDataset, collate_prompts
    from mamformer_b200.sgrpo import StochasticGRPOConfig
    from mamformer_b200.tokenizer import MamformerTokenizer
    from mamformer_b200.utils.metrics import MetricsLogger, setup_logging

    args = build_parser().parse_args(argv)
    rank, world, local, device = _common.init_distributed()
    log = setup_logging(rank)
    ck = None if args.checkpoint.lower() == "none" else args.checkpoint
    policy, cfg = _common.load_model(args.config, ck, device)
    policy.train()
    tok = MamformerTokenizer()
    gcfg = GRPOConfig(group_size=args.group_size, gen_max_tokens=args.gen_max_tokens,
                      gen_temperature=args.gen_temperature, gen_top_k=args.gen_top_k, gen_top_p=args.gen_top_p,
                      kl_beta=args.kl_beta, learning_rate=args.learning_rate, weight_decay=args.weight_decay,
                      max_grad_norm=args.max_grad_norm, grad_accum=args.gradient_accumulation_steps,
                      sub_batch_size=args.sub_batch_size or None, warmup_steps=args.warmup_steps,
                      max_steps=args.max_steps,
                      sgrpo=StochasticGRPOConfig(enabled=args.sgrpo, p=args.sgrpo_p, alpha=args.sgrpo_alpha,
                                                 k=args.sgrpo_k))
    gcfg.sgrpo.validate()
    dtype = torch.bfloat16 if args.bf16 else (torch.float16 if args.fp16 else None)
    trainer = GRPOTrainer(policy, tok, gcfg, compute_dtype=dtype)
    if args.resume:
        trainer.global_step = load_checkpoint(args.resume, trainer.policy, trainer.optimizer, trainer.scheduler)
    ds = PromptDataset(args.data, tok, args.max_prompt_len)
    for it in ds.items:
        it.setdefault("reward_type", args.reward_type)
    dl = torch.utils.data.DataLoader(ds, batch_size=args.batch_size, shuffle=True, collate_fn=collate_prompts)
    metrics = MetricsLogger(args.output_dir, rank, world)
    while trainer.global_step < args.max_steps:
        for batch in dl:
            metrics.step_start()
            m = trainer.step(batch)
            s = trainer.global_step
            if s % args.log_every == 0:
                metrics.step_end(s, float(m["loss"]), int(m["response_tokens"]) * args.batch_size * args.group_size,
                                 trainer.scheduler.get_last_lr()[0],
                                 {k: m[k] for k in ("policy_loss", "kl_div", "mean_reward")})
            if args.save_every and s % args.save_every == 0 and rank == 0:
                save_checkpoint(os.path.join(args.output_dir, f"checkpoint_grpo_step_{s}.pt"), trainer.policy,
                                trainer.optimizer, trainer.scheduler, s)
            if s >= args.max_steps:
                break
    if rank == 0:
        save_checkpoint(os.path.join(args.output_dir, "checkpoint_final.pt"), trainer.policy, trainer.optimizer,
                        trainer.scheduler, trainer.global_step)


if __name__ == "__main__":
    main()
