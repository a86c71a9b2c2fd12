#!/usr/bin/env python
"""Text generation: one prompt or an interactive loop, optional thinking modes.

Reference: ``scripts/generate.py`` (CLI 202-276): sampling flags, beam search, repetition
penalty, thinking mode (NoThink / FastThink / CoreThink / DeepThink) with budgets and paths.
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402


def build_parser():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", required=True)
    p.add_argument("--checkpoint", default=None)
    p.add_argument("--prompt", default=None)
    p.add_argument("--device", default="cpu")
    p.add_argument("--max_new_tokens", type=int, default=256)
    p.add_argument("--temperature", type=float, default=0.7)
    p.add_argument("--top_k", type=int, default=50)
    p.add_argument("--top_p", type=float, default=0.9)
    p.add_argument("--repetition_penalty", type=float, default=1.0)
    p.add_argument("--num_beams", type=int, default=1)
    p.add_argument("--thinking", default=None, help="NoThink | FastThink | CoreThink | DeepThink")
    p.add_argument("--think_budget", type=int, default=0)
    p.add_argument("--num_paths", type=int, default=0)
    p.add_argument("--summary_budget", type=int, default=0)
    p.add_argument("--show_thinking", action="store_true")
    p.add_argument("--bf16", action="store_true")
    p.add_argument("--seed", type=int, default=42, help="seeds the weights of a model built without a checkpoint "
                                                         "and the sampling")
    return p


def generate_text(model, tok, prompt, args):
    import torch
    from mamformer_b200.generation import RuntimeGenerationConfig
    from mamformer_b200.thinking import ThinkingConfig
    dev = next(model.parameters()).device
    ids = torch.tensor([tok.encode(prompt, add_bos=True)], device=dev)
    model.config.generation.repetition_penalty = args.repetition_penalty
    if args.thinking and args.thinking != "NoThink":
        tc = ThinkingConfig.from_preset(args.thinking, args.think_budget, args.num_paths, args.summary_budget,
                                        args.show_thinking)
        out = model.generate(ids, max_new_tokens=args.max_new_tokens, temperature=args.temperature,
                             top_k=args.top_k, top_p=args.top_p, eos_token_id=tok.eos_token_id, thinking_config=tc)
        seq = out["generated_ids"] if isinstance(out, dict) else out
    elif args.num_beams > 1:
        seq = model.generate_ids(ids, num_beams=args.num_beams, max_new_tokens=args.max_new_tokens, temperature=0.0,
                                 eos_token_id=tok.eos_token_id)
    else:
        seq = model.generate(ids, max_new_tokens=args.max_new_tokens, temperature=args.temperature,
                             top_k=args.top_k, top_p=args.top_p, eos_token_id=tok.eos_token_id)
    return tok.decode(seq[0, ids.shape[1]:].tolist(), skip_special_tokens=not args.show_thinking)


def main(argv=None):
    import torch
    from mamformer_b200.tokenizer import MamformerTokenizer
    args = build_parser().parse_args(argv)
    torch.manual_seed(args.seed)
    model, cfg = _common.load_model(args.config, args.checkpoint, args.device,
                                    torch.bfloat16 if args.bf16 else None)
    tok = MamformerTokenizer()
    if args.prompt is not None:
        print(generate_text(model, tok, args.prompt, args))
        return
    print("interactive mode: empty line to quit")
    while True:
        try:
            line = input(">>> ")
        except EOFError:
            break
        if not line.strip():
            break
        print(generate_text(model, tok, line, args))


if __name__ == "__main__":
    main()
