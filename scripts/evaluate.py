#!/usr/bin/env python
"""Benchmark evaluation: multiple-choice likelihood (MMLU, HellaSwag, ARC), GSM8K, HumanEval.

Reference: ``scripts/evaluate.py`` (BENCHMARKS 46-110, scorers 116-461, ``evaluate`` 464-568).
Items are read from local JSONL files ``<data_dir>/<benchmark>.jsonl`` (this machine has no
network for the hub datasets the reference downloads):

* multiple choice: ``{"question", "choices": [...], "answer": index}`` - the choice with the
  highest length-normalised log-likelihood wins;
* gsm8k: ``{"question", "answer"}`` - greedy generation, last number compared numerically;
* humaneval: ``{"prompt", "test_cases": [...], "entry_point"}`` - generated code run through the
  sandboxed code reward.
"""
import argparse
import json
import os
import re
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402

BENCHMARKS = {"mmlu": "mc", "hellaswag": "mc", "arc_easy": "mc", "arc_challenge": "mc", "gsm8k": "gen",
              "humaneval": "code"}


def _items(data_dir, name, max_samples):
    path = os.path.join(data_dir, f"{name}.jsonl")
    if not os.path.exists(path):
        return None
    out = [json.loads(l) for l in open(path, encoding="utf-8") if l.strip()]
    return out[:max_samples] if max_samples else out


def choice_logprob(model, tok, context: str, continuation: str) -> float:
    import torch
    dev = next(model.parameters()).device
    ctx = tok.encode(context, add_bos=True)
    cont = tok.encode(continuation, add_bos=False)
    ids = torch.tensor([ctx + cont], device=dev)
    labels = ids.clone()
    labels[:, : len(ctx)] = -100
    with torch.no_grad():
        return float(model.get_log_probs(ids, labels=labels))      # mean over the continuation


def eval_mc(model, tok, items):
    correct = 0
    for it in items:
        ctx = f"Question: {it['question']}\nAnswer:"
        scores = [choice_logprob(model, tok, ctx, " " + str(c)) for c in it["choices"]]
        correct += int(max(range(len(scores)), key=scores.__getitem__) == int(it["answer"]))
    return correct / max(1, len(items))


def _last_number(s):
    m = re.findall(r"-?\d+(?:\.\d+)?", s.replace(",", ""))
    return float(m[-1]) if m else None


def eval_gsm8k(model, tok, items, max_new_tokens=256):
    import torch
    dev = next(model.parameters()).device
    ok = 0
    for it in items:
        ids = torch.tensor([tok.encode(f"Question: {it['question']}\nAnswer:", add_bos=True)], device=dev)
        out = model.generate(ids, max_new_tokens=max_new_tokens, temperature=0.0, eos_token_id=tok.eos_token_id)
        got = _last_number(tok.decode(out[0, ids.shape[1]:].tolist()))
        want = _last_number(str(it["answer"]).split("####")[-1])
        ok += int(got is not None and want is not None and abs(got - want) < 1e-6)
    return ok / max(1, len(items))


def eval_humaneval(model, tok, items, max_new_tokens=384):
    import torch
    from mamformer_b200.rewards import code_reward
    dev = next(model.parameters()).device
    tot = 0.0
    for it in items:
        ids = torch.tensor([tok.encode(it["prompt"], add_bos=True)], device=dev)
        out = model.generate(ids, max_new_tokens=max_new_tokens, temperature=0.0, eos_token_id=tok.eos_token_id)
        body = it["prompt"] + tok.decode(out[0, ids.shape[1]:].tolist())
        tot += float(code_reward("```python\n" + body + "\n```", it.get("test_cases", []),
                                 it.get("entry_point", "solution")) == 1.0)
    return tot / max(1, len(items))


def evaluate(model, tok, benchmarks, data_dir, max_samples=100):
    res = {}
    for b in benchmarks:
        items = _items(data_dir, b, max_samples)
        if items is None:
            res[b] = None
            continue
        kind = BENCHMARKS[b]
        res[b] = eval_mc(model, tok, items) if kind == "mc" else (
            eval_gsm8k(model, tok, items) if kind == "gen" else eval_humaneval(model, tok, items))
    return res


def main(argv=None):
    from mamformer_b200.tokenizer import MamformerTokenizer
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", required=True)
    p.add_argument("--checkpoint", default=None)
    p.add_argument("--benchmarks", default="all", help="comma list or 'all': " + ",".join(BENCHMARKS))
    p.add_argument("--device", default="cpu")
    p.add_argument("--max_samples", type=int, default=100)
    p.add_argument("--data_dir", default="./data/eval")
    args = p.parse_args(argv)
    model, _ = _common.load_model(args.config, args.checkpoint, args.device)
    names = list(BENCHMARKS) if args.benchmarks == "all" else [b.strip() for b in args.benchmarks.split(",")]
    res = evaluate(model, MamformerTokenizer(), names, args.data_dir, args.max_samples)
    for k, v in res.items():
        print(f"{k:15s} {'no data in ' + args.data_dir if v is None else f'{100 * v:.2f}%'}")
    print(json.dumps(res))


if __name__ == "__main__":
    main()
