#!/usr/bin/env python
"""Download Chinese pre-training datasets from the Hugging Face hub into JSONL (same CLI as download_data.py).

Reference: ``scripts/download_data.py`` / ``download_cn.py``.  Needs network access and the
``datasets`` package; on an offline machine it says so and exits with status 2.
"""
import argparse
import json
import os
import sys


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--dataset", required=True, help="hub dataset id")
    p.add_argument("--split", default="train")
    p.add_argument("--text_field", default="text")
    p.add_argument("--output", required=True, help="output JSONL path")
    p.add_argument("--max_docs", type=int, default=0)
    a = p.parse_args(argv)
    try:
        from datasets import load_dataset
    except ImportError:
        print("the 'datasets' package is not installed (and the hub needs network access)", file=sys.stderr)
        sys.exit(2)
    ds = load_dataset(a.dataset, split=a.split, streaming=True)
    os.makedirs(os.path.dirname(os.path.abspath(a.output)), exist_ok=True)
    with open(a.output, "w", encoding="utf-8") as f:
        for i, row in enumerate(ds):
            if a.max_docs and i >= a.max_docs:
                break
            f.write(json.dumps({"text": row.get(a.text_field, "")}, ensure_ascii=False) + "\n")


if __name__ == "__main__":
    main()
