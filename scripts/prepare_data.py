#!/usr/bin/env python
"""Tokenise JSONL / text into ``.bin`` shards (+ ``metadata.json``) for pre-training.

Reference: ``scripts/prepare_data.py`` (77-233): documents are tokenised with BOS/EOS, packed
into ``seq_len + 1``-token chunks written round-robin to ``num_shards`` files (uint16, uint32 for
vocabularies of 65536 or more).
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402


def iter_documents(path, input_type, text_field="text", max_docs=0):
    n = 0
    with open(path, encoding="utf-8") as f:
        if input_type == "txt":
            docs = (d for d in f.read().split("\n\n") if d.strip())
        else:
            docs = (json.loads(l).get(text_field, "") for l in f if l.strip())
        for d in docs:
            yield d
            n += 1
            if max_docs and n >= max_docs:
                return


def main(argv=None):
    from mamformer_b200.data import write_shards
    from mamformer_b200.tokenizer import MamformerTokenizer
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--input", required=True, help="JSONL or TXT file")
    p.add_argument("--input_type", default="jsonl", choices=["jsonl", "txt", "hf"])
    p.add_argument("--hf_split", default="train")
    p.add_argument("--hf_text_field", default="text")
    p.add_argument("--output", required=True)
    p.add_argument("--tokenizer", default="simple", help="'simple' (byte-level) or a local HF tokenizer path")
    p.add_argument("--seq_len", type=int, default=8192)
    p.add_argument("--num_shards", type=int, default=64)
    p.add_argument("--max_docs", type=int, default=0)
    args = p.parse_args(argv)
    if args.input_type == "hf":
        raise SystemExit("hub datasets need network access; export them to JSONL first")
    if args.tokenizer == "simple":
        tok = MamformerTokenizer()
    else:
        from transformers import AutoTokenizer
        tok = MamformerTokenizer(AutoTokenizer.from_pretrained(args.tokenizer, local_files_only=True))
    stream = (tok.encode(d, add_bos=True, add_eos=True) for d in
              iter_documents(args.input, args.input_type, args.hf_text_field, args.max_docs))
    meta = write_shards(stream, args.output, args.seq_len, tok.vocab_size, args.num_shards)
    print(json.dumps(meta))


if __name__ == "__main__":
    main()
