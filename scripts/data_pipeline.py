#!/usr/bin/env python
"""Curate raw documents into a domain-mixed JSONL corpus (then ``prepare_data.py`` tokenises it).

Reference: ``scripts/data_pipeline.py`` (CLI 1045-1098).  Reads a directory of JSON/JSONL/CSV/
HTML/Markdown/LaTeX/code/text files, filters, scores, near-deduplicates and classifies documents,
and writes ``mixed.jsonl`` plus ``pipeline_stats.json``.
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402,F401


def main(argv=None):
    from mamformer_b200.data_pipeline import DataMixConfig, DataPipeline
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--input", required=True, help="input directory or file")
    p.add_argument("--output", required=True)
    p.add_argument("--config", default=os.path.join(_common.ROOT, "configs", "data_mix.yaml"))
    p.add_argument("--domain", default=None, help="force every document into one domain")
    a = p.parse_args(argv)
    pipe = DataPipeline(DataMixConfig.from_yaml(a.config) if os.path.exists(a.config) else None, a.domain)
    if os.path.isdir(a.input):
        pipe.process_directory(a.input)
    else:
        pipe.process_file(a.input)
    pipe.save_mixer_state(a.output)
    print(pipe.generate_report())


if __name__ == "__main__":
    main()
