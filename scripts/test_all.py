#!/usr/bin/env python
"""Run the test suite: CPU tests, the gloo multi-process tests and (with a GPU) the GPU tests.

Reference: ``scripts/test_all.py`` (module import checks, a forward/backward per preset and a
2-rank gloo distributed check).  Here the same coverage lives in ``tests/``; this wrapper runs it.
"""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def main():
    import torch
    marks = "not gpu" if not torch.cuda.is_available() else "gpu or not gpu"
    rc = subprocess.call([sys.executable, "-m", "pytest", os.path.join(ROOT, "tests"), "-q", "-m", marks], cwd=ROOT)
    sys.exit(rc)


if __name__ == "__main__":
    main()
