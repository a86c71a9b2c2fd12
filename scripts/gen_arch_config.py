#!/usr/bin/env python
"""Write ``configs/_arch_verify.yaml``: the small model with every Ultra feature switched on
that the bit-parity tests build in both frameworks (reference: ``scripts/gen_arch_config.py``,
whose architecture values are kept).  The values live in ``configs/_gen_zoo.py``
(``arch_verify_config``), which also regenerates the rest of the zoo.

    python scripts/gen_arch_config.py [--out configs/_arch_verify.yaml]
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--out", default=os.path.join(_common.ROOT, "configs", "_arch_verify.yaml"))
    a = p.parse_args(argv)
    sys.path.insert(0, os.path.join(_common.ROOT, "configs"))
    import _gen_zoo
    cfg = _gen_zoo.arch_verify_config()
    cfg.to_yaml(a.out)
    print(f"Generated {a.out}: {cfg.summary()}")
    return a.out


if __name__ == "__main__":
    main()
