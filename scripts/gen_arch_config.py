#!/usr/bin/env python
"""Write ``configs/_arch_verify.yaml`` (reference ``scripts/gen_arch_config.py``)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402,F401

if __name__ == "__main__":
    sys.path.insert(0, os.path.join(_common.ROOT, "configs"))
    import _gen_zoo
    _gen_zoo.main()
