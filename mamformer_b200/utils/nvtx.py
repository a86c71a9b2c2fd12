"""NVTX ranges for profilers (Nsight Systems / ncu ``--nvtx``) around layers and collectives.

``rng(name)`` is a context manager that pushes an NVTX range on CUDA builds and does nothing on
CPU.  Ranges are on unless ``MAMF_NVTX=0``; with no profiler attached a push / pop pair costs
well under a microsecond of host time and nothing on the device.
"""

from __future__ import annotations

import contextlib
import os

import torch

_ON = os.environ.get("MAMF_NVTX", "1") != "0" and torch.cuda.is_available()


@contextlib.contextmanager
def rng(name: str):
    if not _ON:
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def enabled() -> bool:
    return _ON


class PhaseTimer:
    """CUDA-event marks on the current stream; ``summary()`` gives milliseconds per phase name
    (the time from the previous mark to the mark carrying the name), summed over calls.  Off
    unless ``enabled`` (no events recorded, no synchronisation)."""

    def __init__(self, enabled: bool = False):
        self.enabled = enabled
        self._marks = []

    def mark(self, name: str) -> None:
        if self.enabled:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._marks.append((name, ev))

    def reset(self) -> None:
        self._marks = []

    def summary(self) -> dict:
        if not self._marks:
            return {}
        torch.cuda.synchronize()
        out: dict = {}
        for (_, a), (name, b) in zip(self._marks[:-1], self._marks[1:]):
            if name.startswith("begin"):
                continue
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


def ranged(name: str):
    """Decorator: run the function inside ``rng(name)``."""
    import functools

    def deco(fn):
        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            with rng(name):
                return fn(*args, **kwargs)
        return wrapper
    return deco
