"""Failure detection and recovery for training jobs.

Reference behaviour (``scripts/train.py:378-447``): skip a step whose inputs or loss are not
finite; after 3 consecutive non-finite losses reload the newest ``checkpoint_step_*.pt``; zero the
gradients and skip when a periodic scan finds a non-finite gradient; on CUDA out-of-memory free
the cache, zero the gradients, write ``checkpoint_oom_recovery_step_N.pt`` and continue.

Added here (all detection happens on the host; nothing faults, traps or hangs a GPU):

* every in-kernel wait (the expert-parallel / tensor-parallel barrier, the GEMM and attention
  pipeline waits) is bounded and records an error code instead of hanging;
  :func:`check_device_status` reads those words after the stream has drained and raises
  :class:`CommTimeoutError` / :class:`KernelTimeoutError`;
* :class:`Heartbeat` publishes each rank's step and wall time in the ``torch.distributed`` store;
  :meth:`Heartbeat.check` raises :class:`RankFailureError` naming ranks that stopped advancing or
  reported a failure, so the others stop before their next collective instead of waiting for a
  timeout inside it;
* :class:`ResilientTrainer` wraps :class:`~mamformer_b200.engine.Trainer` with the reference's
  NaN / OOM policy, checkpoint rollback (skipping unreadable checkpoint files) and heartbeats.
"""

from __future__ import annotations

import glob
import logging
import math
import os
import re
import time
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

logger = logging.getLogger(__name__)


class CommTimeoutError(RuntimeError):
    """A bounded cross-GPU wait inside a kernel gave up (a peer did not arrive)."""


class KernelTimeoutError(RuntimeError):
    """A bounded pipeline wait inside the GEMM gave up."""


class RankFailureError(RuntimeError):
    """Another rank reported a failure or stopped sending heartbeats."""


def check_device_status(clear: bool = True) -> None:
    """Raise if a native kernel recorded a timeout (reads two device words; call between steps)."""
    from mamformer_b200.ops._ext import ext
    C = ext()
    if C is None or not torch.cuda.is_available():
        return
    comm = int(C.comm_error())
    gemm = int(C.gemm_error())
    if clear and comm:
        C.comm_clear_error()
    if clear and gemm:
        C.gemm_clear_error()
    # the attention kernels' words (forward, backward) are cleared by the read itself
    attn = 0
    for name in ("flash_tc_error", "flash_tc_bwd_error"):
        fn = getattr(C, name, None)
        if fn is not None:
            attn = attn or int(fn())
    if comm:
        raise CommTimeoutError(f"cross-GPU barrier timed out waiting for peer {comm - 100}")
    if gemm:
        raise KernelTimeoutError(f"tcgen05 GEMM pipeline wait timed out (code {gemm})")
    if attn:
        raise KernelTimeoutError(f"tcgen05 attention kernel reported code {attn} "
                                 "(a pipeline wait timed out, or a checked index was out of range)")


class Heartbeat:
    """Per-rank liveness through the process-group store (host side only)."""

    def __init__(self, store=None, rank: Optional[int] = None, world: Optional[int] = None,
                 stale_after_s: float = 300.0, prefix: str = "mamf_hb"):
        if store is None:
            from torch.distributed.distributed_c10d import _get_default_store
            store = _get_default_store()
        self.store = store
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.stale_after_s = stale_after_s
        self.prefix = prefix

    def beat(self, step: int) -> None:
        self.store.set(f"{self.prefix}/{self.rank}", f"{step}:{time.time():.3f}")

    def report_failure(self, reason: str) -> None:
        self.store.set(f"{self.prefix}/fail/{self.rank}", reason[:200])

    def status(self) -> dict:
        out = {}
        for r in range(self.world):
            try:
                if self.store.check([f"{self.prefix}/fail/{r}"]):
                    out[r] = ("failed", self.store.get(f"{self.prefix}/fail/{r}").decode())
                    continue
                if not self.store.check([f"{self.prefix}/{r}"]):
                    out[r] = ("absent", None)
                    continue
                step, ts = self.store.get(f"{self.prefix}/{r}").decode().split(":")
                out[r] = ("alive", (int(step), float(ts)))
            except Exception as e:          # store unreachable: treat as failure of that rank
                out[r] = ("failed", repr(e))
        return out

    def check(self, now: Optional[float] = None, require_all: bool = False) -> None:
        now = time.time() if now is None else now
        bad = []
        for r, (state, info) in self.status().items():
            if state == "failed":
                bad.append(f"rank {r} failed: {info}")
            elif state == "absent" and require_all:
                bad.append(f"rank {r} never reported")
            elif state == "alive" and now - info[1] > self.stale_after_s:
                bad.append(f"rank {r} silent for {now - info[1]:.0f}s (last step {info[0]})")
        if bad:
            raise RankFailureError("; ".join(bad))


def finite(x) -> bool:
    if torch.is_tensor(x):
        return bool(torch.isfinite(x).all())
    return math.isfinite(float(x))


def grads_finite(optimizer) -> bool:
    """One device reduction over every fp32 gradient buffer (or the .grad tensors)."""
    flags = []
    for _, seg in getattr(optimizer, "segments", []):
        flags.append(torch.isfinite(seg.grad).all())
    if not flags:
        for g in optimizer.param_groups:
            for p in g["params"]:
                if p.grad is not None:
                    flags.append(torch.isfinite(p.grad).all())
    return bool(torch.stack(flags).all()) if flags else True


def checkpoints_newest_first(directory: str) -> List[str]:
    found = []
    for p in glob.glob(os.path.join(directory, "checkpoint_step_*")):
        m = re.search(r"step_(\d+)", os.path.basename(p))
        if m:
            found.append((int(m.group(1)), p))
    return [p for _, p in sorted(found, reverse=True)]


@dataclass
class FaultPolicy:
    max_consecutive_nan: int = 3
    nan_grad_check_every: int = 100
    oom_recovery: bool = True
    checkpoint_dir: Optional[str] = None


class ResilientTrainer:
    """``train_step`` with the reference's failure handling around a :class:`Trainer`."""

    def __init__(self, trainer, policy: FaultPolicy = FaultPolicy(), heartbeat: Optional[Heartbeat] = None):
        self.trainer = trainer
        self.policy = policy
        self.heartbeat = heartbeat
        self.consecutive_nan = 0
        self.events: List[str] = []

    def _rollback(self) -> bool:
        from mamformer_b200.checkpoint import load_checkpoint
        for path in checkpoints_newest_first(self.policy.checkpoint_dir or "."):
            try:
                step = load_checkpoint(path, self.trainer.model, self.trainer.optimizer, self.trainer.scheduler)
            except Exception as e:        # unreadable / truncated file: try the next one
                self.events.append(f"skip unreadable checkpoint {os.path.basename(path)}: {type(e).__name__}")
                continue
            self.trainer.step_count = step
            self.events.append(f"rolled back to {os.path.basename(path)}")
            return True
        self.events.append("no usable checkpoint for rollback")
        return False

    def train_step(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None) -> Optional[float]:
        tr = self.trainer
        if self.heartbeat is not None:
            self.heartbeat.check()
        if input_ids.is_floating_point() and not finite(input_ids):
            self.events.append("skip: non-finite input")
            return None
        check = bool(self.policy.nan_grad_check_every) and (tr.step_count + 1) % self.policy.nan_grad_check_every == 0
        try:
            loss = tr.train_step(input_ids, labels, sync_loss=True, check_grads=check)
        except torch.cuda.OutOfMemoryError:
            if not self.policy.oom_recovery:
                raise
            torch.cuda.empty_cache()
            tr.optimizer.zero_grad()
            self.events.append("oom: cache freed, step skipped")
            if self.policy.checkpoint_dir:
                from mamformer_b200.checkpoint import save_checkpoint
                save_checkpoint(os.path.join(self.policy.checkpoint_dir,
                                             f"checkpoint_oom_recovery_step_{tr.step_count}.pt"),
                                tr.model, tr.optimizer, tr.scheduler, tr.step_count)
            return None
        if loss is None or not math.isfinite(loss):
            self.consecutive_nan += 1
            self.events.append(f"skip: non-finite loss ({self.consecutive_nan} in a row)")
            if self.consecutive_nan >= self.policy.max_consecutive_nan:
                self._rollback()
                self.consecutive_nan = 0
            return None
        self.consecutive_nan = 0
        if self.heartbeat is not None:
            self.heartbeat.beat(tr.step_count)
        return loss
