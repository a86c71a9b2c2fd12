"""Parallel-runtime diagnostics: communication timing, expert load balance, pipeline bubble.

Reference: ``mamformer/parallelism/diagnostics.py`` (``CommOpStats`` 45-62, ``StepStats`` 65-78,
``ExpertLoadStats`` 81-91, ``CommMonitor`` 94-178, ``LoadBalanceAnalyzer`` 181-302,
``PipelineBubbleAnalyzer`` 305-369, ``ParallelismMonitor`` 372-565).  Same reports and
thresholds (collapse below normalised entropy 0.5, starvation below 1% of the mean load,
overload above 5x, bubble (p-1)/(p-1+m)).  Differences: on CUDA, communication and compute
intervals are timed with CUDA events on the current stream and resolved lazily (no host
synchronisation per call; the reference brackets asynchronous GPU work with
``time.perf_counter``); ``ParallelismMonitor.reset`` resets its analyzers (the reference calls
``reset`` methods the analyzers do not have).
"""

from __future__ import annotations

import logging
import math
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

logger = logging.getLogger(__name__)


@dataclass
class CommOpStats:
    total_time: float = 0.0
    count: int = 0
    total_bytes: int = 0
    current_start: Optional[object] = None

    @property
    def avg_time_ms(self) -> float:
        return self.total_time / max(self.count, 1) * 1000.0

    @property
    def total_bandwidth_gbps(self) -> float:
        return 0.0 if self.total_time == 0 else self.total_bytes / self.total_time / 1e9


@dataclass
class StepStats:
    step: int = 0
    compute_time: float = 0.0
    comm_time: float = 0.0
    loss: float = 0.0
    tokens_per_second: float = 0.0
    pipeline_bubble_ratio: float = 0.0

    @property
    def compute_comm_ratio(self) -> float:
        return self.compute_time / max(self.comm_time, 1e-8)


@dataclass
class ExpertLoadStats:
    layer_idx: int = 0
    per_expert_load: List[float] = field(default_factory=list)
    load_entropy: float = 0.0
    max_load_ratio: float = 0.0
    idle_experts: int = 0


class _Timer:
    """Interval timer: CUDA events when a GPU is in use, wall clock otherwise."""

    def __init__(self, use_cuda: Optional[bool] = None):
        self.cuda = torch.cuda.is_available() if use_cuda is None else use_cuda
        self._open: List[Tuple] = []     # unresolved (start, end, sink)

    def start(self):
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            return e
        return time.perf_counter()

    def stop(self, start, sink) -> None:
        """``sink(seconds)`` is called once the interval is known."""
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._open.append((start, e, sink))
        else:
            sink(time.perf_counter() - start)

    def resolve(self) -> None:
        if not self._open:
            return
        self._open[-1][1].synchronize()
        for s, e, sink in self._open:
            sink(s.elapsed_time(e) / 1000.0)
        self._open.clear()


class CommMonitor:
    def __init__(self, use_cuda: Optional[bool] = None):
        self.ops: Dict[str, CommOpStats] = {}
        self.compute_time = 0.0
        self._timer = _Timer(use_cuda)
        self._compute_start = None

    def start_compute(self) -> None:
        self._compute_start = self._timer.start()

    def end_compute(self) -> None:
        if self._compute_start is not None:
            self._timer.stop(self._compute_start, self._add_compute)
            self._compute_start = None

    def _add_compute(self, dt: float) -> None:
        self.compute_time += dt

    def start_comm(self, op_name: str, tensor_size: Optional[int] = None) -> None:
        st = self.ops.setdefault(op_name, CommOpStats())
        st.current_start = self._timer.start()
        if tensor_size:
            st.total_bytes += int(tensor_size)

    def end_comm(self, op_name: str) -> None:
        st = self.ops.get(op_name)
        if st is None or st.current_start is None:
            return

        def sink(dt, st=st):
            st.total_time += dt
        self._timer.stop(st.current_start, sink)
        st.count += 1
        st.current_start = None

    def get_total_comm_time(self) -> float:
        self._timer.resolve()
        return sum(s.total_time for s in self.ops.values())

    def get_bottleneck_ops(self, top_k: int = 5) -> List[Tuple[str, CommOpStats]]:
        self._timer.resolve()
        return sorted(self.ops.items(), key=lambda kv: kv[1].total_time, reverse=True)[:top_k]

    def get_summary(self) -> dict:
        self._timer.resolve()
        total = sum(s.total_time for s in self.ops.values())
        return {
            "total_comm_time_ms": total * 1000.0,
            "total_compute_time_ms": self.compute_time * 1000.0,
            "compute_comm_ratio": self.compute_time / max(total, 1e-8),
            "ops": {k: {"count": v.count, "avg_ms": v.avg_time_ms, "total_ms": v.total_time * 1000.0,
                        "GB/s": v.total_bandwidth_gbps} for k, v in self.ops.items()},
        }

    def reset(self) -> None:
        self._timer.resolve()
        self.ops.clear()
        self.compute_time = 0.0


class LoadBalanceAnalyzer:
    def __init__(self, n_layers: int, n_experts_per_layer: int):
        self.n_layers = n_layers
        self.n_experts = n_experts_per_layer
        self._load_ema: Dict[int, torch.Tensor] = {}
        self._ema_decay = 0.99
        self.collapse_threshold = 0.5
        self.starvation_pct = 0.01
        self.overload_ratio = 5.0

    def update(self, layer_idx: int, expert_counts: torch.Tensor) -> None:
        c = expert_counts.detach().float().cpu()
        tot = float(c.sum())
        if tot == 0:
            return
        load = c / tot
        prev = self._load_ema.get(layer_idx)
        self._load_ema[layer_idx] = load if prev is None else self._ema_decay * prev + (1 - self._ema_decay) * load

    def analyze_layer(self, layer_idx: int) -> ExpertLoadStats:
        load = self._load_ema.get(layer_idx)
        if load is None:
            return ExpertLoadStats(layer_idx=layer_idx)
        n = load.numel()
        nz = load[load > 0]
        ent = float(-(nz * nz.log()).sum())
        max_ent = math.log(n) if n > 1 else 1.0
        avg = 1.0 / n
        return ExpertLoadStats(layer_idx=layer_idx, per_expert_load=load.tolist(),
                               load_entropy=ent / max_ent if max_ent > 0 else 0.0,
                               max_load_ratio=float(load.max()) / avg,
                               idle_experts=int((load < self.starvation_pct * avg).sum()))

    def get_warnings(self) -> List[str]:
        out = []
        for i in range(self.n_layers):
            if i not in self._load_ema:      # no data (a fully collapsed layer has entropy 0 and is reported)
                continue
            st = self.analyze_layer(i)
            if st.load_entropy < self.collapse_threshold:
                out.append(f"Layer {i}: EXPERT COLLAPSE - entropy={st.load_entropy:.3f}, "
                           f"{st.idle_experts} idle experts, max load={st.max_load_ratio:.1f}x avg")
            elif st.idle_experts > 0:
                out.append(f"Layer {i}: {st.idle_experts} experts starved "
                           f"(<{self.starvation_pct * 100:.0f}% avg load)")
            if st.max_load_ratio > self.overload_ratio:
                out.append(f"Layer {i}: expert overloaded ({st.max_load_ratio:.1f}x avg)")
        return out

    def get_summary(self) -> dict:
        stats = [self.analyze_layer(i) for i in range(self.n_layers) if i in self._load_ema]
        if not stats:
            return {"status": "no_data"}
        ents = [s.load_entropy for s in stats]
        return {"avg_load_entropy": f"{sum(ents) / len(ents):.4f}", "min_load_entropy": f"{min(ents):.4f}",
                "total_idle_experts": sum(s.idle_experts for s in stats),
                "max_load_ratio": f"{max(s.max_load_ratio for s in stats):.1f}x",
                "status": "HEALTHY" if min(ents) > self.collapse_threshold else "WARNING: collapse detected"}

    def reset(self) -> None:
        self._load_ema.clear()


class PipelineBubbleAnalyzer:
    def __init__(self, pp_size: int, num_microbatches: int):
        self.pp_size = pp_size
        self.num_microbatches = num_microbatches
        self.theoretical_bubble = ((pp_size - 1) / (pp_size - 1 + num_microbatches)) if pp_size > 1 else 0.0
        self._compute, self._idle = [], []

    def record_step(self, compute_time: float, idle_time: float) -> None:
        self._compute.append(compute_time)
        self._idle.append(idle_time)

    def get_actual_bubble_ratio(self) -> float:
        tot = sum(self._compute) + sum(self._idle)
        return sum(self._idle) / tot if tot > 0 else 0.0

    def get_efficiency(self) -> float:
        return 1.0 - self.get_actual_bubble_ratio()

    def _get_recommendation(self) -> str:
        actual = self.get_actual_bubble_ratio()
        if self.pp_size <= 1:
            return "no pipeline parallelism"
        if actual > 0.3:
            return f"bubble {actual:.0%}: raise micro-batches above {4 * self.pp_size}"
        if actual > self.theoretical_bubble * 1.5:
            return "bubble well above theory: check stage balance and p2p overlap"
        return "pipeline healthy"

    def get_summary(self) -> dict:
        return {"pp_size": self.pp_size, "num_microbatches": self.num_microbatches,
                "theoretical_bubble": self.theoretical_bubble, "actual_bubble": self.get_actual_bubble_ratio(),
                "efficiency": self.get_efficiency(), "recommendation": self._get_recommendation()}

    def reset(self) -> None:
        self._compute.clear()
        self._idle.clear()


class ParallelismMonitor:
    """Aggregates the three analyzers; logs every ``log_interval`` steps on rank 0."""

    def __init__(self, n_layers: int = 0, n_experts: int = 0, pp_size: int = 1, num_microbatches: int = 1,
                 log_interval: int = 100, rank: int = 0, use_cuda: Optional[bool] = None):
        self.comm = CommMonitor(use_cuda)
        self.load = LoadBalanceAnalyzer(n_layers, n_experts)
        self.bubble = PipelineBubbleAnalyzer(pp_size, num_microbatches)
        self.log_interval = log_interval
        self.rank = rank
        self.history: List[StepStats] = []
        self._step_start = None

    def start_step(self) -> None:
        self._step_start = time.perf_counter()
        self.comm.reset()

    def start_compute(self) -> None:
        self.comm.start_compute()

    def end_compute(self) -> None:
        self.comm.end_compute()

    def comm_start(self, op_name: str, tensor_size: Optional[int] = None) -> None:
        self.comm.start_comm(op_name, tensor_size)

    def comm_end(self, op_name: str) -> None:
        self.comm.end_comm(op_name)

    def update_expert_load(self, layer_idx: int, expert_counts: torch.Tensor) -> None:
        self.load.update(layer_idx, expert_counts)

    def end_step(self, global_step: int, loss: float, tokens_processed: int = 0) -> StepStats:
        wall = time.perf_counter() - (self._step_start or time.perf_counter())
        comm = self.comm.get_total_comm_time()
        st = StepStats(step=global_step, compute_time=self.comm.compute_time, comm_time=comm, loss=float(loss),
                       tokens_per_second=tokens_processed / wall if wall > 0 else 0.0,
                       pipeline_bubble_ratio=self.bubble.theoretical_bubble)
        self.history.append(st)
        if self.rank == 0 and self.log_interval and global_step % self.log_interval == 0:
            self._log_diagnostics(global_step)
        return st

    def _log_diagnostics(self, step: int) -> None:
        s = self.history[-1]
        logger.info("[step %d] loss=%.4f tok/s=%.0f compute=%.1fms comm=%.1fms ratio=%.2f", step, s.loss,
                    s.tokens_per_second, s.compute_time * 1e3, s.comm_time * 1e3, s.compute_comm_ratio)
        for name, op in self.comm.get_bottleneck_ops(3):
            logger.info("  comm %-20s %6d calls  %.3f ms avg  %.1f GB/s", name, op.count, op.avg_time_ms,
                        op.total_bandwidth_gbps)
        for w in self.load.get_warnings():
            logger.warning("  %s", w)

    def get_full_report(self) -> dict:
        return {"communication": self.comm.get_summary(), "load_balance": self.load.get_summary(),
                "pipeline": self.bubble.get_summary(),
                "steps": [s.__dict__ for s in self.history[-10:]]}

    def reset(self) -> None:
        self.comm.reset()
        self.load.reset()
        self.bubble.reset()
        self.history.clear()
