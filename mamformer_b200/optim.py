"""Mixed-precision AdamW over flat buffers, parameter groups and the LR schedule.

Reference behaviour kept (``scripts/train.py:134-164, 255-277``):

* AdamW, betas (0.9, 0.95), eps 1e-8, weight decay 0.1 except for parameters whose name
  contains ``norm``, ``bias``, ``gate``, ``alpha``, ``lambda_log`` or ``A_log`` (GRPO also
  exempts ``comm_strength``).  ``gate`` also matches every ``gate_proj``, so those get no decay,
  exactly as in the reference;
* LinearLR warm-up from 0.01x, then cosine decay to ``min_lr_ratio`` x peak, stepped once
  per optimizer step; gradient clipping at 1.0.

B200 design:

* model matrices live in flat bf16 buffers (parameters are views into them); fp32 master
  weights, fp32 gradients and the two moments live in flat fp32 buffers, segmented by
  (master kind, weight decay, data-parallel reduction) - one fused kernel launch per segment
  updates master, moments and the bf16 copy in a single pass;
* every gradient is added into the fp32 gradient buffer by a post-accumulate hook
  (micro-batch accumulation in fp32) and the autograd copy is released;
* the gradient norm is reduced on the device and the clip factor is read by the update
  kernel from device memory: no host synchronisation in ``step``;
* data parallelism: replicated gradient segments are summed over the dense data-parallel group
  (every rank that holds the same non-expert weights), expert-parallel segments over the
  expert data-parallel group (ranks that hold the same expert shard; each owner already holds
  the sum over its EP group's tokens).  The sums run as bucketed NCCL all-reduces launched from
  the gradient hooks of the last micro-batch, so they overlap the rest of the backward pass;
  buckets are launched in one fixed order on every rank (a bucket waits for its predecessors),
  and whatever did not become ready during the backward is launched by ``step``.
  ``dp_transport="p2p"`` replaces NCCL on this path: the gradient segments are allocated in
  symmetric memory and each bucket is summed by the NVLink kernels of ``csrc/dp_grad.cu``
  (bounded barrier, reduce-scatter by P2P loads in fixed rank order, all-gather; or, with
  ``MAMF_DP_NVLS=1`` and a multicast object, one switch-side ``multimem`` reduction and
  multicast store) on a side stream that starts when the bucket's last gradient is in;
* the squared gradient norm is summed without float atomics (fixed-order partials), so every
  replica computes the same clip factor and replicas stay bitwise equal.
"""

from __future__ import annotations

import math
import os
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist
from torch.optim.lr_scheduler import CosineAnnealingLR, LinearLR, SequentialLR

NO_DECAY_KEYS = ("norm", "bias", "gate", "alpha", "lambda_log", "A_log")
_ALIGN = 64   # elements; keeps every parameter 256-byte aligned in fp32


def is_no_decay(name: str, extra: Tuple[str, ...] = ()) -> bool:
    return any(k in name for k in NO_DECAY_KEYS + tuple(extra))


def param_groups(model: torch.nn.Module, weight_decay: float = 0.1,
                 extra_no_decay: Tuple[str, ...] = ()) -> List[dict]:
    decay, no_decay = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        (no_decay if is_no_decay(name, extra_no_decay) else decay).append(p)
    return [{"params": decay, "weight_decay": weight_decay},
            {"params": no_decay, "weight_decay": 0.0}]


def create_lr_scheduler(optimizer, warmup_steps: int = 2000, max_steps: int = 100000,
                        learning_rate: float = 3e-4, min_lr_ratio: float = 0.1):
    warmup_steps = max(1, int(warmup_steps))
    warm = LinearLR(optimizer, start_factor=0.01, end_factor=1.0, total_iters=warmup_steps)
    cos = CosineAnnealingLR(optimizer, T_max=max(1, max_steps - warmup_steps),
                            eta_min=learning_rate * min_lr_ratio)
    return SequentialLR(optimizer, schedulers=[warm, cos], milestones=[warmup_steps])


def _native():
    from mamformer_b200.ops._ext import ext
    return ext()


class _Segment:
    """One flat run of parameters sharing (master kind, decay, dp reduction).

    With ``shard_group`` (ZeRO-1) the fp32 master weights and both moments cover only this
    rank's 1/n slice [lo, hi) of the segment; gradients stay full (micro-batch accumulation),
    the update runs on the slice and the updated weights are all-gathered back into the flat
    parameter buffer."""

    def __init__(self, params: List[torch.nn.Parameter], wd: float, dp_reduce: bool, device,
                 world: int, shard_group=None, symm_group=None):
        self.params = params
        self.wd = wd
        self.dp_reduce = dp_reduce
        self.low = params[0].dtype != torch.float32
        self.offsets = []
        off = 0
        for p in params:
            self.offsets.append(off)
            off += (p.numel() + _ALIGN - 1) // _ALIGN * _ALIGN
        sw = _group_size(shard_group)
        self.shard_group = shard_group if sw > 1 else None
        pad = _ALIGN * math.lcm(max(1, world), sw)
        self.numel = max(pad, (off + pad - 1) // pad * pad)
        sr = dist.get_rank(shard_group) if self.shard_group is not None else 0
        self.lo, self.hi = sr * self.numel // sw, (sr + 1) * self.numel // sw
        f32 = dict(device=device, dtype=torch.float32)
        n_local = self.hi - self.lo
        # with `symm_group` the gradient buffer lives in symmetric memory (every rank of the group
        # maps it), so the data-parallel reduction can run as this repository's NVLink kernels
        self.symm = None
        if symm_group is not None:
            import torch.distributed._symmetric_memory as symm_mem
            self.grad = symm_mem.empty(self.numel, dtype=torch.float32, device=device)
            self.grad.zero_()
            self.symm = symm_mem.rendezvous(self.grad, symm_group)
            self.symm_epoch = 0
        else:
            self.grad = torch.zeros(self.numel, **f32)
        self.m = torch.zeros(n_local, **f32)
        self.v = torch.zeros(n_local, **f32)
        self.low_flat = torch.zeros(self.numel, device=device, dtype=params[0].dtype) if self.low else None
        # full fp32 values (the parameters of an fp32 segment view this buffer)
        full = torch.zeros(self.numel, **f32)
        with torch.no_grad():
            for p, o in zip(params, self.offsets):
                n = p.numel()
                full[o:o + n].copy_(p.detach().reshape(-1).float())
                if self.low:
                    self.low_flat[o:o + n].copy_(p.detach().reshape(-1))
                    p.data = self.low_flat[o:o + n].view_as(p)
                else:
                    p.data = full[o:o + n].view_as(p)
                p.main_grad = self.grad[o:o + n].view_as(p)
        if self.low:
            self.master = full[self.lo:self.hi].clone() if self.shard_group is not None else full
            self.full32 = None
        else:
            self.full32 = full
            self.master = full[self.lo:self.hi]

    @property
    def sharded(self) -> bool:
        return self.shard_group is not None

    def gather_params(self) -> None:
        """All-gather the updated slice into the full flat parameter buffer."""
        if not self.sharded:
            return
        buf = self.low_flat if self.low else self.full32
        dist.all_gather_into_tensor(buf, buf[self.lo:self.hi].clone(), group=self.shard_group)

    def full_master(self) -> torch.Tensor:
        """fp32 values of the whole segment (collective over the shard group when sharded)."""
        if not self.sharded:
            return self.master if self.low else self.full32
        if not self.low:
            return self.full32
        out = torch.empty(self.numel, device=self.master.device, dtype=torch.float32)
        dist.all_gather_into_tensor(out, self.master, group=self.shard_group)
        return out


def _group_size(g) -> int:
    return dist.get_world_size(g) if (g is not None and dist.is_available() and dist.is_initialized()) else 1


class _Bucket:
    __slots__ = ("seg", "lo", "hi", "params", "group", "pending", "work")

    def __init__(self, seg, lo, hi, params, group):
        self.seg, self.lo, self.hi, self.params, self.group = seg, lo, hi, params, group
        self.pending = 0
        self.work = None


class GradReducer:
    """Bucketed all-reduce of the fp32 gradient segments, overlapped with the backward pass.

    ``arm()`` before the backward of the last micro-batch; gradient hooks then count each
    bucket down and launch ready buckets (in the fixed launch order) as async all-reduces;
    ``finish()`` launches the rest and waits."""

    def __init__(self, segments, dense_group, expert_group, bucket_mb: float = 64.0, order=None):
        self.buckets: List[_Bucket] = []
        cap = max(1, int(bucket_mb * (1 << 20) / 4))
        pidx = order or {}
        for _, seg in segments:
            if not seg.dp_reduce:
                continue
            group = expert_group if seg.expert else dense_group
            hi = lo = seg.numel
            cur = []
            for p, o in reversed(list(zip(seg.params, seg.offsets))):   # backward order ~ reverse
                if cur and hi - o > cap:
                    self.buckets.append(_Bucket(seg, lo, hi, cur, group))
                    hi, cur = lo, []
                lo = o
                cur.append(p)
            if cur:
                self.buckets.append(_Bucket(seg, 0, hi, cur, group))
        # launch order: the bucket whose earliest parameter comes last in the model first
        self.buckets.sort(key=lambda b: -min(pidx.get(id(p), 0) for p in b.params))
        self._of = {}
        for i, b in enumerate(self.buckets):
            for p in b.params:
                self._of[id(p)] = i
        self.armed = False
        self._next = 0
        self._side = None

    def arm(self) -> None:
        self.armed = True
        self._next = 0
        for b in self.buckets:
            b.pending = len(b.params)
            b.work = None

    def ready(self, p) -> None:
        if not self.armed:
            return
        i = self._of.get(id(p))
        if i is None:
            return
        b = self.buckets[i]
        if b.pending > 0:
            b.pending -= 1
        self._launch_ready()

    def _launch(self, b: _Bucket) -> None:
        from mamformer_b200.utils.nvtx import rng
        with rng(f"dp.bucket[{b.lo}:{b.hi}]"):
            if b.seg.symm is not None:
                self._launch_p2p(b)
            elif b.seg.sharded:
                b.work = _reduce_to_owners(b.seg, b.lo, b.hi, b.group)
            else:
                b.work = dist.all_reduce(b.seg.grad[b.lo:b.hi], group=b.group, async_op=True)

    def _launch_p2p(self, b: _Bucket) -> None:
        """Sum the bucket over the group with the NVLink kernels on a side stream: bounded barrier,
        reduce-scatter (P2P loads) or switch reduction (NVLS multimem), barrier, all-gather,
        barrier.  The side stream starts after the bucket's last accumulation on this stream."""
        from mamformer_b200.ops._ext import require_native
        C = require_native()
        seg, h = b.seg, b.seg.symm
        cur = torch.cuda.current_stream()
        if self._side is None:
            self._side = torch.cuda.Stream(device=seg.grad.device)
        ready = torch.cuda.Event()
        ready.record(cur)
        self._side.wait_event(ready)
        P, me = h.world_size, h.rank
        pads = h.signal_pad_ptrs

        def barrier():
            seg.symm_epoch += 1
            C.ep_barrier(pads, me, seg.symm_epoch, _DP_SLOT0)

        with torch.cuda.stream(self._side):
            if _DP_IMPL == "pull":
                dp_pull_allreduce(h, seg.grad, b.lo, b.hi, barrier, self.__dict__.setdefault("_tmp", {}))
                done = torch.cuda.Event()
                done.record(self._side)
                b.work = _StreamWork(done)
                return
            barrier()                                   # every rank finished accumulating the bucket
            mc = int(getattr(h, "multicast_ptr", 0) or 0) if _use_nvls() else 0
            if mc:
                C.dp_allreduce_nvls(mc, P, me, b.lo, b.hi, 1.0, False)
                barrier()                               # every slice stored into every copy
            else:
                C.dp_reduce_scatter(h.buffer_ptrs, me, b.lo, b.hi, 1.0, False)
                barrier()                               # every slice reduced
                C.dp_all_gather(h.buffer_ptrs, me, b.lo, b.hi)
                barrier()                               # every peer done reading this rank's slice
            done = torch.cuda.Event()
            done.record(self._side)
        b.work = _StreamWork(done)

    def _launch_ready(self) -> None:
        while self._next < len(self.buckets) and self.buckets[self._next].pending == 0:
            self._launch(self.buckets[self._next])
            self._next += 1

    def finish(self) -> None:
        while self._next < len(self.buckets):
            self._launch(self.buckets[self._next])
            self._next += 1
        for b in self.buckets:
            if b.work is not None:
                b.work.wait()
                b.work = None
        self.armed = False


_DP_SLOT0 = 640   # signal-pad words used by the data-parallel barrier (after the EP / TP ones)
_DP_IMPL = "pull"     # peer-memory all-reduce: "pull" (copy engines) or "kernel" (SM P2P loads)


def dp_slice_bounds(lo: int, hi: int, P: int, q: int):
    """Rank q's slice of bucket [lo, hi): whole 16-byte words, as the native kernels use."""
    sl = ((hi - lo + P - 1) // P + 3) // 4 * 4
    s0 = min(hi, lo + q * sl)
    return s0, min(hi, s0 + sl)


def dp_pull_allreduce(h, buf: torch.Tensor, lo: int, hi: int, barrier, tmp: dict) -> None:
    """Sum buf[lo:hi] over the symmetric-memory group on the current stream with the copy
    engines: barrier; the owner of each slice pulls the peers' copies of it into local buffers
    and adds them in place (only the owner computes a slice, so every replica ends with the
    same bits); barrier; every rank pulls the other owners' reduced slices into its own buffer;
    barrier.  Each remote float crosses NVLink once per phase."""
    P, r = h.world_size, h.rank
    s0, s1 = dp_slice_bounds(lo, hi, P, r)
    barrier()                                       # every rank finished accumulating the bucket
    if s1 > s0:
        n = s1 - s0
        for i in range(1, P):
            q = (r + i) % P
            t = tmp.get(i)
            if t is None or t.numel() < n:
                t = torch.empty(n, device=buf.device, dtype=torch.float32)
                tmp[i] = t
            t = t[:n]
            t.copy_(h.get_buffer(q, (n,), torch.float32, s0), non_blocking=True)
            buf[s0:s1].add_(t)
    barrier()                                       # every slice reduced by its owner
    for i in range(1, P):
        q = (r + i) % P
        q0, q1 = dp_slice_bounds(lo, hi, P, q)
        if q1 > q0:
            buf[q0:q1].copy_(h.get_buffer(q, (q1 - q0,), torch.float32, q0), non_blocking=True)
    barrier()                                       # every peer done reading this rank's slice


def _use_nvls() -> bool:
    """NVSwitch multicast reduction for the peer-memory gradient all-reduce (opt-in)."""
    return os.environ.get("MAMF_DP_NVLS", "0") == "1"


class _Works:
    """Several collective handles behind one ``wait()``."""

    def __init__(self, works):
        self.works = works

    def wait(self) -> None:
        for w in self.works:
            w.wait()


def _reduce_to_owners(seg, lo: int, hi: int, group) -> _Works:
    """ZeRO-1 bucket reduction: a rank's optimizer reads only its own slice [seg.lo, seg.hi) of
    the summed gradient, so the bucket [lo, hi) is summed onto the owner of each slice it
    overlaps (``dist.reduce``, about half the bytes an all-reduce moves).  The other ranks'
    copies of those elements are left partial and are never read."""
    sw = _group_size(group)
    n = seg.numel
    works = []
    for q in range(sw):                       # the same owner order on every rank
        a, z = max(lo, q * n // sw), min(hi, (q + 1) * n // sw)
        if a < z:
            dst = dist.get_global_rank(group, q) if group is not None else q
            works.append(dist.reduce(seg.grad[a:z], dst=dst, group=group, async_op=True))
    return _Works(works)


class _StreamWork:
    """Completion of a side-stream reduction, with the ``wait()`` of a collective handle."""

    def __init__(self, event):
        self.event = event

    def wait(self) -> None:
        torch.cuda.current_stream().wait_event(self.event)


def mark_grad_ready(p: torch.Tensor) -> None:
    """Tell the data-parallel reducer that ``p.main_grad`` is final for this backward (for
    gradients accumulated in place by a kernel instead of through autograd)."""
    red = getattr(p, "_mamf_reducer", None)
    if red is not None:
        red.ready(p)


def _p2p_ok(transport: str, group, device) -> bool:
    """Peer-memory gradient reduction: requested ("p2p"), on CUDA, 2..8 ranks."""
    if transport != "p2p":
        return False
    if torch.device(device).type != "cuda" or group is None:
        return False
    return 2 <= _group_size(group) <= 8


class MixedPrecisionAdamW(torch.optim.Optimizer):
    """``dp_group``: dense data-parallel group (all replicas of the non-expert weights; also
    the 1/world gradient scale).  ``expert_dp_group``: replicas of this rank's expert shard
    (None: none).  ``ep_group``: the expert-parallel group, over which the squared norm of the
    expert shards is summed (None: ``dp_group``, i.e. every rank owns a distinct shard)."""

    def __init__(self, params, lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.1, max_grad_norm: float = 1.0,
                 dp_group: Optional[dist.ProcessGroup] = None, no_dp_reduce=None,
                 expert_dp_group: Optional[dist.ProcessGroup] = None,
                 ep_group: Optional[dist.ProcessGroup] = None, bucket_mb: float = 64.0,
                 param_order=None, zero_stage: int = 0, dp_transport: str = "nccl"):
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self.max_grad_norm = max_grad_norm
        self.dp_group = dp_group
        self.expert_dp_group = expert_dp_group
        self.ep_group = ep_group if ep_group is not None else (dp_group if no_dp_reduce else None)
        self.world = _group_size(dp_group)
        expert_world = _group_size(expert_dp_group)
        skip = set(id(p) for p in (no_dp_reduce or []))
        dev = self.param_groups[0]["params"][0].device
        self.segments: List[Tuple[int, _Segment]] = []
        for gi, g in enumerate(self.param_groups):
            buckets: Dict[tuple, list] = {}
            for p in g["params"]:
                buckets.setdefault((p.dtype, id(p) in skip), []).append(p)
            for (dt, is_exp), ps in buckets.items():
                red = (expert_world > 1) if is_exp else (self.world > 1)
                shard = dp_group if (zero_stage >= 1 and not is_exp and self.world > 1) else None
                grp = expert_dp_group if is_exp else dp_group
                symm_grp = grp if (red and shard is None and _p2p_ok(dp_transport, grp, dev)) else None
                seg = _Segment(ps, g["weight_decay"], red, dev, self.world, shard_group=shard,
                               symm_group=symm_grp)
                seg.expert = is_exp
                self.segments.append((gi, seg))
        self.reducer = GradReducer(self.segments, dp_group, expert_dp_group, bucket_mb, param_order)
        for _, seg in self.segments:
            for p in seg.params:
                p._mamf_reducer = self.reducer
        self._hooks = [p.register_post_accumulate_grad_hook(_accumulate_grad)
                       for _, seg in self.segments for p in seg.params]
        self._sq = torch.zeros(1, device=dev)
        self._scale = torch.ones(1, device=dev)
        self.last_grad_norm = torch.zeros(1, device=dev)
        self._step = 0

    # -- gradients -------------------------------------------------------------------------
    def zero_grad(self, set_to_none: bool = True):
        for _, seg in self.segments:
            seg.grad.zero_()
            for p in seg.params:
                p.grad = None

    def reduce_gradients(self) -> None:
        """Finish the data-parallel gradient sums (launching buckets not launched yet)."""
        self.reducer.finish()

    @torch.no_grad()
    def step(self, closure=None, reduce: bool = True):
        if reduce:
            self.reduce_gradients()
        C = _native()
        self._step += 1
        self._sq.zero_()
        use_native = C is not None and self._sq.is_cuda
        # Both kinds of segment hold sum_r dL_r/dtheta (replicated ones after the all-reduce,
        # expert-parallel ones because dispatch brought every rank's tokens to the owner), so
        # both are scaled by 1/world.  Replicated segments are identical on every rank; the
        # expert-parallel part of the squared norm is summed over ranks.
        sq_ep = torch.zeros_like(self._sq) if _group_size(self.ep_group) > 1 else None
        sq_sh = torch.zeros_like(self._sq) if any(seg.sharded for _, seg in self.segments) else None
        for _, seg in self.segments:
            acc = sq_ep if (sq_ep is not None and seg.expert) else (sq_sh if seg.sharded else self._sq)
            g = seg.grad[seg.lo:seg.hi] if seg.sharded else seg.grad
            if use_native:
                C.sq_norm_accumulate(g, acc)
            else:
                acc += g.pow(2).sum()
        if sq_ep is not None:
            dist.all_reduce(sq_ep, group=self.ep_group)
            self._sq += sq_ep
        if sq_sh is not None:
            dist.all_reduce(sq_sh, group=self.dp_group)
            self._sq += sq_sh
        if use_native:
            C.clip_scale(self._sq, self._scale, float(self.max_grad_norm or 0.0), 1.0 / self.world,
                         self.last_grad_norm)
        else:
            nrm = self._sq.sqrt() / self.world
            s = 1.0 / self.world
            if self.max_grad_norm and float(nrm) > self.max_grad_norm:
                s *= self.max_grad_norm / (float(nrm) + 1e-6)
            self._scale.fill_(s)
            self.last_grad_norm.copy_(nrm)
        for gi, seg in self.segments:
            grp = self.param_groups[gi]
            b1, b2 = grp["betas"]
            g = seg.grad[seg.lo:seg.hi] if seg.sharded else seg.grad
            low = seg.low_flat[seg.lo:seg.hi] if (seg.low and seg.sharded) else seg.low_flat
            if use_native:
                C.adamw_step(seg.master, g, seg.m, seg.v, low, float(grp["lr"]), b1, b2,
                             grp["eps"], seg.wd, self._step, self._scale)
            else:
                _adamw_torch(seg.master, g, seg.m, seg.v, low, grp["lr"], b1, b2, grp["eps"], seg.wd,
                             self._step, self._scale)
            seg.gather_params()
        return None

    def grad_norm(self) -> torch.Tensor:
        return self.last_grad_norm

    def master_views(self) -> Dict[int, torch.Tensor]:
        """param id -> fp32 weight (collective over the shard groups when ZeRO is on)."""
        out = {}
        for _, seg in self.segments:
            full = seg.full_master()
            for p, o in zip(seg.params, seg.offsets):
                out[id(p)] = full[o:o + p.numel()].view(p.shape)
        return out

    # -- checkpointing ---------------------------------------------------------------------
    def state_dict(self):
        return {"step": self._step,
                "segments": [{"master": s.master.cpu(), "m": s.m.cpu(), "v": s.v.cpu(),
                              "shard": (s.lo, s.hi, s.numel)} for _, s in self.segments],
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups]}

    @property
    def sharded(self) -> bool:
        return any(seg.sharded for _, seg in self.segments)

    def load_state_dict(self, state):
        segs = state["segments"]
        for (_, seg), st in zip(self.segments, segs):
            if tuple(st.get("shard", (0, seg.numel, seg.numel))) != (seg.lo, seg.hi, seg.numel):
                raise ValueError("optimizer state was saved with another sharding layout")
        self._step = int(state["step"])
        for (_, seg), st in zip(self.segments, segs):
            seg.master.copy_(st["master"])
            seg.m.copy_(st["m"])
            seg.v.copy_(st["v"])
            if seg.low:
                (seg.low_flat[seg.lo:seg.hi] if seg.sharded else seg.low_flat).copy_(seg.master)
            seg.gather_params()
        for g, sg in zip(self.param_groups, state["param_groups"]):
            g.update({k: v for k, v in sg.items() if k in ("lr", "betas", "eps", "weight_decay", "initial_lr")})


def _accumulate_grad(p: torch.Tensor) -> None:
    g = p.grad
    if g is None:
        return
    C = _native()
    if C is not None and g.is_cuda:
        C.grad_accumulate(p.main_grad, g.contiguous())
    else:
        p.main_grad.add_(g.float())
    p.grad = None
    red = getattr(p, "_mamf_reducer", None)
    if red is not None and red.armed:
        red.ready(p)


def _adamw_torch(master, grad, m, v, low, lr, b1, b2, eps, wd, step, scale):
    g = grad * scale
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    bc1 = 1 - b1 ** step
    bc2 = 1 - b2 ** step
    master.mul_(1 - lr * wd)
    master.addcdiv_(m, (v.sqrt() / math.sqrt(bc2)).add_(eps), value=-lr / bc1)
    if low is not None:
        low.copy_(master)
