"""Expert parallelism: routed experts sharded over the EP group, tokens moved to their owners.

Reference: ``mamformer/parallelism/expert_parallel.py`` (``ExpertParallelGroup`` 48-176,
``expert_dispatch`` 178-253, ``expert_combine`` 255-340, ``EPMoE`` 342-543, ``shard_experts_ep``
545-575).  The reference's ``shard_experts_ep`` only warns (retroactive sharding is not
implemented) and its ``EPMoE`` sends every top-k slot through its own padded all-to-all.  Here
``shard_experts_ep`` really shards a built model: every ``DeepSeekMoE`` keeps the experts
``[r*E/P, (r+1)*E/P)`` of its stacked weights and gets an :class:`EPEngine` that moves all k
slots of all tokens at once.  Two transports:

* ``"p2p"`` (CUDA, EP group inside one NVSwitch domain): symmetric-memory stages and the kernels
  of ``csrc/moe_rows.cu``, planned entirely on the device.  Per layer the sender sorts its
  top-k assignments by expert (native counting sort) and writes its rows once, sorted, into its
  own stage; it pushes its per-expert counts into every peer's count matrix with P2P stores,
  and that exchange doubles as the barrier that publishes the stage.  Every rank then lays out
  every owner's 64-aligned expert segments from the same matrix, so it knows where each of its
  rows lands; each owner pulls its rows straight into its expert-grouped GEMM operand (one warp
  per row, pad rows zeroed), the down-projection GEMM writes into the owner's stage, and each
  sender's combine kernel reads its k rows per token from the owners over NVLink and sums them
  with the gates in fp32.  The backward is the mirror image.  The owners' buffers have a fixed
  capacity, so the host never waits inside the forward or backward; see :class:`EPEngine`.
* ``"nccl"`` (any device, also gloo on CPU): one variable-size ``all_to_all_single`` per
  direction (autograd-aware), then the same grouped expert computation.

Gradient bookkeeping: routed-expert weights are tagged ``_mamf_expert``; the optimizer reduces
them over the ``expert_dp`` group (replicas of the same shard) instead of ``dense_dp``.
"""

from __future__ import annotations

import math
import os
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from mamformer_b200 import ops

ALIGN = 64
_SIGNAL_SLOT0 = 256      # first signal-pad word used by the EP barrier


class ExpertParallelGroup:
    """Expert ownership and variable-size all-to-all over one EP process group."""

    def __init__(self, ep_size: Optional[int] = None, ep_rank: Optional[int] = None,
                 group: Optional[dist.ProcessGroup] = None):
        ready = dist.is_available() and dist.is_initialized()
        if ep_size is None:
            ep_size = dist.get_world_size(group) if (ready and group is not None) else 1
        self.ep_size = int(ep_size)
        self.group = group
        if ep_rank is not None:
            self.ep_rank = int(ep_rank)
        elif group is not None and ready:
            self.ep_rank = dist.get_rank(group)
        else:
            self.ep_rank = 0
        self._is_initialized = group is not None and ready

    def get_expert_range(self, n_total_experts: int) -> Tuple[int, int]:
        per = (n_total_experts + self.ep_size - 1) // self.ep_size
        start = self.ep_rank * per
        return start, min(start + per, n_total_experts)

    def get_expert_rank(self, expert_idx: int, n_total_experts: int) -> int:
        per = (n_total_experts + self.ep_size - 1) // self.ep_size
        return expert_idx // per

    def all_to_all(self, tensor: torch.Tensor, split_sizes: List[int]) -> torch.Tensor:
        """Variable-length all-to-all of rows: ``split_sizes[r]`` rows go to rank r; returns the
        rows received from every rank, in rank order (counts exchanged first)."""
        if not self._is_initialized or self.ep_size == 1:
            return tensor
        send = torch.tensor(split_sizes, dtype=torch.long, device=tensor.device)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        out_splits = recv.cpu().tolist()
        return _AllToAll.apply(tensor, out_splits, list(split_sizes), self.group)


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, out_splits, in_splits, group):
        ctx.splits = (out_splits, in_splits)
        ctx.group = group
        out = x.new_empty((sum(out_splits),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), out_splits, in_splits, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out_splits, in_splits = ctx.splits
        gi = g.new_empty((sum(in_splits),) + tuple(g.shape[1:]))
        dist.all_to_all_single(gi, g.contiguous(), in_splits, out_splits, group=ctx.group)
        return gi, None, None, None


def expert_dispatch(x: torch.Tensor, expert_indices: torch.Tensor, n_experts: int,
                    ep_group: ExpertParallelGroup):
    """Send each row of ``x`` to the rank owning ``expert_indices[row]``.

    Returns ``(dispatched_x, sort_order, send_counts)`` like the reference; the received rows are
    ordered by (source rank, expert)."""
    order = torch.argsort(expert_indices.reshape(-1).long(), stable=True)
    owner = expert_indices.reshape(-1).long()[order] // ((n_experts + ep_group.ep_size - 1) // ep_group.ep_size)
    counts = torch.bincount(owner, minlength=ep_group.ep_size)
    out = ep_group.all_to_all(x[order], counts.cpu().tolist())
    return out, order, counts


def expert_combine(expert_outputs: torch.Tensor, sort_order: torch.Tensor, token_counts: torch.Tensor,
                   total_tokens: int, ep_group: ExpertParallelGroup,
                   recv_counts: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Inverse of :func:`expert_dispatch`: return rows to their source and undo the sort."""
    if ep_group._is_initialized and ep_group.ep_size > 1:
        if recv_counts is None:
            recv_counts = torch.empty_like(token_counts)
            dist.all_to_all_single(recv_counts, token_counts, group=ep_group.group)
        back = _AllToAll.apply(expert_outputs, token_counts.cpu().tolist(), recv_counts.cpu().tolist(),
                               ep_group.group)
    else:
        back = expert_outputs
    return back.new_zeros((total_tokens,) + tuple(back.shape[1:])).index_copy(0, sort_order, back)


# ---------------------------------------------------------------------------------------------
class _SymStage:
    """Symmetric-memory buffers of one EP group (grown collectively, never shrunk):

    * ``x``  (Q rows, bf16): this rank's token rows sorted by expert (forward), or its
      gate-scaled output-gradient rows (backward); owners pull from it;
    * ``y``  (capacity rows, bf16): expert outputs of this rank's experts; senders gather from it;
    * ``dx`` (capacity rows, fp32): input-gradient rows of this rank's experts;
    * ``cnt`` (P, E) int32: row s holds sender s's per-expert counts (pushed by s)."""

    def __init__(self, group, device, d, P, E):
        self.group, self.device, self.d, self.P, self.E = group, device, d, P, E
        self.rows_x = self.rows_y = 0
        self.x = self.y = self.dx = None
        self.hx = self.hy = self.hdx = None
        self.cnt, self.hcnt = self._alloc((P, E), torch.int32)

    def _alloc(self, shape, dtype):
        import torch.distributed._symmetric_memory as symm
        t = symm.empty(shape, dtype=dtype, device=self.device)
        return t, symm.rendezvous(t, self.group)

    def ensure(self, rows_x: int, rows_y: int) -> None:
        """Collective: every rank calls this with the same sizes (fixed by T*k and the capacity,
        never by the routing), so it only allocates on first use or after a capacity increase."""
        if rows_x <= self.rows_x and rows_y <= self.rows_y:
            return
        torch.cuda.current_stream(self.device).synchronize()   # old stages may still be read
        if rows_x > self.rows_x:
            self.rows_x = rows_x
            self.x, self.hx = self._alloc((rows_x, self.d), torch.bfloat16)
        if rows_y > self.rows_y:
            self.rows_y = rows_y
            self.y, self.hy = self._alloc((rows_y, self.d), torch.bfloat16)
            self.dx, self.hdx = self._alloc((rows_y, self.d), torch.float32)


class EPEngine:
    """Installed as ``DeepSeekMoE.ep_engine`` by :func:`shard_experts_ep`.

    Peer-memory transport without host round trips: the routing plan (counting sort, count
    exchange, owner layout) is built on the device.  Each owner's expert-grouped buffers have a
    fixed capacity of ``min(P, capacity_factor) * T * k + 64 * E/P`` rows (T tokens per rank);
    a step whose routing needs more rows at some owner sets a device status word, is discarded
    by :meth:`step_overflowed` (read once per optimizer step, while the GPU still runs the last
    backward) and is rerun by the trainer with a larger capacity.  With ``capacity_factor >= P``
    no step can overflow and nothing is checked."""

    def __init__(self, ep_group: ExpertParallelGroup, dense_dp_group=None, dp_factor: Optional[int] = None,
                 backend: str = "auto", capacity_factor: Optional[float] = None):
        self.ep = ep_group
        self.dense_dp_group = dense_dp_group if dense_dp_group is not None else ep_group.group
        if dp_factor is None:
            dp_factor = dist.get_world_size(self.dense_dp_group) if self.dense_dp_group is not None else ep_group.ep_size
        self.dp_factor = int(dp_factor)
        self.backend = os.environ.get("MAMF_EP_BACKEND", backend)
        if capacity_factor is None:
            capacity_factor = float(os.environ.get("MAMF_EP_CAPACITY", "2.0"))
        self.capacity_factor = float(capacity_factor)
        self._stage = None
        self._epoch = 0
        self.status = None            # device int32 [overflow flag, max rows any owner needed]
        self._status_host = None
        self._status_event = None
        self._snapshot = None
        self.overflow_steps = 0
        from mamformer_b200.utils.nvtx import PhaseTimer
        self.timer = PhaseTimer(os.environ.get("MAMF_EP_PROFILE", "0") == "1")

    # -- helpers used by DeepSeekMoE ------------------------------------------------------------
    def global_counts(self, counts: torch.Tensor) -> torch.Tensor:
        """Per-expert token counts summed over every data-parallel replica (same on all ranks,
        so the aux-loss-free biases stay identical)."""
        if self.dense_dp_group is None:
            return counts
        c = counts.clone()
        dist.all_reduce(c, group=self.dense_dp_group)
        return c

    def _use_p2p(self, x: torch.Tensor) -> bool:
        if self.backend == "nccl" or not x.is_cuda or self.ep.ep_size > 8:
            return False
        if self.backend == "p2p":
            return True
        return x.dtype == torch.bfloat16 and x.shape[1] % 64 == 0

    def routed(self, m, xf: torch.Tensor, idx: torch.Tensor, gates: torch.Tensor) -> torch.Tensor:
        from mamformer_b200.ops import moe as moe_ops
        if self._use_p2p(xf) and moe_ops.supported(xf, m.routed_gate_proj) and m.n_routed_experts <= 256:
            return _P2PRouted.apply(xf.contiguous(), gates, idx, m.routed_gate_proj, m.routed_up_proj,
                                    m.routed_down_proj, self, m)
        y = self._exchange_nccl(m, xf, idx)
        T, k = idx.shape
        return (y.view(T, k, -1).float() * gates.float().unsqueeze(-1)).sum(1).to(xf.dtype)

    def expert_outputs(self, m, xf: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        T, k = idx.shape
        return self._exchange_nccl(m, xf, idx).view(T, k, -1)

    def check_error(self) -> None:
        from mamformer_b200.ops._ext import ext
        C = ext()
        if C is not None and torch.cuda.is_available():
            err = int(C.comm_error())
            if err:
                C.comm_clear_error()
                raise RuntimeError(f"expert-parallel barrier timed out waiting for EP rank {err - 100}")
            bad = int(C.plan_error())
            if bad:
                raise RuntimeError("routing plan saw an expert id outside [0, E)")

    # -- capacity and the once-per-step overflow check ------------------------------------------
    def capacity(self, q_rows: int, n_local: int) -> int:
        f = min(float(self.ep.ep_size), self.capacity_factor)
        rows = int(math.ceil(f * q_rows)) + ALIGN * n_local
        return (rows + 127) // 128 * 128

    @property
    def can_overflow(self) -> bool:
        return self.capacity_factor < self.ep.ep_size

    def _ensure_status(self, device) -> None:
        if self.status is None:
            self.status = torch.zeros(2, dtype=torch.int32, device=device)
            self._status_host = torch.zeros(2, dtype=torch.int32).pin_memory()
            self._status_event = torch.cuda.Event()

    def begin_step(self, model: nn.Module) -> None:
        """Start of an optimizer step: clear the status word and keep a copy of the MoE routing
        state (biases, load EMA, counters) so that a discarded step leaves no trace."""
        dev = next(model.parameters()).device
        if not self.can_overflow or dev.type != "cuda":
            return
        self._ensure_status(dev)
        self.status.zero_()
        self._snapshot = [(b, b.detach().clone()) for mod in _moe_modules(model) for b in mod.buffers()]

    def record_status(self) -> None:
        """After the step's last forward: make the status identical on every data-parallel
        replica and start its copy to the host (read by :meth:`step_overflowed`)."""
        if not self.can_overflow or self.status is None:
            return
        if self.dense_dp_group is not None and dist.get_world_size(self.dense_dp_group) > self.ep.ep_size:
            dist.all_reduce(self.status, op=dist.ReduceOp.MAX, group=self.dense_dp_group)
        self._status_host.copy_(self.status, non_blocking=True)
        self._status_event.record()

    def step_overflowed(self) -> bool:
        """True when some owner needed more rows than the capacity in this step.  Then the
        routing state is restored and the capacity raised; the caller reruns the step."""
        if not self.can_overflow or self._status_event is None:
            return False
        self._status_event.synchronize()
        if int(self._status_host[0]) == 0:
            return False
        need = int(self._status_host[1])
        self.overflow_steps += 1
        for buf, saved in self._snapshot or []:
            buf.copy_(saved)
        q_rows = max(1, self._stage.rows_x if self._stage is not None else 1)
        self.capacity_factor = max(self.capacity_factor * 1.5, 1.25 * need / q_rows)
        return True

    # -- nccl / gloo transport -----------------------------------------------------------------
    def _exchange_nccl(self, m, xf, idx):
        """Expert outputs of every slot, in slot order (T*k, d)."""
        T, d = xf.shape
        k = idx.shape[1]
        E, El, P, g = m.n_routed_experts, m.n_local_experts, self.ep.ep_size, self.ep.group
        flat = idx.reshape(-1).long()
        order = torch.argsort(flat, stable=True)
        send_e = torch.bincount(flat, minlength=E)
        recv_e = torch.empty_like(send_e)
        dist.all_to_all_single(recv_e, send_e, group=g)
        both = torch.stack([send_e.view(P, El).sum(1), recv_e.view(P, El).sum(1)]).cpu()
        in_s, out_s = both[0].tolist(), both[1].tolist()
        xs = xf.index_select(0, order // k)
        xr = _AllToAll.apply(xs, out_s, in_s, g)
        le = torch.repeat_interleave(torch.arange(El, device=xf.device).repeat(P), recv_e,
                                     output_size=int(sum(out_s)))
        yr = ops.moe_expert_outputs(xr, le[:, None], m.routed_gate_proj, m.routed_up_proj,
                                    m.routed_down_proj).reshape(-1, d)
        ys = _AllToAll.apply(yr, in_s, out_s, g)
        return ys.new_zeros(ys.shape).index_copy(0, order, ys)

    # -- p2p transport ---------------------------------------------------------------------------
    def barrier(self, C) -> None:
        self._epoch += 1
        C.ep_barrier(self._stage.hcnt.signal_pad_ptrs, self.ep.ep_rank, self._epoch, _SIGNAL_SLOT0)

    def plan_device(self, m, x: torch.Tensor, idx: torch.Tensor):
        """Routing plan on the device (no host synchronisation): sort this rank's assignments
        by expert and write its rows, sorted, into its stage; exchange the counts through peer
        memory (the exchange is also the barrier that publishes the stage); lay out every
        owner's buffer; locate each assignment's row in its owner's buffer."""
        from mamformer_b200.ops.native import _C as C
        T, d = x.shape
        k = idx.shape[1]
        Q = T * k
        E, El, P, me = m.n_routed_experts, m.n_local_experts, self.ep.ep_size, self.ep.ep_rank
        dev = x.device
        flat = idx.reshape(-1).long().contiguous()
        srow, counts, start = C.moe_sort_plan(flat, E, False)
        cap = self.capacity(Q, El)
        if self._stage is None:
            self._stage = _SymStage(self.ep.group, dev, d, P, E)
        st = self._stage
        st.ensure(Q, cap)
        self._ensure_status(dev)
        C.moe_scatter_rows(st.x, srow, x, k)
        self._epoch += 1
        C.ep_exchange_counts(st.hcnt.buffer_ptrs, st.hcnt.signal_pad_ptrs, counts, me, self._epoch, _SIGNAL_SLOT0)
        plan = torch.empty(C.ep_plan_size(P, El), dtype=torch.int32, device=dev)
        C.ep_layout(st.cnt, me, cap, plan, self.status)
        pos = torch.empty(Q, dtype=torch.int64, device=dev)
        owner = torch.empty(Q, dtype=torch.int32, device=dev)
        C.ep_positions(flat, srow, start, plan, P, cap, pos, owner)
        return dict(srow=srow, plan=plan, seg=plan[: El + 1], tile_off=plan[El + 1: 2 * El + 2], pos=pos,
                    owner=owner, cap=cap)


class _P2PRouted(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gates, idx, w_gate, w_up, w_down, eng: EPEngine, m):
        from mamformer_b200.ops import moe as moe_ops
        from mamformer_b200.ops.native import _C
        from mamformer_b200.utils.nvtx import rng
        T, d = x.shape
        k = idx.shape[1]
        P = eng.ep.ep_size
        tm = eng.timer
        tm.mark("begin_fwd")
        with rng("ep.plan_dispatch"):
            pl = eng.plan_device(m, x, idx)
        tm.mark("fwd.plan+exchange")
        st = eng._stage
        cap = pl["cap"]
        # owners pull their rows (already expert-sorted by each sender) into the grouped operand
        xp = torch.empty(cap, d, device=x.device, dtype=x.dtype)
        with rng("ep.pull"):
            _C.ep_pull_rows(xp, st.hx.buffer_ptrs, d, st.rows_x, pl["plan"], P)
            eng.barrier(_C)                              # every stage read: stages reusable
        tm.mark("fwd.pull")
        with rng("ep.expert_gemms"):
            hg, hu, act, yp = moe_ops.mlp_forward(xp, pl["seg"], pl["tile_off"], w_gate, w_up, w_down,
                                                  y_out=st.y[:cap])
        tm.mark("fwd.gemm")
        with rng("ep.combine"):
            eng.barrier(_C)                              # every owner's outputs complete
            g32 = gates.float().reshape(-1).contiguous()
            out = torch.empty(T, d, device=x.device, dtype=x.dtype)
            y_rows = torch.empty(T * k, d, device=x.device, dtype=x.dtype)
            _C.moe_combine(out, st.hy.buffer_ptrs, d, st.rows_y, torch.bfloat16, pl["owner"], pl["pos"], g32, k, y_rows)
            eng.barrier(_C)                              # every output read: y stage reusable
        tm.mark("fwd.combine")
        ctx.save_for_backward(xp, hg, hu, act, y_rows, pl["pos"], pl["srow"], pl["owner"], pl["plan"], g32,
                              w_gate, w_up, w_down)
        ctx.meta = (T, k, d, cap, m.n_local_experts, gates.dtype)
        ctx.eng = eng
        return out

    @staticmethod
    def backward(ctx, dout):
        from mamformer_b200.ops import moe as moe_ops
        from mamformer_b200.ops.native import _C
        from mamformer_b200.utils.nvtx import rng
        (xp, hg, hu, act, y_rows, pos, srow, owner, plan, g32, w_gate, w_up, w_down) = ctx.saved_tensors
        T, k, d, cap, El, gdt = ctx.meta
        eng = ctx.eng
        st = eng._stage
        P = eng.ep.ep_size
        tm = eng.timer
        tm.mark("begin_bwd")
        dout = dout.to(xp.dtype).contiguous()
        dg = torch.empty(T * k, device=xp.device, dtype=torch.float32)
        with rng("ep.bwd_dispatch"):
            # gate-scaled gradient rows, expert-sorted, into this rank's stage; owners pull them
            _C.moe_combine_bwd(dout, y_rows, None, g32, dg, st.x, srow, k)
            eng.barrier(_C)
            dyp = torch.empty(cap, d, device=xp.device, dtype=xp.dtype)
            _C.ep_pull_rows(dyp, st.hx.buffer_ptrs, d, st.rows_x, plan, P)
            eng.barrier(_C)
        tm.mark("bwd.pull")
        seg, tile_off = plan[: El + 1], plan[El + 1: 2 * El + 2]
        with rng("ep.expert_gemms_bwd"):
            dxp, (gw_g, gw_u, gw_d) = moe_ops.mlp_backward(dyp, xp, hg, hu, act, seg, tile_off, w_gate, w_up,
                                                          w_down, dx_out=st.dx[:cap])
        tm.mark("bwd.gemm")
        with rng("ep.bwd_combine"):
            eng.barrier(_C)
            dx = torch.empty(T, d, device=xp.device, dtype=xp.dtype)
            _C.moe_combine(dx, st.hdx.buffer_ptrs, d, st.rows_y, torch.float32, owner, pos, None, k, None)
            eng.barrier(_C)
        tm.mark("bwd.combine")
        return dx, dg.view(T, k).to(gdt), None, gw_g, gw_u, gw_d, None, None


# ---------------------------------------------------------------------------------------------
def _moe_modules(model: nn.Module):
    from mamformer_b200.models.moe import DeepSeekMoE
    return [mod for mod in model.modules() if isinstance(mod, DeepSeekMoE)]


def shard_experts_ep(model: nn.Module, ep_group: ExpertParallelGroup, dp_factor: Optional[int] = None,
                     dense_dp_group=None, backend: str = "auto",
                     capacity_factor: Optional[float] = None) -> nn.Module:
    """Keep this rank's slice of every MoE layer's routed experts and install the EP engine.

    Must run before the optimizer is built (the optimizer's flat buffers take the sliced
    parameters).  The number of routed experts must be divisible by the EP size."""
    if ep_group.ep_size <= 1:
        return model
    eng = EPEngine(ep_group, dense_dp_group=dense_dp_group, dp_factor=dp_factor, backend=backend,
                   capacity_factor=capacity_factor)
    for mod in _moe_modules(model):
        E = mod.n_routed_experts
        if E % ep_group.ep_size:
            raise ValueError(f"{E} routed experts do not split evenly over EP={ep_group.ep_size}")
        s, e = ep_group.get_expert_range(E)
        prebuilt = mod.routed_gate_proj.shape[0] != E            # built as a slice (build_expert_slice)
        if prebuilt and (mod.expert_offset, mod.expert_offset + mod.n_local_experts) != (s, e):
            raise ValueError(f"MoE module holds experts [{mod.expert_offset}, "
                             f"{mod.expert_offset + mod.n_local_experts}) but EP rank owns [{s}, {e})")
        for name in ("routed_gate_proj", "routed_up_proj", "routed_down_proj"):
            w = getattr(mod, name)
            p = w if prebuilt else nn.Parameter(w.detach()[s:e].clone(), requires_grad=w.requires_grad)
            p._mamf_expert = True
            p._mamf_ep_range = (s, e)
            setattr(mod, name, p)
        mod.expert_offset = s
        mod.n_local_experts = e - s
        mod.ep_engine = eng
    model._mamf_ep_engine = eng
    return model


def expert_parameters(model: nn.Module) -> List[nn.Parameter]:
    """Parameters sharded by expert parallelism (reduced over ``expert_dp`` only)."""
    return [p for p in model.parameters() if getattr(p, "_mamf_expert", False)]


class EPMoE(nn.Module):
    """Stand-alone expert-parallel MoE layer (reference ``EPMoE``, ``expert_parallel.py:342``):
    a ``DeepSeekMoE`` holding only this rank's routed experts."""

    def __init__(self, d_model: int, n_shared_experts: int = 2, shared_expert_dim: int = 2304,
                 n_routed_experts: int = 64, top_k: int = 8, routed_expert_dim: int = 576,
                 ep_group: Optional[ExpertParallelGroup] = None, aux_loss_free: bool = True,
                 bias_update_speed: float = 0.001, dropout: float = 0.0, backend: str = "auto"):
        super().__init__()
        from mamformer_b200.models.moe import DeepSeekMoE
        self.ep_group = ep_group or ExpertParallelGroup(ep_size=1)
        self.moe = DeepSeekMoE(d_model, n_shared_experts, shared_expert_dim, n_routed_experts, top_k,
                               routed_expert_dim, aux_loss_free=aux_loss_free,
                               bias_update_speed=bias_update_speed, dropout=dropout)
        shard_experts_ep(self.moe, self.ep_group, backend=backend)
        self.expert_start, self.expert_end = self.ep_group.get_expert_range(n_routed_experts)
        self.n_local_experts = self.expert_end - self.expert_start
        self.n_routed_experts_total = n_routed_experts
        self.top_k = top_k

    def forward(self, x: torch.Tensor):
        out, aux = self.moe(x)
        aux["local_experts"] = self.n_local_experts
        aux["total_experts"] = self.n_routed_experts_total
        return out, aux
