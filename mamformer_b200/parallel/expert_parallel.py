"""Expert parallelism: routed experts sharded over the EP group, tokens moved to their owners.

Reference: ``mamformer/parallelism/expert_parallel.py`` (``ExpertParallelGroup`` 48-176,
``expert_dispatch`` 178-253, ``expert_combine`` 255-340, ``EPMoE`` 342-543, ``shard_experts_ep``
545-575).  The reference's ``shard_experts_ep`` only warns (retroactive sharding is not
implemented) and its ``EPMoE`` sends every top-k slot through its own padded all-to-all.  Here
``shard_experts_ep`` really shards a built model: every ``DeepSeekMoE`` keeps the experts
``[r*E/P, (r+1)*E/P)`` of its stacked weights and gets an :class:`EPEngine` that moves all k
slots of all tokens at once.  Two transports:

* ``"p2p"`` (CUDA, EP group inside one NVSwitch domain): symmetric-memory stages and the kernels
  of ``csrc/moe_rows.cu``.  Per layer and direction the sender writes its rows once, already
  sorted by expert, into its own stage; after a signal-pad barrier each owner pulls its runs
  straight into its 64-aligned, expert-grouped GEMM operand (no all-to-all buffer, no local
  re-permutation), the down-projection GEMM writes its output into the owner's stage, and each
  sender's combine kernel reads its k rows per token from the owners over NVLink and sums them
  with the gates in fp32.  The backward is the mirror image (gate-scaled gradient rows pulled
  by the owners, fp32 input-gradient rows gathered and summed by the senders).
* ``"nccl"`` (any device, also gloo on CPU): one variable-size ``all_to_all_single`` per
  direction (autograd-aware), then the same grouped expert computation.

The per-expert token counts are exchanged once per layer with one small collective and read on
the host (the sizes of the owner's buffers depend on them).

Gradient bookkeeping: routed-expert weights are tagged ``_mamf_expert``; the optimizer reduces
them over the ``expert_dp`` group (replicas of the same shard) instead of ``dense_dp``.
"""

from __future__ import annotations

import os
from typing import List, Optional, Tuple

import numpy as np
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
    """Symmetric-memory stages of one EP group (grown collectively, never shrunk)."""

    def __init__(self, group, device, d):
        self.group = group
        self.device = device
        self.d = d
        self.rows_x = 0
        self.rows_y = 0
        self.x = self.y = self.dx = None
        self.hx = self.hy = self.hdx = None

    def _alloc(self, rows, dtype):
        import torch.distributed._symmetric_memory as symm
        t = symm.empty((max(rows, 1), self.d), dtype=dtype, device=self.device)
        return t, symm.rendezvous(t, self.group)

    def ensure(self, rows_x: int, rows_y: int) -> None:
        """Every rank calls this with the same sizes (derived from the all-gathered counts)."""
        if rows_x <= self.rows_x and rows_y <= self.rows_y:
            return
        torch.cuda.current_stream(self.device).synchronize()   # old stages may still be read
        if rows_x > self.rows_x:
            self.rows_x = (rows_x * 5 // 4 + ALIGN - 1) // ALIGN * ALIGN
            self.x, self.hx = self._alloc(self.rows_x, torch.bfloat16)
        if rows_y > self.rows_y:
            self.rows_y = (rows_y * 5 // 4 + ALIGN - 1) // ALIGN * ALIGN
            self.y, self.hy = self._alloc(self.rows_y, torch.bfloat16)
            self.dx, self.hdx = self._alloc(self.rows_y, torch.float32)


class EPEngine:
    """Installed as ``DeepSeekMoE.ep_engine`` by :func:`shard_experts_ep`."""

    def __init__(self, ep_group: ExpertParallelGroup, dense_dp_group=None, dp_factor: Optional[int] = None,
                 backend: str = "auto"):
        self.ep = ep_group
        self.dense_dp_group = dense_dp_group if dense_dp_group is not None else ep_group.group
        if dp_factor is None:
            dp_factor = dist.get_world_size(self.dense_dp_group) if self.dense_dp_group is not None else ep_group.ep_size
        self.dp_factor = int(dp_factor)
        self.backend = os.environ.get("MAMF_EP_BACKEND", backend)
        self._stage = None
        self._epoch = 0

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
        if self._use_p2p(xf) and moe_ops.supported(xf, m.routed_gate_proj):
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
        C.ep_barrier(self._stage.hx.signal_pad_ptrs, self.ep.ep_rank, self._epoch, _SIGNAL_SLOT0)

    def plan_p2p(self, m, idx: torch.Tensor, d: int):
        """Exchange per-expert counts (one all-gather + one host read) and derive: this rank's
        slot positions in the owners' grouped buffers, its pull runs as an owner, its segment
        table, and the stage sizes (identical on every rank)."""
        E, El, P, me = m.n_routed_experts, m.n_local_experts, self.ep.ep_size, self.ep.ep_rank
        dev = idx.device
        flat = idx.reshape(-1).long()
        Q = flat.numel()
        order = torch.argsort(flat, stable=True)
        send_e = torch.bincount(flat, minlength=E)
        allc = torch.empty(P, E, dtype=send_e.dtype, device=dev)
        dist.all_gather_into_tensor(allc, send_e, group=self.ep.group)
        Ch = allc.cpu().numpy().astype(np.int64)                      # (P, E)
        tot = Ch.sum(0)                                                # per expert, all sources
        loc = tot.reshape(P, El)
        pad = (loc + ALIGN - 1) // ALIGN * ALIGN
        seg_all = np.zeros((P, El + 1), np.int64)
        seg_all[:, 1:] = np.cumsum(pad, 1)                             # owner r's segments
        src_start = np.zeros((P, E), np.int64)
        src_start[:, 1:] = np.cumsum(Ch, 1)[:, :-1]                    # sorted position per source
        before = np.cumsum(Ch, 0) - Ch                                 # rows of sources s' < s
        owner_e = np.arange(E) // El
        base = seg_all[owner_e, np.arange(E) % El] + before[me]
        runs = []
        for le in range(El):
            e = me * El + le
            for s in range(P):
                n = int(Ch[s, e])
                if n:
                    runs.append((int(seg_all[me, le] + before[s, e]), s, int(src_start[s, e]), n))
        rows_me = int(seg_all[me, -1])
        rows_y = int(seg_all[:, -1].max())
        rows_x = int(Ch.sum(1).max())
        tabs = torch.from_numpy(np.stack([base, src_start[me]])).to(dev)
        e_sorted = flat[order]
        q = torch.arange(Q, device=dev)
        pos_sorted = tabs[0][e_sorted] + q - tabs[1][e_sorted]
        pos = torch.empty_like(pos_sorted)
        pos[order] = pos_sorted
        inv = torch.empty_like(order)
        inv[order] = q
        owner = (flat // El).to(torch.int32)
        seg = torch.from_numpy(seg_all[me]).to(dev, torch.int32)
        runs_t = torch.tensor(runs if runs else [[0, 0, 0, 0]], dtype=torch.long, device=dev)
        max_len = max((r[3] for r in runs), default=0)
        if self._stage is None:
            self._stage = _SymStage(self.ep.group, dev, d)
        self._stage.ensure(max(rows_x, Q), rows_y)
        return dict(pos=pos, inv=inv, owner=owner, seg=seg, runs=runs_t, n_runs=len(runs), max_len=max_len,
                    rows=rows_me)


class _P2PRouted(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gates, idx, w_gate, w_up, w_down, eng: EPEngine, m):
        from mamformer_b200.ops import gemm, moe as moe_ops
        from mamformer_b200.ops.native import _C
        T, d = x.shape
        k = idx.shape[1]
        pl = eng.plan_p2p(m, idx, d)
        st = eng._stage
        Q = T * k
        tile_off = gemm.tile_offsets(pl["seg"])
        # dispatch: sorted rows into my stage, owners pull their runs
        _C.moe_scatter_rows(st.x, pl["inv"], x, k)
        eng.barrier(_C)
        xp = torch.zeros(pl["rows"], d, device=x.device, dtype=x.dtype)
        if pl["n_runs"]:
            _C.ep_pull_runs(xp, st.hx.buffer_ptrs, d, pl["runs"][: pl["n_runs"]], pl["max_len"])
        eng.barrier(_C)
        hg, hu, act, yp = moe_ops.mlp_forward(xp, pl["seg"], tile_off, w_gate, w_up, w_down,
                                              y_out=st.y[: pl["rows"]])
        eng.barrier(_C)
        g32 = gates.float().reshape(-1).contiguous()
        out = torch.empty(T, d, device=x.device, dtype=x.dtype)
        y_rows = torch.empty(Q, d, device=x.device, dtype=x.dtype)
        _C.moe_combine(out, st.hy.buffer_ptrs, d, torch.bfloat16, pl["owner"], pl["pos"], g32, k, y_rows)
        eng.barrier(_C)
        ctx.save_for_backward(xp, hg, hu, act, y_rows, pl["pos"], pl["inv"], pl["owner"], pl["seg"], tile_off,
                              pl["runs"], g32, w_gate, w_up, w_down)
        ctx.meta = (T, k, d, pl["n_runs"], pl["max_len"], pl["rows"], gates.dtype)
        ctx.eng = eng
        return out

    @staticmethod
    def backward(ctx, dout):
        from mamformer_b200.ops import moe as moe_ops
        from mamformer_b200.ops.native import _C
        (xp, hg, hu, act, y_rows, pos, inv, owner, seg, tile_off, runs, g32, w_gate, w_up,
         w_down) = ctx.saved_tensors
        T, k, d, n_runs, max_len, rows, gdt = ctx.meta
        eng = ctx.eng
        st = eng._stage
        dout = dout.to(xp.dtype).contiguous()
        dg = torch.empty(T * k, device=xp.device, dtype=torch.float32)
        _C.moe_combine_bwd(dout, y_rows, None, g32, dg, st.x, inv, k)
        eng.barrier(_C)
        dyp = torch.zeros(rows, d, device=xp.device, dtype=xp.dtype)
        if n_runs:
            _C.ep_pull_runs(dyp, st.hx.buffer_ptrs, d, runs[:n_runs], max_len)
        eng.barrier(_C)
        dxp, (gw_g, gw_u, gw_d) = moe_ops.mlp_backward(dyp, xp, hg, hu, act, seg, tile_off, w_gate, w_up, w_down,
                                                      dx_out=st.dx[:rows])
        eng.barrier(_C)
        dx = torch.empty(T, d, device=xp.device, dtype=xp.dtype)
        _C.moe_combine(dx, st.hdx.buffer_ptrs, d, torch.float32, owner, pos, None, k, None)
        eng.barrier(_C)
        return dx, dg.view(T, k).to(gdt), None, gw_g, gw_u, gw_d, None, None


# ---------------------------------------------------------------------------------------------
def _moe_modules(model: nn.Module):
    from mamformer_b200.models.moe import DeepSeekMoE
    return [mod for mod in model.modules() if isinstance(mod, DeepSeekMoE)]


def shard_experts_ep(model: nn.Module, ep_group: ExpertParallelGroup, dp_factor: Optional[int] = None,
                     dense_dp_group=None, backend: str = "auto") -> nn.Module:
    """Keep this rank's slice of every MoE layer's routed experts and install the EP engine.

    Must run before the optimizer is built (the optimizer's flat buffers take the sliced
    parameters).  The number of routed experts must be divisible by the EP size."""
    if ep_group.ep_size <= 1:
        return model
    eng = EPEngine(ep_group, dense_dp_group=dense_dp_group, dp_factor=dp_factor, backend=backend)
    for mod in _moe_modules(model):
        E = mod.n_routed_experts
        if E % ep_group.ep_size:
            raise ValueError(f"{E} routed experts do not split evenly over EP={ep_group.ep_size}")
        s, e = ep_group.get_expert_range(E)
        for name in ("routed_gate_proj", "routed_up_proj", "routed_down_proj"):
            w = getattr(mod, name)
            p = nn.Parameter(w.detach()[s:e].clone(), requires_grad=w.requires_grad)
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
