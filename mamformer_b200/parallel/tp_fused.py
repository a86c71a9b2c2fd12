"""Sequence-parallel tensor parallelism with the collectives overlapped with the GEMMs over NVLink.

Activations between TP blocks are sharded by rows (tokens) over the TP group.  A column-parallel
linear needs the full sequence (all-gather -> GEMM); a row-parallel linear produces partial sums
that must be reduced onto the owning rank (GEMM -> reduce-scatter).  Each has two forms:

* "pull" (default): the copy engines move every remote shard / partial once over NVLink from the
  peer's symmetric-memory buffer into local memory on a side stream, while the tensor cores
  multiply local rows; each remote block is multiplied (or summed) as soon as it lands.
* "kernel": one tcgen05 GEMM does both - mode "gathered-A" (the TMA producer reads every rank's
  row shard straight from that rank's symmetric buffer, plain TMA loads of peer memory, no
  multicast, local shard first) and mode "scattered-D" (the epilogue stores each tile of shard r
  into rank r's staging slot, followed by a local sum of the P slots).  Measured slower on 2
  B200s: the producer re-reads each remote tile once per output n-tile.

A bounded signal-pad barrier (the expert-parallel barrier kernel) orders producers and consumers;
nothing waits on the host.

Reference: ``mamformer/parallelism/tensor_parallel.py`` (``_tp_all_gather`` 90-103,
``_tp_reduce_scatter`` 105-121 - defined there but unused; ``ColumnParallelLinear`` 136-190,
``RowParallelLinear`` 192-250).  Backward: the column layer's input gradient is a GEMM ->
reduce-scatter, the row layer's input gradient an all-gather -> GEMM (the same two fused modes);
weight gradients use the gathered operand (pulled over NVLink into a local buffer) and
accumulate into the optimizer's fp32 buffer in the GEMM epilogue.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from mamformer_b200.utils.nvtx import ranged

_SLOT0 = 320      # signal-pad words used by this module's barrier (after the expert-parallel ones)


class _Workspace:
    """Per-group symmetric buffers: `gather` (rows x K, this rank's shard) and `stage`
    (P x rows x N, partial sums written by the peers); grown collectively."""

    def __init__(self, group):
        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.gather = self.stage = None
        self.hg = self.hs = None
        self.n_gather = self.n_stage = 0
        self.epoch = 0

    def _alloc(self, numel, device):
        import torch.distributed._symmetric_memory as symm
        t = symm.empty(numel, dtype=torch.bfloat16, device=device)
        return t, symm.rendezvous(t, self.group)

    def ensure(self, n_gather: int, n_stage: int, device) -> None:
        if n_gather > self.n_gather or n_stage > self.n_stage:
            torch.cuda.current_stream(device).synchronize()
        if n_gather > self.n_gather:
            self.n_gather = (n_gather * 5 // 4 + 63) // 64 * 64
            self.gather, self.hg = self._alloc(self.n_gather, device)
        if n_stage > self.n_stage:
            self.n_stage = (n_stage * 5 // 4 + 63) // 64 * 64
            self.stage, self.hs = self._alloc(self.n_stage, device)

    def barrier(self, C) -> None:
        self.epoch += 1
        C.ep_barrier(self.hg.signal_pad_ptrs, self.rank, self.epoch, _SLOT0)

    def side_stream(self, device):
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=device)
        return self._side

    def pull_buffer(self, i: int, rows: int, K: int, device) -> torch.Tensor:
        """Local landing buffer i for a pulled peer shard (grown on demand, kept across calls)."""
        bufs = self.__dict__.setdefault("_pull", {})
        b = bufs.get(i)
        if b is None or b.numel() < rows * K:
            b = torch.empty(rows * K, device=device, dtype=torch.bfloat16)
            bufs[i] = b
        return b[: rows * K].view(rows, K)


_WS = {}


def _ws(group) -> _Workspace:
    key = id(group)
    if key not in _WS:
        _WS[key] = _Workspace(group)
    return _WS[key]


def _C():
    from mamformer_b200.ops._ext import require_native
    return require_native()


# all-gather -> GEMM implementation: "pull" (default) or "kernel"
_AG_IMPL = "pull"


@ranged("tp.ag_gemm")
def ag_gemm(x_local: torch.Tensor, w: torch.Tensor, group, b_mn: bool = False, impl: str = None) -> torch.Tensor:
    """all_gather_rows(x_local) @ w^T (w (N, K)), or @ w (w (K, N)) with ``b_mn``; x_local (rows, K).

    ``impl="pull"``: the copy engines pull every peer's shard from its symmetric buffer into a
    local buffer (each remote row crosses NVLink once) on a side stream while the tensor cores
    multiply the local shard; each remote shard's GEMM starts as soon as its copy lands.
    ``impl="kernel"``: one tcgen05 GEMM whose TMA producer reads the peers' shards directly (no
    multicast); every output n-tile re-reads its remote A tile over NVLink."""
    if (impl or _AG_IMPL) == "kernel":
        return ag_gemm_kernel(x_local, w, group, b_mn)
    from mamformer_b200.ops import gemm
    C = _C()
    ws = _ws(group)
    rows, K = x_local.shape
    N = w.shape[1] if b_mn else w.shape[0]
    P, r = ws.P, ws.rank
    ws.ensure(rows * K, 0 if ws.stage is not None else 64, x_local.device)
    ws.gather[: rows * K].view(rows, K).copy_(x_local)
    ws.barrier(C)                                   # every shard written
    out = torch.empty(P * rows, N, device=x_local.device, dtype=torch.bfloat16)
    cur = torch.cuda.current_stream()
    side = ws.side_stream(x_local.device)
    start = torch.cuda.Event()
    start.record(cur)
    side.wait_event(start)
    pulled = []
    with torch.cuda.stream(side):
        for i in range(1, P):
            q = (r + i) % P
            buf = ws.pull_buffer(i - 1, rows, K, x_local.device)
            buf.copy_(ws.hg.get_buffer(q, (rows, K), torch.bfloat16), non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(side)
            pulled.append((q, buf, ev))
    mm = gemm.mm_nn if b_mn else gemm.mm
    mm(x_local, w, out=out[r * rows:(r + 1) * rows])
    for q, buf, ev in pulled:
        cur.wait_event(ev)
        mm(buf, w, out=out[q * rows:(q + 1) * rows])
    ws.barrier(C)                                   # every peer done pulling this rank's shard
    return out


def ag_gemm_kernel(x_local: torch.Tensor, w: torch.Tensor, group, b_mn: bool = False) -> torch.Tensor:
    """The single-kernel variant of :func:`ag_gemm` (TMA reads of the peers' shards)."""
    C = _C()
    ws = _ws(group)
    rows, K = x_local.shape
    N = w.shape[1] if b_mn else w.shape[0]
    ws.ensure(rows * K, 0 if ws.stage is not None else 64, x_local.device)
    ws.gather[: rows * K].view(rows, K).copy_(x_local)
    ws.barrier(C)                                   # every shard written
    out = torch.empty(ws.P * rows, N, device=x_local.device, dtype=torch.bfloat16)
    C.gemm_ag(ws.hg.buffer_ptrs, rows, K, ws.rank, w, b_mn, out)
    ws.barrier(C)                                   # every peer done reading the shards
    return out


_RS_IMPL = "pull"


@ranged("tp.gemm_rs")
def gemm_rs(y: torch.Tensor, w: torch.Tensor, group, b_mn: bool = False, impl: str = None) -> torch.Tensor:
    """reduce_scatter_rows(y @ w^T) over the group: returns this rank's (rows / P, N) block.

    ``impl="pull"``: each rank first multiplies the row blocks owned by the other ranks into its
    own symmetric staging buffer, then (bounded barrier) the copy engines pull every peer's
    partial for this rank's rows into local buffers on a side stream while the tensor cores
    multiply this rank's own rows; the partials are summed as they land.
    ``impl="kernel"``: one tcgen05 GEMM whose epilogue stores each row block straight into the
    owner's staging slot over NVLink, then a local sum of the slots."""
    if (impl or _RS_IMPL) == "kernel":
        return gemm_rs_kernel(y, w, group, b_mn)
    from mamformer_b200.ops import gemm
    C = _C()
    ws = _ws(group)
    M, K = y.shape
    P, r = ws.P, ws.rank
    rows = M // P
    N = w.shape[1] if b_mn else w.shape[0]
    ws.ensure(64 if ws.gather is None else 0, P * rows * N, y.device)
    y = y.contiguous()
    mm = gemm.mm_nn if b_mn else gemm.mm
    stage = ws.stage[: P * rows * N].view(P * rows, N)
    for i in range(1, P):                           # the other ranks' row blocks first
        q = (r + i) % P
        mm(y[q * rows:(q + 1) * rows], w, out=stage[q * rows:(q + 1) * rows])
    ws.barrier(C)                                   # every rank's partials for the others are staged
    cur = torch.cuda.current_stream()
    side = ws.side_stream(y.device)
    start = torch.cuda.Event()
    start.record(cur)
    side.wait_event(start)
    pulled = []
    with torch.cuda.stream(side):
        for i in range(1, P):
            q = (r - i) % P
            buf = ws.pull_buffer(i - 1, rows, N, y.device)
            buf.copy_(ws.hs.get_buffer(q, (rows, N), torch.bfloat16, r * rows * N), non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(side)
            pulled.append((buf, ev))
    out = mm(y[r * rows:(r + 1) * rows], w)         # this rank's own partial, overlapping the pulls
    for buf, ev in pulled:
        cur.wait_event(ev)
        out.add_(buf)
    ws.barrier(C)                                   # every peer done pulling from this rank's stage
    return out


def gemm_rs_kernel(y: torch.Tensor, w: torch.Tensor, group, b_mn: bool = False) -> torch.Tensor:
    """The single-kernel variant of :func:`gemm_rs` (epilogue stores into the peers' staging)."""
    C = _C()
    ws = _ws(group)
    M, K = y.shape
    P = ws.P
    rows = M // P
    N = w.shape[1] if b_mn else w.shape[0]
    ws.ensure(64 if ws.gather is None else 0, P * rows * N, y.device)
    base = [p_ + ws.rank * rows * N * 2 for p_ in ws.hs.buffer_ptrs]   # my slot in every peer's stage
    C.gemm_rs(y.contiguous(), w, b_mn, base, rows, N, ws.rank)
    ws.barrier(C)                                   # every partial landed
    out = torch.empty(rows, N, device=y.device, dtype=torch.bfloat16)
    stage = ws.stage[: P * rows * N].view(P * rows, N)
    pos = (torch.arange(P, device=y.device).view(1, P) * rows + torch.arange(rows, device=y.device).view(rows, 1))
    C.moe_combine(out, [stage.data_ptr()], N, stage.numel() // N, torch.bfloat16, None, pos.reshape(-1), None, P, None)
    ws.barrier(C)                                   # stage free for the next call
    return out


def gather_rows(x_local: torch.Tensor, group) -> torch.Tensor:
    """Plain all-gather of row shards (NCCL), for the weight-gradient operands."""
    P = dist.get_world_size(group)
    out = torch.empty(P * x_local.shape[0], *x_local.shape[1:], device=x_local.device, dtype=x_local.dtype)
    dist.all_gather_into_tensor(out, x_local.contiguous(), group=group)
    return out


def _wgrad(w, dy, x):
    from mamformer_b200.ops import gemm
    from mamformer_b200.optim import mark_grad_ready
    mg = getattr(w, "main_grad", None)
    if mg is not None:
        gemm.mm_tn_acc(dy, x, mg, accumulate=True)
        mark_grad_ready(w)
        return None
    dw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
    gemm.mm_tn_acc(dy, x, dw, accumulate=True)
    return dw.to(w.dtype)


class _AGLinear(torch.autograd.Function):
    """y (T, n) = all_gather(x) W^T ; x (T/P, K) row shard, W (n, K) column shard."""

    @staticmethod
    def forward(ctx, x, w, group):
        ctx.save_for_backward(x, w)
        ctx.group = group
        return ag_gemm(x, w, group)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = gemm_rs(dy, w, ctx.group, b_mn=True)            # reduce_scatter(dy W)
        dw = _wgrad(w, dy, gather_rows(x, ctx.group))
        return dx, dw, None


class _RSLinear(torch.autograd.Function):
    """z (T/P, d) = reduce_scatter(y W^T) ; y (T, n) full rows of this rank's channel shard."""

    @staticmethod
    def forward(ctx, y, w, group):
        ctx.save_for_backward(y, w)
        ctx.group = group
        return gemm_rs(y, w, group)

    @staticmethod
    def backward(ctx, dz):
        y, w = ctx.saved_tensors
        dz = dz.contiguous()
        dy = ag_gemm(dz, w, ctx.group, b_mn=True)            # all_gather(dz) W
        dw = _wgrad(w, gather_rows(dz, ctx.group), y)
        return dy, dw, None


class SequenceParallelColumnLinear(nn.Module):
    """Column-parallel linear fed by row-sharded activations (fused all-gather -> GEMM)."""

    def __init__(self, in_features: int, out_features: int, group, init_std: float = 0.02):
        super().__init__()
        self.group = group
        P = dist.get_world_size(group)
        assert out_features % P == 0
        self.weight = nn.Parameter(torch.empty(out_features // P, in_features))
        nn.init.normal_(self.weight, std=init_std)

    def forward(self, x):
        shp = x.shape
        y = _AGLinear.apply(x.reshape(-1, shp[-1]), self.weight, self.group)
        return y.view(-1, *shp[1:-1], self.weight.shape[0]) if x.dim() > 2 else y


class SequenceParallelRowLinear(nn.Module):
    """Row-parallel linear whose output is reduce-scattered by rows (fused GEMM -> RS)."""

    def __init__(self, in_features: int, out_features: int, group, init_std: float = 0.02):
        super().__init__()
        self.group = group
        P = dist.get_world_size(group)
        assert in_features % P == 0
        self.weight = nn.Parameter(torch.empty(out_features, in_features // P))
        nn.init.normal_(self.weight, std=init_std)

    def forward(self, y):
        return _RSLinear.apply(y.reshape(-1, y.shape[-1]), self.weight, self.group)


class SequenceParallelSwiGLU(nn.Module):
    """SwiGLU FFN in the sequence-parallel TP layout: x (T/P, d) -> (T/P, d)."""

    def __init__(self, d_model: int, d_ff: int, group):
        super().__init__()
        self.gate_proj = SequenceParallelColumnLinear(d_model, d_ff, group)
        self.up_proj = SequenceParallelColumnLinear(d_model, d_ff, group)
        self.down_proj = SequenceParallelRowLinear(d_ff, d_model, group)

    def forward(self, x):
        from mamformer_b200 import ops
        return self.down_proj(ops.swiglu(self.gate_proj(x), self.up_proj(x)))
