"""Tensor parallelism (Megatron-style column/row sharding) for the hybrid blocks.

Reference: ``mamformer/parallelism/tensor_parallel.py`` (``_tp_all_reduce`` 60-72,
``_tp_all_gather`` 90-103, ``_tp_reduce_scatter`` 105-121, ``ColumnParallelLinear`` 136-190,
``RowParallelLinear`` 192-250, ``TPAttention`` 252-380, ``TPMamba2Block`` 382-520,
``TPDeepSeekMoE`` 522-668, ``shard_model_tp`` 670-700).  The reference's ``shard_model_tp`` only
warns (retroactive sharding not implemented) and its ``TPMamba2Block`` gives every rank its own
B/C/dt projections of its channel slice, which is a different model from the unsharded one.
Here :func:`shard_model_tp` shards a built model in place and the sharded model computes the
same function as the unsharded one:

* attention (GQA, KDA-Diff linear/full): Q/K/V (and the K/V state-injection and MLA expand
  projections) column-parallel by heads, per-head lambda and GroupNorm affine sliced, output
  projection row-parallel;
* Mamba block: in_proj column-parallel (matching x and z channel slices), conv / D / dt-expand
  sliced by channel, dt-compress / B / C projections row-parallel (their outputs are shared by
  all channels), A_log replicated with its gradient summed over the TP group, the per-step
  channel-mean state for K/V injection averaged over the TP group, out_proj row-parallel;
* SwiGLU FFNs and shared experts: gate/up column, down row.
Routed experts are sharded by expert parallelism, not by TP; a model whose MoE layers would
need TP-sharded routed experts is rejected.

Autograd collectives (``f`` / ``g`` of Megatron): ``copy_to_tp`` is identity forward and
all-reduce backward; ``reduce_from_tp`` is all-reduce forward and identity backward.

With ``shard_model_tp(fused=True)`` (the default), on CUDA in bf16 (and when the token count splits into
128-row shards) every TP all-reduce that follows a GEMM is fused into it: the row-parallel
forward and the column-parallel input-gradient run as the tcgen05 GEMM whose epilogue stores
each row shard of the partial product straight into the owning rank's staging buffer over
NVLink (GEMM -> reduce-scatter in one kernel, see ``tp_fused.gemm_rs``), followed by an
all-gather of the reduced shards; the local GEMMs and the weight gradients (accumulated into the
fp32 optimizer buffer) run on the same kernel.  ``tp_fused.gemm_rs`` defaults to its overlapped
form (the other ranks' row blocks first, then copy-engine pulls of the peers' partials while the
own rows multiply): 0.446 ms against 0.560 ms for GEMM + NCCL reduce-scatter on 2 B200s at
T = 16384, K = N = 4096 (``utils/comm_bench.py``).  ``fused=False`` keeps GEMM + NCCL all-reduce.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

_TP_GROUP: Optional[dist.ProcessGroup] = None
_DIAG = (None, None)


def set_tp_group(group: Optional[dist.ProcessGroup]) -> None:
    global _TP_GROUP
    _TP_GROUP = group


_set_tp_group = set_tp_group


def get_tp_group() -> Optional[dist.ProcessGroup]:
    return _TP_GROUP


def get_tp_rank_size(group=None) -> Tuple[int, int]:
    g = group if group is not None else _TP_GROUP
    if g is None or not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    return dist.get_rank(g), dist.get_world_size(g)


def set_comm_diagnostics(start_fn, end_fn) -> None:
    """Install callbacks ``start(op, bytes)`` / ``end(op)`` around every TP collective."""
    global _DIAG
    _DIAG = (start_fn, end_fn)


def _diag(op, t):
    class _Ctx:
        def __enter__(self):
            if _DIAG[0] is not None:
                _DIAG[0](op, t.numel() * t.element_size())

        def __exit__(self, *a):
            if _DIAG[1] is not None:
                _DIAG[1](op)
    return _Ctx()


def _all_reduce(t, group):
    with _diag("tp_all_reduce", t):
        dist.all_reduce(t, group=group)
    return t


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        return _all_reduce(g.contiguous().clone(), ctx.group), None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        return _all_reduce(x.contiguous().clone(), group)

    @staticmethod
    def backward(ctx, g):
        return g, None


class _MeanFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.n = dist.get_world_size(group)
        return _all_reduce(x.contiguous().clone(), group) / ctx.n

    @staticmethod
    def backward(ctx, g):
        return g / ctx.n, None


class _GatherLastDim(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        n = dist.get_world_size(group)
        ctx.group, ctx.n, ctx.r = group, n, dist.get_rank(group)
        parts = [torch.empty_like(x) for _ in range(n)]
        with _diag("tp_all_gather", x):
            dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, -1)

    @staticmethod
    def backward(ctx, g):
        return g.chunk(ctx.n, -1)[ctx.r].contiguous(), None


class _ScatterLastDim(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        n = dist.get_world_size(group)
        ctx.group = group
        return x.chunk(n, -1)[dist.get_rank(group)].contiguous()

    @staticmethod
    def backward(ctx, g):
        return _GatherLastDim.apply(g, ctx.group), None


def copy_to_tp(x, group=None):
    g = group if group is not None else _TP_GROUP
    return x if g is None else _CopyToTP.apply(x, g)


def reduce_from_tp(x, group=None):
    g = group if group is not None else _TP_GROUP
    return x if g is None else _ReduceFromTP.apply(x, g)


def mean_from_tp(x, group=None):
    g = group if group is not None else _TP_GROUP
    return x if g is None else _MeanFromTP.apply(x, g)


def gather_from_tp(x, group=None):
    g = group if group is not None else _TP_GROUP
    return x if g is None else _GatherLastDim.apply(x, g)


def scatter_to_tp(x, group=None):
    g = group if group is not None else _TP_GROUP
    return x if g is None else _ScatterLastDim.apply(x, g)


# reference-named aliases (tensor_parallel.py:60-121)
def _tp_all_reduce(t):
    return reduce_from_tp(t)


def _tp_all_gather(t, dim: int = -1):
    assert dim in (-1, t.dim() - 1), "all-gather along the last dimension"
    return gather_from_tp(t)


def _tp_reduce_scatter(t, dim: int = -1):
    g = _TP_GROUP
    if g is None:
        return t
    n, r = dist.get_world_size(g), dist.get_rank(g)
    full = _all_reduce(t.contiguous().clone(), g)
    return full.chunk(n, dim)[r].contiguous()


# ---------------------------------------------------------------------------------------------
def _sliced(p: torch.Tensor, dim: int, index: torch.Tensor) -> nn.Parameter:
    """This rank's slice of an unsharded parameter; ``_mamf_tp_slice`` records (dim, index) so
    checkpoints can be consolidated and tests can compare against the unsharded model."""
    out = nn.Parameter(p.detach().index_select(dim, index.to(p.device)).clone(), requires_grad=p.requires_grad)
    out._mamf_tp_slice = (dim, index)
    return out


def _fused_ok(x2: torch.Tensor, w: torch.Tensor, group) -> bool:
    """The fused GEMM + reduce-scatter applies: CUDA bf16 operands, 16-byte rows, and the token
    count splits into shards of whole 128-row tiles."""
    if group is None or not x2.is_cuda or x2.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        return False
    P = dist.get_world_size(group)
    T = x2.shape[0]
    return (P > 1 and T % (P * 128) == 0 and x2.shape[1] % 8 == 0 and w.shape[0] % 8 == 0
            and w.shape[1] % 8 == 0)


def _gather_shards(z: torch.Tensor, group) -> torch.Tensor:
    P = dist.get_world_size(group)
    out = torch.empty(P * z.shape[0], z.shape[1], device=z.device, dtype=z.dtype)
    with _diag("tp_all_gather", z):
        dist.all_gather_into_tensor(out, z.contiguous(), group=group)
    return out


class _FusedRowLinear(torch.autograd.Function):
    """y (T, N) = sum_r x_r W_r^T: fused GEMM -> reduce-scatter, then all-gather of the shards.
    Backward needs no collective: dx_r = dy W_r, dW_r += dy^T x_r."""

    @staticmethod
    def forward(ctx, x2, w, group):
        from mamformer_b200.parallel import tp_fused
        ctx.save_for_backward(x2, w)
        ctx.group = group
        return _gather_shards(tp_fused.gemm_rs(x2, w, group), group)

    @staticmethod
    def backward(ctx, dy):
        from mamformer_b200.ops import gemm
        from mamformer_b200.parallel.tp_fused import _wgrad
        x2, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = gemm.mm_nn(dy, w) if ctx.needs_input_grad[0] else None
        dw = _wgrad(w, dy, x2) if ctx.needs_input_grad[1] else None
        return dx, dw, None


class _FusedColumnLinear(torch.autograd.Function):
    """y_r = x W_r^T with x replicated; its input gradient sum_r dy_r W_r is the fused
    GEMM -> reduce-scatter followed by an all-gather."""

    @staticmethod
    def forward(ctx, x2, w, group):
        from mamformer_b200.ops import gemm
        ctx.save_for_backward(x2, w)
        ctx.group = group
        return gemm.mm(x2, w)

    @staticmethod
    def backward(ctx, dy):
        from mamformer_b200.parallel import tp_fused
        from mamformer_b200.parallel.tp_fused import _wgrad
        x2, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = _gather_shards(tp_fused.gemm_rs(dy, w, ctx.group, b_mn=True), ctx.group)
        dw = _wgrad(w, dy, x2) if ctx.needs_input_grad[1] else None
        return dx, dw, None


class ColumnParallelLinear(nn.Module):
    """y_local = x W_local^T (+ b_local); W sharded along its output dimension."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, gather_output: bool = False,
                 group=None, init_std: float = 0.02):
        super().__init__()
        self.group = group if group is not None else _TP_GROUP
        r, n = get_tp_rank_size(self.group)
        assert out_features % n == 0, f"out_features {out_features} % tp {n}"
        self.in_features, self.out_features = in_features, out_features
        self.out_local = out_features // n
        self.gather_output = gather_output
        self.weight = nn.Parameter(torch.empty(self.out_local, in_features))
        self.bias = nn.Parameter(torch.zeros(self.out_local)) if bias else None
        nn.init.normal_(self.weight, mean=0.0, std=init_std)

    @classmethod
    def from_linear(cls, lin: nn.Linear, rows: torch.Tensor, group, gather_output: bool = False):
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.group = group
        m.in_features, m.out_features = lin.in_features, lin.out_features
        m.out_local = int(rows.numel())
        m.gather_output = gather_output
        m.weight = _sliced(lin.weight, 0, rows)
        m.bias = _sliced(lin.bias, 0, rows) if lin.bias is not None else None
        return m

    def forward(self, x):
        if getattr(self, "fused", True) and not self.gather_output and self.bias is None:
            x2 = x.reshape(-1, x.shape[-1])
            if _fused_ok(x2, self.weight, self.group):
                y = _FusedColumnLinear.apply(x2.contiguous(), self.weight, self.group)
                return y.view(*x.shape[:-1], self.out_local)
        x = copy_to_tp(x, self.group)
        y = F.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))
        return gather_from_tp(y, self.group) if self.gather_output else y

    def extra_repr(self):
        return f"in={self.in_features}, out={self.out_features} (local {self.out_local})"


class RowParallelLinear(nn.Module):
    """y = all_reduce(x_local W_local^T) (+ b); W sharded along its input dimension."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, input_is_parallel: bool = True,
                 group=None, init_std: float = 0.02):
        super().__init__()
        self.group = group if group is not None else _TP_GROUP
        r, n = get_tp_rank_size(self.group)
        assert in_features % n == 0, f"in_features {in_features} % tp {n}"
        self.in_features, self.out_features = in_features, out_features
        self.in_local = in_features // n
        self.input_is_parallel = input_is_parallel
        self.weight = nn.Parameter(torch.empty(out_features, self.in_local))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        nn.init.normal_(self.weight, mean=0.0, std=init_std)

    @classmethod
    def from_linear(cls, lin: nn.Linear, cols: torch.Tensor, group):
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.group = group
        m.in_features, m.out_features = lin.in_features, lin.out_features
        m.in_local = int(cols.numel())
        m.input_is_parallel = True
        m.weight = _sliced(lin.weight, 1, cols)
        m.bias = nn.Parameter(lin.bias.detach().clone()) if lin.bias is not None else None
        return m

    def forward(self, x):
        if not self.input_is_parallel:
            x = scatter_to_tp(x, self.group)
        if getattr(self, "fused", True):
            x2 = x.reshape(-1, x.shape[-1])
            if _fused_ok(x2, self.weight, self.group):
                y = _FusedRowLinear.apply(x2.contiguous(), self.weight, self.group)
                y = y.view(*x.shape[:-1], self.out_features)
                return y if self.bias is None else y + self.bias.to(y.dtype)
        y = reduce_from_tp(F.linear(x, self.weight.to(x.dtype)), self.group)
        return y if self.bias is None else y + self.bias.to(y.dtype)

    def extra_repr(self):
        return f"in={self.in_features} (local {self.in_local}), out={self.out_features}"


# ---------------------------------------------------------------------------------------------
def _block_rows(n_total: int, r: int, n: int, block: int = 1) -> torch.Tensor:
    """Indices of rank r's contiguous 1/n share of n_total rows (in units of `block`)."""
    per = n_total // n
    assert per * n == n_total and per % block == 0, f"{n_total} rows do not split over tp={n}"
    return torch.arange(r * per, (r + 1) * per)


def _grad_all_reduce_hook(p: nn.Parameter, group) -> None:
    """Replicated parameter whose local gradient is a partial sum over this rank's shard."""
    p.register_hook(lambda g: _all_reduce(g.contiguous().clone(), group))
    p._mamf_tp_partial = True


def _col(parent, name, rows, group):
    setattr(parent, name, ColumnParallelLinear.from_linear(getattr(parent, name), rows, group))


def _row(parent, name, cols, group):
    setattr(parent, name, RowParallelLinear.from_linear(getattr(parent, name), cols, group))


def _shard_heads(mod, r, n, group, q_names, kv_names, kv_extra=()):
    H, G, hd = mod.n_heads, mod.n_kv_heads, mod.head_dim
    if H % n or G % n:
        raise ValueError(f"heads ({H} q / {G} kv) do not split over tp={n}")
    qrows = _block_rows(H * hd, r, n, hd)
    kvrows = _block_rows(G * hd, r, n, hd)
    for nm in q_names:
        _col(mod, nm, qrows, group)
    for nm in tuple(kv_names) + tuple(kv_extra):
        if getattr(mod, nm, None) is not None:
            _col(mod, nm, kvrows, group)
    _row(mod, "o_proj", qrows, group)
    mod.n_heads, mod.n_kv_heads = H // n, G // n
    if hasattr(mod, "lambda_raw") and mod.lambda_raw.numel() == H:
        hs = torch.arange(r * (H // n), (r + 1) * (H // n))
        mod.lambda_raw = _sliced(mod.lambda_raw, 0, hs)
    gn = getattr(mod, "group_norm", None)
    if gn is not None:
        new = nn.GroupNorm(H // n, (H // n) * hd, eps=gn.eps)
        new.weight = _sliced(gn.weight, 0, qrows)
        new.bias = _sliced(gn.bias, 0, qrows)
        mod.group_norm = new


def _shard_mamba(mod, r, n, group):
    di = mod.d_inner
    rows = _block_rows(di, r, n)
    in_rows = torch.cat([rows, rows + di])
    _col(mod, "in_proj", in_rows, group)
    conv = mod.conv1d
    newc = nn.Conv1d(rows.numel(), rows.numel(), conv.kernel_size[0], groups=rows.numel(),
                     padding=conv.padding, bias=conv.bias is not None)
    newc.weight = _sliced(conv.weight, 0, rows)
    if conv.bias is not None:
        newc.bias = _sliced(conv.bias, 0, rows)
    mod.conv1d = newc
    _row(mod.dt_proj, "0", rows, group)
    _col(mod.dt_proj, "1", rows, group)
    _row(mod, "B_proj", rows, group)
    _row(mod, "C_proj", rows, group)
    mod.D = _sliced(mod.D, 0, rows)
    _row(mod, "out_proj", rows, group)
    _grad_all_reduce_hook(mod.A_log, group)
    mod.d_inner = di // n
    mod.tp_group = group


def _shard_ffn(mod, r, n, group):
    I = mod.gate_proj.out_features
    rows = _block_rows(I, r, n)
    _col(mod, "gate_proj", rows, group)
    _col(mod, "up_proj", rows, group)
    _row(mod, "down_proj", rows, group)


def shard_model_tp(model: nn.Module, tp_size: int, group=None, fused: bool = True) -> nn.Module:
    """Shard every supported block of ``model`` over the TP group, in place.  Must run before
    the optimizer is built.  ``fused``: fuse the reduce-scatter half of each TP all-reduce into
    the preceding GEMM where the shapes allow (CUDA, bf16)."""
    group = group if group is not None else _TP_GROUP
    if tp_size <= 1:
        return model
    if group is None:
        raise RuntimeError("shard_model_tp needs the TP process group (DistributedCoordinator.initialize)")
    r, n = get_tp_rank_size(group)
    assert n == tp_size
    from mamformer_b200.models.attention import GroupedQueryAttention as Attention
    from mamformer_b200.models.ffn import SwiGLUFFN
    from mamformer_b200.models.kda_diff import FullDiffAttention, LinearDiffAttention
    from mamformer_b200.models.mamba2 import Mamba2Block
    from mamformer_b200.models.moe import DeepSeekMoE, _SwiGLUExpert
    mods = list(model.modules())
    for m in mods:
        if isinstance(m, DeepSeekMoE) and m.n_routed_experts > 0:
            raise NotImplementedError("routed experts are sharded with expert parallelism (ep_size), not TP")
    for m in mods:
        if isinstance(m, Mamba2Block):
            _shard_mamba(m, r, n, group)
        elif isinstance(m, LinearDiffAttention):
            _shard_heads(m, r, n, group, ("q1_proj", "q2_proj"), ("k_proj", "v_proj"),
                         ("h_state_k_proj", "h_state_v_proj"))
        elif isinstance(m, FullDiffAttention):
            _shard_heads(m, r, n, group, ("q1_proj", "q2_proj"), ("k_expand", "v_expand"),
                         ("h_state_k_proj", "h_state_v_proj"))
        elif isinstance(m, Attention):
            _shard_heads(m, r, n, group, ("q_proj",), ("k_proj", "v_proj"))
        elif isinstance(m, (SwiGLUFFN, _SwiGLUExpert)):
            _shard_ffn(m, r, n, group)
    for m in model.modules():
        if hasattr(m, "kv_dim") and hasattr(m, "k_expand"):
            m.kv_dim = m.k_expand.out_local
        if isinstance(m, (ColumnParallelLinear, RowParallelLinear)):
            m.fused = fused
    model._mamf_tp = (r, n)
    return model


# ---------------------------------------------------------------------------------------------
class TPAttention(nn.Module):
    """Stand-alone TP GQA attention (reference ``TPAttention``): local heads, row-parallel
    output projection."""

    def __init__(self, d_model: int, n_heads: int, n_kv_heads: int, head_dim: int, max_seq_len: int = 8192,
                 rope_theta: float = 10000.0, sliding_window: int = 0, group=None, **kw):
        super().__init__()
        from mamformer_b200.models.attention import GroupedQueryAttention
        self.inner = GroupedQueryAttention(d_model, n_heads, n_kv_heads, head_dim, max_seq_len=max_seq_len,
                               rope_theta=rope_theta, sliding_window=sliding_window, **kw)
        g = group if group is not None else _TP_GROUP
        r, n = get_tp_rank_size(g)
        if n > 1:
            _shard_heads(self.inner, r, n, g, ("q_proj",), ("k_proj", "v_proj"))

    def forward(self, x, attention_mask=None, use_cache=False, cache=None, **kw):
        return self.inner(x, attention_mask=attention_mask, use_cache=use_cache, cache=cache, **kw)


class TPMamba2Block(nn.Module):
    """Stand-alone TP Mamba block computing the same function as the unsharded block."""

    def __init__(self, d_model: int, d_state: int = 128, d_conv: int = 4, expand: int = 1,
                 dt_rank: Optional[int] = None, group=None):
        super().__init__()
        from mamformer_b200.models.mamba2 import Mamba2Block
        self.inner = Mamba2Block(d_model, d_state=d_state, d_conv=d_conv, expand=expand,
                                 dt_rank=dt_rank if dt_rank is not None else math.ceil(d_model / 16))
        g = group if group is not None else _TP_GROUP
        r, n = get_tp_rank_size(g)
        if n > 1:
            _shard_mamba(self.inner, r, n, g)

    def forward(self, u, use_cache: bool = False, cache=None, return_h_states: bool = False):
        return self.inner(u, use_cache=use_cache, cache=cache, return_h_states=return_h_states)


class TPSwiGLUFFN(nn.Module):
    """Stand-alone TP SwiGLU FFN (column gate/up, row down)."""

    def __init__(self, d_model: int, d_ff: int, group=None):
        super().__init__()
        from mamformer_b200.models.ffn import SwiGLUFFN
        self.inner = SwiGLUFFN(d_model, d_ff)
        g = group if group is not None else _TP_GROUP
        r, n = get_tp_rank_size(g)
        if n > 1:
            _shard_ffn(self.inner, r, n, g)

    def forward(self, x):
        return self.inner(x)
