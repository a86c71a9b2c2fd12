"""Routed-expert computation on the tensor cores (single device; the expert-parallel engine
reuses the same pieces on each rank's local experts).

Forward for T tokens with top-k assignments (reference semantics ``moe.py:310-332``):

1. counting sort of the T*k assignments by expert: each expert's rows start at a 64-aligned
   offset ``seg[e]`` of a permuted buffer whose size is a fixed upper bound (T*k + 64*E rows),
   so nothing here waits for the host; pad rows are zero;
2. ``H_g = X_e W_gate_e^T``, ``H_u = X_e W_up_e^T`` (tcgen05 grouped GEMM, one launch each);
3. ``A = silu(H_g) * H_u`` (native SwiGLU);
4. ``Y_e = A_e W_down_e^T`` (grouped GEMM);
5. ``out[t] = sum_j gate[t, j] * Y[pos[t, j]]``.

Backward: ``dY`` rows = gate * dout, ``dgate = <dout, Y>``; ``dA = dY W_down`` and
``dX = dH_g W_gate + dH_u W_up`` (grouped GEMMs with MN-major weights); weight gradients
``dW_e += dY_e^T A_e`` etc. (grouped-K GEMMs) are accumulated by the GEMM epilogue straight into
the optimizer's fp32 gradient buffer (``param.main_grad``) when it exists, so no bf16 gradient
is materialised for the 128 experts.
"""

from __future__ import annotations

from typing import Optional

import torch

from mamformer_b200.ops import gemm

ALIGN = 64


def plan(idx: torch.Tensor, n_experts: int):
    """Counting-sort plan for the (T, k) expert indices.

    Returns (pos (T*k,) int64 row of each assignment in the permuted buffer, seg (E+1,) int32,
    tile_off (E+1,) int32, counts (E,) int32/int64, rows (int, upper bound of the buffer size)).
    On CUDA one native counting sort (``csrc/moe_rows.cu`` ``moe_sort_plan``) builds the plan on
    the device; the eager form below is the CPU path and the oracle of its test."""
    flat = idx.reshape(-1).long()
    rows = (flat.numel() + ALIGN * n_experts + ALIGN - 1) // ALIGN * ALIGN
    if flat.is_cuda and n_experts <= 256:
        from mamformer_b200.ops._ext import require_native
        srow, counts, start, seg, tile_off, pos = require_native().moe_sort_plan(flat, n_experts, True)
        return pos, seg, tile_off, counts, rows
    return plan_eager(flat, n_experts) + (rows,)


def plan_eager(flat: torch.Tensor, n_experts: int):
    """Eager counting sort: (pos, seg int32, tile_off int32, counts int64)."""
    counts = torch.bincount(flat, minlength=n_experts)
    padded = (counts + ALIGN - 1) // ALIGN * ALIGN
    seg = torch.zeros(n_experts + 1, dtype=torch.int64, device=flat.device)
    seg[1:] = torch.cumsum(padded, 0)
    start = torch.zeros(n_experts, dtype=torch.int64, device=flat.device)
    start[1:] = torch.cumsum(counts, 0)[:-1]
    order = torch.sort(flat, stable=True).indices
    sorted_e = flat[order]
    rank = torch.arange(flat.numel(), device=flat.device) - start[sorted_e]
    pos = torch.empty_like(flat)
    pos[order] = seg[sorted_e] + rank
    seg32 = seg.to(torch.int32)
    return pos, seg32, gemm.tile_offsets(seg32), counts


def _grouped_buffer(rows, d, dtype, device, seg, counts):
    """Expert-grouped row buffer whose pad rows are zero; the real rows are left for the caller
    to write (native: only the pads are cleared, instead of the whole buffer)."""
    if device.type == "cuda" and dtype == torch.bfloat16 and counts.dtype == torch.int32 and d % 8 == 0:
        from mamformer_b200.ops._ext import require_native
        buf = torch.empty(rows, d, device=device, dtype=dtype)
        require_native().moe_zero_pad_rows(buf, seg, counts)
        return buf
    return torch.zeros(rows, d, device=device, dtype=dtype)


def _grad_sink(w: torch.Tensor):
    """fp32 buffer the weight gradient is accumulated into (the optimizer's, if attached)."""
    mg = getattr(w, "main_grad", None)
    if mg is not None:
        return mg, True
    return torch.zeros(w.shape, device=w.device, dtype=torch.float32), False


def mlp_forward(xp, seg, tile_off, w_gate, w_up, w_down, y_out=None):
    """Grouped SwiGLU experts on expert-grouped rows: returns (hg, hu, act, yp)."""
    from mamformer_b200.ops.native import _C
    hg = gemm.grouped_mm(xp, w_gate, seg, tile_off)
    hu = gemm.grouped_mm(xp, w_up, seg, tile_off)
    act = _C.swiglu_fwd(hg, hu)
    yp = gemm.grouped_mm(act, w_down, seg, tile_off, out=y_out)
    return hg, hu, act, yp


def mlp_backward(dyp, xp, hg, hu, act, seg, tile_off, w_gate, w_up, w_down, dx_out=None):
    """Backward of :func:`mlp_forward`.  Returns (dxp fp32, grads) where grads holds the bf16
    weight gradients of the weights without an optimizer buffer (None for the others, whose
    gradient was accumulated in place)."""
    from mamformer_b200.ops.native import _C
    dact = gemm.grouped_mm_nn(dyp, w_down, seg, tile_off)
    gd, own_d = _grad_sink(w_down)
    gemm.grouped_wgrad(dyp, act, seg, gd, accumulate=True)
    dhg, dhu = _C.swiglu_bwd(hg, hu, dact)
    dxp = gemm.grouped_mm_nn(dhg, w_gate, seg, tile_off, out=dx_out, out_dtype=torch.float32)
    _C.gemm_tn(dhu, False, w_up, True, dxp, True, seg, tile_off, 1, 1.0)
    gg, own_g = _grad_sink(w_gate)
    gemm.grouped_wgrad(dhg, xp, seg, gg, accumulate=True)
    gu, own_u = _grad_sink(w_up)
    gemm.grouped_wgrad(dhu, xp, seg, gu, accumulate=True)
    from mamformer_b200.optim import mark_grad_ready
    for w, own in ((w_gate, own_g), (w_up, own_u), (w_down, own_d)):
        if own:
            mark_grad_ready(w)
    grads = (None if own_g else gg.to(w_gate.dtype), None if own_u else gu.to(w_up.dtype),
             None if own_d else gd.to(w_down.dtype))
    return dxp, grads


class _RoutedExperts(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gates, idx, w_gate, w_up, w_down, combine):
        from mamformer_b200.ops.native import _C
        T, d = x.shape
        k = idx.shape[1]
        E = w_gate.shape[0]
        pos, seg, tile_off, counts, rows = plan(idx, E)
        xp = _grouped_buffer(rows, d, x.dtype, x.device, seg, counts)
        _C.moe_scatter_rows(xp, pos, x, k)
        hg, hu, act, yp = mlp_forward(xp, seg, tile_off, w_gate, w_up, w_down)
        g32 = gates.float().reshape(-1).contiguous()
        ctx.save_for_backward(xp, hg, hu, act, yp, pos, seg, tile_off, g32, w_gate, w_up, w_down, counts)
        ctx.combine = combine
        ctx.shape = (T, k, d)
        ctx.gdtype = gates.dtype
        if combine:
            out = torch.empty(T, d, device=x.device, dtype=x.dtype)
            _C.moe_combine(out, [yp.data_ptr()], yp.stride(0), yp.shape[0], yp.dtype, None, pos, g32, k, None)
            return out
        return yp[pos].view(T, k, d)

    @staticmethod
    def backward(ctx, dout):
        from mamformer_b200.ops.native import _C
        xp, hg, hu, act, yp, pos, seg, tile_off, g32, w_gate, w_up, w_down, counts = ctx.saved_tensors
        T, k, d = ctx.shape
        rows = xp.shape[0]
        dyp = _grouped_buffer(rows, d, xp.dtype, xp.device, seg, counts)
        dout = dout.to(xp.dtype).contiguous()
        if ctx.combine:
            dg = torch.empty(T * k, device=xp.device, dtype=torch.float32)
            _C.moe_combine_bwd(dout, yp, pos, g32, dg, dyp, pos, k)
            dgates = dg.view(T, k).to(ctx.gdtype)
        else:
            dgates = None
            _C.moe_scatter_rows(dyp, pos, dout.reshape(T * k, d), 1)
        dxp, (gw_g, gw_u, gw_d) = mlp_backward(dyp, xp, hg, hu, act, seg, tile_off, w_gate, w_up, w_down)
        dx = torch.empty(T, d, device=xp.device, dtype=xp.dtype)
        _C.moe_combine(dx, [dxp.data_ptr()], dxp.stride(0), dxp.shape[0], dxp.dtype, None, pos, None, k, None)
        return dx, dgates, None, gw_g, gw_u, gw_d, None


def supported(x: torch.Tensor, w_gate: torch.Tensor) -> bool:
    d, I = x.shape[1], w_gate.shape[1]
    return (x.is_cuda and x.dtype == torch.bfloat16 and w_gate.dtype == torch.bfloat16
            and d % 64 == 0 and I % 64 == 0)


def routed(x, idx, gates, w_gate, w_up, w_down):
    return _RoutedExperts.apply(x.contiguous(), gates, idx, w_gate, w_up, w_down, True)


def expert_outputs(x, idx, w_gate, w_up, w_down):
    dummy = torch.ones(idx.shape, device=x.device, dtype=torch.float32)
    return _RoutedExperts.apply(x.contiguous(), dummy, idx, w_gate, w_up, w_down, False)
