"""Linear layers on the tcgen05 GEMM, with the weight gradient accumulated in the GEMM epilogue.

``y = x W^T (+ b)``: forward ``gemm.mm``; backward ``dx = dy W`` (``gemm.mm_nn``) and
``dW += dy^T x`` written by the fp32-accumulating epilogue straight into the optimizer's
``W.main_grad`` - no bf16 weight gradient is materialised and no separate accumulation kernel
runs (the autograd path returns ``None`` for the weight and signals the data-parallel reducer
that the buffer is final for this backward).  Used for every ``nn.Linear`` of a model in the
bf16 training layout (``FusedLinear``); shapes the GEMM cannot take (features not a multiple of
8, fewer than 64 rows, fp32) go through ``torch.nn.functional.linear``.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from mamformer_b200.ops import gemm


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, w, b):
        y = gemm.mm(x2, w)
        if b is not None:
            y += b.to(y.dtype)
        ctx.save_for_backward(x2, w)
        ctx.has_b = b is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = gemm.mm_nn(dy, w) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            mg = getattr(w, "main_grad", None)
            if mg is not None:
                gemm.mm_tn_acc(dy, x2, mg, accumulate=True)
                from mamformer_b200.optim import mark_grad_ready
                mark_grad_ready(w)
            else:
                dw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
                gemm.mm_tn_acc(dy, x2, dw, accumulate=True)
                dw = dw.to(w.dtype)
        db = dy.float().sum(0).to(dy.dtype) if ctx.has_b else None
        return dx, dw, db


def supported(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and w.dim() == 2
            and w.shape[0] % 8 == 0 and w.shape[1] % 8 == 0 and x.numel() // x.shape[-1] >= 64)


def linear(x: torch.Tensor, w: torch.Tensor, b=None) -> torch.Tensor:
    if not supported(x, w):
        return F.linear(x, w, b)
    shp = x.shape
    y = _Linear.apply(x.reshape(-1, shp[-1]).contiguous(), w, b)
    return y.view(*shp[:-1], w.shape[0])


class FusedLinear(nn.Linear):
    """``nn.Linear`` whose CUDA bf16 forward/backward run on the native GEMM (same parameters
    and state-dict keys)."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return linear(x, self.weight, self.bias)


class _EmbeddingMG(torch.autograd.Function):
    """Row gather whose weight gradient is scattered straight into ``W.main_grad`` (fp32) by the
    native kernel (csrc/optim.cu): no dense vocab x d gradient, no accumulation pass."""

    @staticmethod
    def forward(ctx, ids, w):
        ctx.save_for_backward(ids)
        ctx.w = w
        return F.embedding(ids, w)

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        w = ctx.w
        from mamformer_b200.ops._ext import require_native
        require_native().embedding_grad_accumulate(w.main_grad, ids.reshape(-1).contiguous(),
                                                   dy.reshape(-1, w.shape[1]).contiguous())
        from mamformer_b200.optim import mark_grad_ready
        mark_grad_ready(w)
        return None, None


class FusedEmbedding(nn.Embedding):
    """``nn.Embedding`` whose weight gradient goes straight into the optimizer's fp32
    ``weight.main_grad`` when there is one (CUDA, no padding index / max-norm / sparse options);
    otherwise the plain module's behaviour.  Same parameters and state-dict keys."""

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        w = self.weight
        if (w.requires_grad and torch.is_grad_enabled() and getattr(w, "main_grad", None) is not None
                and w.is_cuda and self.padding_idx is None and self.max_norm is None and not self.sparse
                and not self.scale_grad_by_freq):
            return _EmbeddingMG.apply(ids, w)
        return super().forward(ids)


def use_native_linear(model: nn.Module) -> int:
    """Switch every plain ``nn.Linear`` of ``model`` to :class:`FusedLinear` and every plain
    ``nn.Embedding`` to :class:`FusedEmbedding`; returns the number of linears switched."""
    n = 0
    for m in model.modules():
        if type(m) is nn.Linear:
            m.__class__ = FusedLinear
            n += 1
        elif type(m) is nn.Embedding:
            m.__class__ = FusedEmbedding
    return n
