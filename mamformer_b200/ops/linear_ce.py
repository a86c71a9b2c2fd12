"""Fused linear + cross-entropy: loss = CE(h W^T, labels), never holding all (T, V) logits.

Forward: for chunks of rows, logits = h_c W^T (tcgen05 GEMM, bf16) and one row kernel keeps the
log-sum-exp and the per-row loss.  Backward recomputes each chunk's logits, turns them in place
into ``(softmax - onehot) * grad / n_valid``, then ``dh_c = dlogits W`` and
``dW += dlogits^T h_c`` (the latter accumulated by the GEMM epilogue into the optimizer's fp32
gradient buffer when the weight has one - for the tied embedding this is the same buffer the
embedding-lookup gradient goes to).  The chunk size bounds the live logits to ~1 GB.  When the whole (T, V) logits fit a budget
(``MAMF_CE_SAVE_GB``, default 4 GB per call) the forward keeps them and the backward skips the
recompute: the gradient is formed in place over all rows and the two backward GEMMs run once over
all T rows (the saved logits are consumed, so the graph cannot be backpropagated twice).
Numerics match ``F.cross_entropy`` on bf16 logits with fp32 softmax statistics (mean over rows
whose label is not ``ignore_index``).
"""

from __future__ import annotations

import torch

from mamformer_b200.ops import gemm
from mamformer_b200.ops._ext import require_native

import os

_CHUNK_BYTES = 1 << 30


def _save_budget() -> float:
    return float(os.environ.get("MAMF_CE_SAVE_GB", "4")) * (1 << 30)


def _chunk_rows(V: int) -> int:
    return max(128, min(8192, (_CHUNK_BYTES // (2 * V)) // 128 * 128))


class _LinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, W, labels, ignore_index):
        C = require_native()
        T, d = h.shape
        V = W.shape[0]
        h = h.contiguous()
        labels = labels.contiguous().long()
        loss_rows = torch.empty(T, device=h.device, dtype=torch.float32)
        lse = torch.empty(T, device=h.device, dtype=torch.float32)
        rc = _chunk_rows(V)
        keep = T * V * 2 <= _save_budget()
        buf = torch.empty(T if keep else min(rc, T), V, device=h.device, dtype=torch.bfloat16)
        for r0 in range(0, T, rc):
            r1 = min(T, r0 + rc)
            lg = buf[r0:r1] if keep else buf[: r1 - r0]
            gemm.mm(h[r0:r1], W, out=lg)
            C.ce_stats(lg, labels[r0:r1], ignore_index, loss_rows[r0:r1], lse[r0:r1])
        n_valid = (labels != ignore_index).sum().float()
        loss = loss_rows.sum() / n_valid.clamp(min=1.0)
        ctx.save_for_backward(h, W, labels, lse, n_valid, buf if keep else h.new_empty(0))
        ctx.keep = keep
        ctx.ignore_index = ignore_index
        return loss

    @staticmethod
    def backward(ctx, g):
        C = require_native()
        h, W, labels, lse, n_valid, saved = ctx.saved_tensors
        T, d = h.shape
        V = W.shape[0]
        scale = g.detach().float().reshape(1).contiguous()
        dh = torch.empty_like(h)
        mg = getattr(W, "main_grad", None)
        own = mg is not None
        dW = mg if own else torch.zeros(V, d, device=h.device, dtype=torch.float32)
        if ctx.keep:
            C.ce_grad_inplace(saved, labels, ctx.ignore_index, lse, scale, n_valid.reshape(1))
            gemm.mm_nn(saved, W, out=dh)
            gemm.mm_tn_acc(saved, h, dW, accumulate=True)
            return dh, (None if own else dW.to(W.dtype)), None, None
        rc = _chunk_rows(V)
        buf = torch.empty(min(rc, T), V, device=h.device, dtype=torch.bfloat16)
        for r0 in range(0, T, rc):
            r1 = min(T, r0 + rc)
            lg = buf[: r1 - r0]
            gemm.mm(h[r0:r1], W, out=lg)
            C.ce_grad_inplace(lg, labels[r0:r1], ctx.ignore_index, lse[r0:r1], scale, n_valid.reshape(1))
            gemm.mm_nn(lg, W, out=dh[r0:r1])
            gemm.mm_tn_acc(lg, h[r0:r1], dW, accumulate=True)
        return dh, (None if own else dW.to(W.dtype)), None, None


def supported(h: torch.Tensor, W: torch.Tensor) -> bool:
    return (h.is_cuda and h.dtype == torch.bfloat16 and W.dtype == torch.bfloat16
            and h.shape[1] % 64 == 0 and W.shape[0] % 8 == 0)


def linear_cross_entropy(h, W, labels, ignore_index: int = -100):
    return _LinearCE.apply(h, W, labels, ignore_index)
