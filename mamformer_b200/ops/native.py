"""Autograd wrappers around the native kernels in ``mamformer_b200._C``.

Importing this module registers the covered op names in ``ops.NATIVE``.  Each wrapper keeps
the tensors its backward kernel needs and nothing else (e.g. the scan saves chunk-start
states, not per-step states).
"""

from __future__ import annotations

import os

import torch

from mamformer_b200.ops import NATIVE
from mamformer_b200.ops._ext import require_native

_C = require_native()


def _register(name: str, source: str):
    def deco(fn):
        NATIVE[name] = source
        return fn
    return deco


# ---------------------------------------------------------------------------------------------
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        shape = x.shape
        x2 = x.contiguous()
        y, rstd = _C.rmsnorm_fwd(x2, w.float().contiguous(), float(eps))
        ctx.save_for_backward(x2, w, rstd)
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx, dw = _C.rmsnorm_bwd(x, w.float().contiguous(), dy.contiguous(), rstd)
        return dx.view(dy.shape), dw.to(w.dtype), None


@_register("rms_norm", "csrc/elementwise.cu")
def rms_norm(x, weight, eps):
    return _RMSNorm.apply(x, weight, eps)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, g, u):
        ctx.save_for_backward(g, u)
        return _C.swiglu_fwd(g, u)

    @staticmethod
    def backward(ctx, dy):
        g, u = ctx.saved_tensors
        dg, du = _C.swiglu_bwd(g, u, dy)
        return dg, du


@_register("swiglu", "csrc/elementwise.cu")
def swiglu(gate, up):
    if gate.shape[-1] * gate.element_size() % 16 or up.stride(-1) != 1 or gate.stride(-1) != 1:
        from mamformer_b200.ops import reference
        return reference.swiglu(gate, up)
    return _SwiGLU.apply(gate, up)


class _Rope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin):
        ctx.save_for_backward(cos, sin)
        return _C.rope_apply(x, cos, sin, False)

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        return _C.rope_apply(dy.contiguous(), cos, sin, True), None, None


@_register("rope", "csrc/elementwise.cu")
def rope(x, cos, sin):
    if x.stride(-1) != 1 or x.stride(-2) != x.shape[-1] or x.stride(0) != x.stride(1) * x.shape[1]:
        x = x.contiguous()
    return _Rope.apply(x, cos, sin)


class _ConvSiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        return _C.conv_silu_fwd(x, w)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dx, dw = _C.conv_silu_bwd(x, w, dy)
        return dx, dw.to(w.dtype)


@_register("causal_conv1d_silu", "csrc/elementwise.cu")
def causal_conv1d_silu(x, weight):
    return _ConvSiLU.apply(x, weight)


class _HeadGroupNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, H, w, b, eps):
        x = x.contiguous()
        y, mr = _C.head_groupnorm_fwd(x, int(H), w, b, float(eps))
        ctx.save_for_backward(x, w, mr)
        ctx.H = int(H)
        ctx.wdt = (w.dtype, b.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, mr = ctx.saved_tensors
        dx, dw, db = _C.head_groupnorm_bwd(x, ctx.H, w, mr, dy.contiguous())
        return dx, None, dw.to(ctx.wdt[0]), db.to(ctx.wdt[1]), None


@_register("head_group_norm", "csrc/elementwise.cu")
def head_group_norm(x, n_heads, weight, bias, eps):
    return _HeadGroupNorm.apply(x, n_heads, weight, bias, eps)


# ---------------------------------------------------------------------------------------------
class _Scan(torch.autograd.Function):
    """Outputs (y, h_states-or-None, final-or-None); gradients for x, dt, A_log, B, C, D, z."""

    @staticmethod
    def forward(ctx, x, dt, A_log, Bm, Cm, D, z, softplus, need_hs, need_final):
        A32 = A_log.float().contiguous()
        D32 = D.float().contiguous()
        y, hs, ckpt, fin = _C.selective_scan_fwd(x, dt, A32, Bm, Cm, D32, z, None, softplus,
                                                 need_hs, need_final)
        ctx.save_for_backward(x, dt, A_log, Bm, Cm, D, z if z is not None else x.new_empty(0), ckpt)
        ctx.has_z = z is not None
        ctx.softplus = softplus
        ctx.need_hs = need_hs
        if need_final:
            ctx.mark_non_differentiable(fin)
        return y, (hs if need_hs else None), (fin if need_final else None)

    @staticmethod
    def backward(ctx, dy, dhs, dfin):
        x, dt, A_log, Bm, Cm, D, z, ckpt = ctx.saved_tensors
        z = z if ctx.has_z else None
        if dy is None:
            dy = torch.zeros_like(x)
        dhs_in = dhs if (ctx.need_hs and dhs is not None) else None
        dx, ddt, dB, dC, dz, dA, dD = _C.selective_scan_bwd(
            x, dt, A_log.float().contiguous(), Bm, Cm, D.float().contiguous(), z, ckpt,
            dy.contiguous(), dhs_in, ctx.softplus)
        al = A_log.float()
        dA_log = dA * torch.exp(al.clamp(-5.0, 5.0)) * ((al > -5.0) & (al < 5.0)).float()
        return (dx, ddt, dA_log.to(A_log.dtype), dB.to(Bm.dtype), dC.to(Cm.dtype), dD.to(D.dtype),
                dz if ctx.has_z else None, None, None, None)


def _scan_ok(x, N):
    return N in (32, 64, 128) and x.dtype in (torch.float32, torch.bfloat16)


@_register("mamba_inner", "csrc/selective_scan.cu")
def mamba_inner(x_act, dt_raw, A_log, Bm, Cm, D, z, need_h_states, return_final=False):
    if not _scan_ok(x_act, Bm.shape[-1]):
        from mamformer_b200.ops import reference
        return reference.mamba_inner(x_act, dt_raw, A_log, Bm, Cm, D, z, need_h_states, return_final=return_final)
    dt_raw = dt_raw if dt_raw.stride(-1) == 1 else dt_raw.contiguous()
    y, hs, fin = _Scan.apply(x_act, dt_raw, A_log, Bm, Cm, D, z, True, need_h_states, return_final)
    return y, hs, fin


@_register("selective_scan", "csrc/selective_scan.cu")
def selective_scan(x, dt, A_log, B, C, D, return_h_states=False, return_final_state=False):
    if not _scan_ok(x, B.shape[-1]):
        from mamformer_b200.ops import reference
        return reference.selective_scan(x, dt, A_log, B, C, D, return_h_states, return_final_state)
    y, hs, fin = _Scan.apply(x, dt, A_log, B, C, D, None, False, return_h_states, return_final_state)
    out = [y]
    if return_h_states:
        out.append(hs)
    if return_final_state:
        out.append(fin)
    return out[0] if len(out) == 1 else tuple(out)


# ---------------------------------------------------------------------------------------------
@_register("moe_routed", "csrc/gemm_tcgen05.cu (grouped) + ops/moe.py")
def moe_routed(x, idx, gates, w_gate, w_up, w_down):
    from mamformer_b200.ops import moe
    if not moe.supported(x, w_gate):
        from mamformer_b200.ops import reference
        return reference.moe_routed(x, idx, gates, w_gate, w_up, w_down)
    return moe.routed(x, idx, gates, w_gate, w_up, w_down)


@_register("linear_cross_entropy", "csrc/cross_entropy.cu + csrc/gemm_tcgen05.cu")
def linear_cross_entropy(h, weight, labels, ignore_index=-100):
    from mamformer_b200.ops import linear_ce
    if not linear_ce.supported(h, weight):
        from mamformer_b200.ops import reference
        return reference.linear_cross_entropy(h, weight, labels, ignore_index)
    return linear_ce.linear_cross_entropy(h, weight, labels, ignore_index)


@_register("moe_expert_outputs", "csrc/gemm_tcgen05.cu (grouped) + ops/moe.py")
def moe_expert_outputs(x, idx, w_gate, w_up, w_down):
    from mamformer_b200.ops import moe
    if not moe.supported(x, w_gate):
        from mamformer_b200.ops import reference
        return reference.moe_expert_outputs(x, idx, w_gate, w_up, w_down)
    return moe.expert_outputs(x, idx, w_gate, w_up, w_down)


# ---------------------------------------------------------------------------------------------
class _LinearDiffAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q1, q2, k, v, lam, kernel_dim):
        out, S, z = _C.linear_attn_fwd(q1, q2, k, v, lam, int(kernel_dim))
        ctx.save_for_backward(q1, q2, k, v, lam, S, z)
        ctx.kernel_dim = int(kernel_dim)
        return out

    @staticmethod
    def backward(ctx, dout):
        q1, q2, k, v, lam, S, z = ctx.saved_tensors
        dq1, dq2, dk, dv, dlam = _C.linear_attn_bwd(q1, q2, k, v, lam, ctx.kernel_dim, S, z,
                                                    dout.to(q1.dtype).contiguous())
        return dq1, dq2, dk, dv, dlam.to(lam.dtype), None


def _la_ok(q1, k, kernel_dim):
    hd = q1.shape[-1]
    return (q1.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and q1.dim() == 4
            and (kernel_dim, hd) in ((128, 128), (64, 128), (64, 64)) and q1.shape[2] % k.shape[2] == 0)


@_register("linear_diff_attention", "csrc/linear_attn.cu")
def linear_diff_attention(q1, q2, k, v, lam, kernel_dim, chunk=256, state=None, return_state=False):
    if state is not None or return_state or not _la_ok(q1, k, kernel_dim):
        from mamformer_b200.ops import reference
        return reference.linear_diff_attention(q1, q2, k, v, lam, kernel_dim, chunk, state=state,
                                               return_state=return_state)
    return _LinearDiffAttn.apply(q1.contiguous(), q2.contiguous(), k.contiguous(), v.contiguous(), lam,
                                 kernel_dim)


# ---------------------------------------------------------------------------------------------
class _RouterTopK(torch.autograd.Function):
    @staticmethod
    def forward(ctx, scores, k):
        gates, idx, _ = _C.router_topk(scores.float().contiguous(), int(k))
        ctx.save_for_backward(gates, idx)
        ctx.E = scores.shape[1]
        ctx.dtype = scores.dtype
        ctx.mark_non_differentiable(idx)
        return gates, idx

    @staticmethod
    def backward(ctx, dg, didx):
        gates, idx = ctx.saved_tensors
        return _C.router_topk_bwd(dg, gates, idx, ctx.E).to(ctx.dtype), None


@_register("router_topk", "csrc/router.cu")
def router_topk(scores, k):
    if scores.dim() != 2 or scores.shape[1] > 256 or k > 16:
        from mamformer_b200.ops import reference
        return reference.router_topk(scores, k)
    return _RouterTopK.apply(scores, k)


@_register("expert_histogram", "csrc/router.cu")
def expert_histogram(idx, n_experts):
    return _C.expert_histogram(idx, int(n_experts))


# ---------------------------------------------------------------------------------------------
_BIG = 1 << 30


class _FlashAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, lo, hi, scale):
        out, lse = _C.flash_attn_fwd(q, k, v, int(lo), int(hi), float(scale))
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.args = (int(lo), int(hi), float(scale))
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        return (*_attn_bwd(q, k, v, out, lse, dout, ctx.args), None, None, None)


def _attn_bwd(q, k, v, out, lse, dout, args):
    """(dq, dk, dv) of softmax attention: the tcgen05 backward (csrc/flash_tc_bwd.cu) at head_dim
    128 in bf16, else the mma.sync kernels of csrc/flash_attn.cu."""
    dout = dout.to(q.dtype).contiguous()
    if _tc_bwd_ok(q, k):
        return tuple(_C.flash_tc_bwd(q, None, k, v, out, None, lse, None, dout, None, *args))
    return tuple(_C.flash_attn_bwd(q, k, v, out, lse, dout, *args))


class _FlashTCPair(torch.autograd.Function):
    """GQA attention with the forward on the tcgen05 kernel (two query heads of one KV head per
    CTA, csrc/flash_tc.cu) and the backward on the tcgen05 backward (csrc/flash_tc_bwd.cu)."""

    @staticmethod
    def forward(ctx, q, k, v, lo, hi, scale):
        out, lse = _C.flash_tc_fwd(q, None, k, v, None, int(lo), int(hi), float(scale))
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.args = (int(lo), int(hi), float(scale))
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        return (*_attn_bwd(q, k, v, out, lse, dout, ctx.args), None, None, None)


class _DiffFlashTC(torch.autograd.Function):
    """Differential attention: one tcgen05 forward for both softmax maps (shared K / V stream,
    lambda combine in the epilogue); backward = one tcgen05 backward over both maps (shared K / V,
    dK and dV of the two maps summed in tensor memory) with dO1 = dout / (1 - lam + 1e-8) and
    dO2 = -lam dout / (1 - lam + 1e-8) applied as per-head factors inside the kernel, and
    d lam = sum dout . (o1 - (1 + 1e-8) o2) / (1 - lam + 1e-8)^2, with o1 - o2 taken from the
    forward kernel's fp32 difference (the two maps are close, so bf16 copies would lose it)."""

    @staticmethod
    def forward(ctx, q1, q2, k, v, lam, lo, hi, scale):
        lam32 = lam.detach().float().contiguous()
        out, o1, o2, lse1, lse2, od = _C.flash_tc_fwd(q1, q2, k, v, lam32, int(lo), int(hi), float(scale))
        ctx.save_for_backward(q1, q2, k, v, o1, o2, lse1, lse2, lam32, od)
        ctx.args = (int(lo), int(hi), float(scale))
        ctx.lam_dtype = lam.dtype
        return out

    @staticmethod
    def backward(ctx, dout):
        q1, q2, k, v, o1, o2, lse1, lse2, lam, od = ctx.saved_tensors
        den = 1.0 / (1.0 - lam + 1e-8)                               # (H,)
        d32 = dout.float()
        if _TC_BWD:
            coef = torch.stack([den, -lam * den]).contiguous()
            dq1, dq2, dk, dv = _C.flash_tc_bwd(q1, q2, k, v, o1, o2, lse1, lse2, dout.to(q1.dtype).contiguous(),
                                               coef, *ctx.args)
        else:
            do1 = (d32 * den.view(1, 1, -1, 1)).to(q1.dtype).contiguous()
            do2 = (d32 * (-lam * den).view(1, 1, -1, 1)).to(q1.dtype).contiguous()
            dq1, dk1, dv1 = _C.flash_attn_bwd(q1, k, v, o1, lse1, do1, *ctx.args)
            dq2, dk2, dv2 = _C.flash_attn_bwd(q2, k, v, o2, lse2, do2, *ctx.args)
            dk, dv = dk1 + dk2, dv1 + dv2
        # in place on the fp32 copy of dout (never on dout itself, which autograd may share with
        # other branches); od is promoted element by element
        prod = d32 if d32.data_ptr() != dout.data_ptr() else d32.clone()
        dlam = prod.mul_(od).sum(dim=(0, 1, 3)) * den * den    # the 1e-8 o2 term is below fp32 noise
        return dq1, dq2, dk, dv, dlam.to(ctx.lam_dtype), None, None, None


_TC_ATTN = os.environ.get("MAMF_FLASH_TC", "1") != "0"
# MAMF_FLASH_TC_BWD=0 keeps the tcgen05 forward but runs the backward on csrc/flash_attn.cu
_TC_BWD = _TC_ATTN and os.environ.get("MAMF_FLASH_TC_BWD", "1") != "0"


def _tc_ok(q, k):
    return (_TC_ATTN and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and q.shape[-1] == 128
            and k.shape[-1] == 128 and q.shape[2] % k.shape[2] == 0 and q.shape[1] <= k.shape[1])


def _tc_bwd_ok(q, k):
    return _TC_BWD and _tc_ok(q, k)


def _fa_ok(q, k):
    return q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and q.shape[-1] in (64, 128) \
        and q.shape[2] % k.shape[2] == 0


def flash_attention(q, k, v, lo=-_BIG, hi=0, scale=None):
    """softmax(q k^T * scale) v over keys with lo <= key - query position <= hi; (B, S, H, hd)."""
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    return _FlashAttn.apply(q.contiguous(), k.contiguous(), v.contiguous(), lo, hi, scale)


@_register("attention", "csrc/flash_tc.cu + csrc/flash_tc_bwd.cu + csrc/flash_attn.cu")
def attention(q, k, v, lo, hi):
    if not _fa_ok(q, k):
        from mamformer_b200.ops import reference
        return reference.attention_band(q, k, v, lo, hi)
    if _tc_ok(q, k) and (q.shape[2] // k.shape[2]) % 2 == 0:
        return _FlashTCPair.apply(q.contiguous(), k.contiguous(), v.contiguous(), lo, hi, q.shape[-1] ** -0.5)
    return flash_attention(q, k, v, lo, hi)


@_register("diff_attention", "csrc/flash_tc.cu + csrc/flash_tc_bwd.cu + csrc/flash_attn.cu")
def diff_attention(q1, q2, k, v, lam, lo, hi, scale=None):
    """(softmax(q1 k^T s) - lam softmax(q2 k^T s)) v / (1 - lam): at head_dim 128 one tcgen05
    forward over a shared K / V stream; otherwise two flash passes combined."""
    if not _fa_ok(q1, k):
        from mamformer_b200.ops import reference
        return reference.diff_attention_band(q1, q2, k, v, lam, lo, hi, scale)
    if _tc_ok(q1, k) and lam.numel() == q1.shape[2]:
        sc = q1.shape[-1] ** -0.5 if scale is None else scale
        return _DiffFlashTC.apply(q1.contiguous(), q2.contiguous(), k.contiguous(), v.contiguous(), lam, lo, hi, sc)
    o1 = flash_attention(q1, k, v, lo, hi, scale)
    o2 = flash_attention(q2, k, v, lo, hi, scale)
    lam4 = lam.view(1, 1, -1, 1).to(o1.dtype)
    return (o1 - lam4 * o2) / (1.0 - lam4 + 1e-8)
