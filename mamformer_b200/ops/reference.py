"""PyTorch reference implementations of every hot op (the CPU path and the numerics oracle).

Each function restates the reference framework's math for one op, in plain PyTorch, with the
same dtype behaviour as the reference where that matters for loss-curve parity:

* ``selective_scan``         - reference ``mamformer/layers/mamba2.py:70-130`` (sequential scan,
                               A_log clamped to [-5, 5], h_states = mean over channels).
* ``linear_diff_attention``  - reference ``kda_diff.py:357-478`` (chunked causal linear attention,
                               phi = elu+1 on the first kernel_dim dims, bf16 intermediates when
                               the input is fp32, fp32 carried state, eps 1e-8 normaliser).
* ``diff_attention``         - reference ``kda_diff.py:826-862`` (two softmaxes, causal mask with
                               finfo.min, sliding-window mask with -inf, (A1 - lam A2)/(1-lam+1e-8)).
* ``sdpa_attention``         - reference ``attention.py:157-181`` (GQA softmax attention).
* ``router_topk``            - reference ``moe.py:163-183`` (top-k on scores, softmax over top-k).
* ``moe_routed``             - reference ``moe.py:310-332`` (gate-weighted sum of SwiGLU experts).

Layouts: attention tensors are (B, S, H, hd) ("bshd"); GQA is by index (head h uses kv head
h // (H / H_kv)), which equals the reference's ``repeat_interleave``.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


# ---------------------------------------------------------------------------------------------
# norms / elementwise
# ---------------------------------------------------------------------------------------------

def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    rms = torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = (xf / rms).to(x.dtype)
    return y * weight if weight.dtype == y.dtype else (y * weight).to(torch.promote_types(y.dtype, weight.dtype))


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x (B, S, H, hd); cos/sin (S, hd/2) fp32.  Half-split rotation."""
    half = x.shape[-1] // 2
    c = cos[None, :, None, :].to(x.dtype)
    s = sin[None, :, None, :].to(x.dtype)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return F.silu(gate) * up


def causal_conv1d(x: torch.Tensor, weight: torch.Tensor,
                  state: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Depthwise causal conv over time.  x (B, S, C), weight (C, K), state (B, K-1, C) or None."""
    K = weight.shape[-1]
    if state is not None:
        xp = torch.cat([state.to(x.dtype), x], 1)
    else:
        xp = F.pad(x, (0, 0, K - 1, 0))
    y = F.conv1d(xp.transpose(1, 2), weight.to(x.dtype).unsqueeze(1), groups=x.shape[-1])
    return y[:, :, -x.shape[1]:].transpose(1, 2).contiguous()


def head_group_norm(x: torch.Tensor, n_heads: int, weight: torch.Tensor, bias: torch.Tensor,
                    eps: float) -> torch.Tensor:
    """GroupNorm with one group per head over (head_dim x S), per sample.

    x is (B, S, H*hd).  Equals ``nn.GroupNorm(H, H*hd)`` applied to ``x.transpose(1, 2)``
    (reference ``kda_diff.py:345-348``)."""
    y = F.group_norm(x.transpose(1, 2), n_heads, weight, bias, eps)
    return y.transpose(1, 2)


# ---------------------------------------------------------------------------------------------
# selective scan
# ---------------------------------------------------------------------------------------------

def selective_scan(x, dt, A_log, B, C, D, return_h_states=False, return_final_state=False,
                   h0: Optional[torch.Tensor] = None, clamp_a: bool = True):
    """h_t = exp(-exp(A) dt_t) h_{t-1} + B_t dt_t x_t ;  y_t = C_t . h_t + D x_t.

    x, dt: (B, S, Di); A_log: (N,); B, C: (B, S, N); D: (Di,).  Returns y and optionally
    h_states (B, S, N) = mean over Di of h_t, and the final state (B, Di, N)."""
    bsz, S, Di = x.shape
    N = A_log.shape[0]
    A = torch.exp(A_log.clamp(-5.0, 5.0) if clamp_a else A_log)
    dte = dt.unsqueeze(-1)
    a = torch.exp(-A.view(1, 1, 1, N) * dte)
    u = (B.unsqueeze(2) * dte) * x.unsqueeze(-1)
    h = torch.zeros(bsz, Di, N, dtype=x.dtype, device=x.device) if h0 is None else h0.to(x.dtype)
    ys = []
    hs = [] if return_h_states else None
    for t in range(S):
        h = a[:, t] * h + u[:, t]
        ys.append((C[:, t].unsqueeze(1) * h).sum(-1))
        if hs is not None:
            hs.append(h.mean(1))
    y = torch.stack(ys, 1) + D.view(1, 1, Di) * x
    out = [y]
    if return_h_states:
        out.append(torch.stack(hs, 1))
    if return_final_state:
        out.append(h)
    return out[0] if len(out) == 1 else tuple(out)


def mamba_inner(x_act, dt_raw, A_log, Bm, Cm, D, z, need_h_states, h0=None,
                return_final=False):
    """Softplus(dt) -> selective scan -> y * silu(z).  Returns (y_gated, h_states|None, final|None)."""
    dt = F.softplus(dt_raw)
    res = selective_scan(x_act, dt, A_log, Bm, Cm, D, return_h_states=need_h_states,
                         return_final_state=return_final, h0=h0)
    if not isinstance(res, tuple):
        res = (res,)
    y = res[0]
    i = 1
    hs = None
    if need_h_states:
        hs = res[i]
        i += 1
    final = res[i] if return_final else None
    return y * F.silu(z), hs, final


# ---------------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------------

def _expand_kv(t: torch.Tensor, groups: int) -> torch.Tensor:
    return t if groups == 1 else t.repeat_interleave(groups, dim=2)


def kernel_feature_map(x: torch.Tensor, kernel_dim: int) -> torch.Tensor:
    return F.elu(x[..., :kernel_dim]) + 1.0


def linear_diff_attention(q1, q2, k, v, lam, kernel_dim: int, chunk: int = 256,
                          state: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                          return_state: bool = False):
    """Causal linear attention with phi=elu+1 on two queries, combined differentially.

    q1, q2: (B, S, H, hd); k, v: (B, S, Hkv, hd); lam: (H,) already clamped.
    Returns (B, S, H, hd) [, (S_state (B,H,K,hd) fp32, z_state (B,H,K) fp32)]."""
    bsz, S, H, hd = q1.shape
    groups = H // k.shape[2]
    kx = _expand_kv(k, groups).transpose(1, 2)
    vx = _expand_kv(v, groups).transpose(1, 2)
    q1t, q2t = q1.transpose(1, 2), q2.transpose(1, 2)
    K = kernel_dim
    cd = torch.bfloat16 if q1.dtype == torch.float32 else q1.dtype
    p1 = kernel_feature_map(q1t, K).to(cd)
    p2 = kernel_feature_map(q2t, K).to(cd)
    pk = kernel_feature_map(kx, K).to(cd)
    if state is not None:
        S_state, z_state = state[0].float().clone(), state[1].float().clone()
    else:
        S_state = torch.zeros(bsz, H, K, hd, device=q1.device, dtype=torch.float32)
        z_state = torch.zeros(bsz, H, K, device=q1.device, dtype=torch.float32)
    o1s, o2s = [], []
    for s0 in range(0, S, chunk):
        s1 = min(S, s0 + chunk)
        L = s1 - s0
        kc, vc = pk[:, :, s0:s1], vx[:, :, s0:s1].to(cd)
        q1c, q2c = p1[:, :, s0:s1], p2[:, :, s0:s1]
        kv = torch.bmm(kc.reshape(-1, K, 1), vc.reshape(-1, 1, hd)).reshape(bsz, H, L, K, hd)
        kv_cum = kv.cumsum(2) + S_state.unsqueeze(2).to(cd)
        k_cum = kc.cumsum(2) + z_state.unsqueeze(2).to(cd)
        kvf = kv_cum.reshape(-1, K, hd)
        o1 = torch.bmm(q1c.reshape(-1, 1, K), kvf).reshape(bsz, H, L, hd)
        o2 = torch.bmm(q2c.reshape(-1, 1, K), kvf).reshape(bsz, H, L, hd)
        kcf = k_cum.reshape(-1, K, 1)
        n1 = torch.bmm(q1c.reshape(-1, 1, K), kcf).reshape(bsz, H, L)
        n2 = torch.bmm(q2c.reshape(-1, 1, K), kcf).reshape(bsz, H, L)
        o1s.append((o1 / (n1.unsqueeze(-1) + 1e-8)).to(q1.dtype))
        o2s.append((o2 / (n2.unsqueeze(-1) + 1e-8)).to(q1.dtype))
        S_state = S_state + kv.sum(2).float()
        z_state = z_state + kc.sum(2).float()
    o1 = torch.cat(o1s, 2)
    o2 = torch.cat(o2s, 2)
    lam4 = lam.view(1, H, 1, 1).to(o1.dtype)
    out = ((o1 - lam4 * o2) / (1.0 - lam4 + 1e-8)).transpose(1, 2)
    if return_state:
        return out, (S_state, z_state)
    return out


def linear_diff_attention_fp32(q1, q2, k, v, lam, kernel_dim: int):
    """Exact fp32 form of the same operator (oracle for the native kernel's numerics)."""
    bsz, S, H, hd = q1.shape
    groups = H // k.shape[2]
    kx = _expand_kv(k, groups).float()
    vx = _expand_kv(v, groups).float()
    p1 = kernel_feature_map(q1.float(), kernel_dim)
    p2 = kernel_feature_map(q2.float(), kernel_dim)
    pk = kernel_feature_map(kx, kernel_dim)
    mask = torch.ones(S, S, device=q1.device).tril()
    out = []
    for p in (p1, p2):
        att = torch.einsum("bshk,bthk->bhst", p, pk) * mask
        num = torch.einsum("bhst,bthd->bshd", att, vx)
        den = att.sum(-1).transpose(1, 2).unsqueeze(-1)
        out.append(num / (den + 1e-8))
    lam4 = lam.view(1, 1, H, 1).float()
    return (out[0] - lam4 * out[1]) / (1.0 - lam4 + 1e-8)


def _masked_logits(q, k, scale, window: int, causal: bool, kv_offset: int,
                   attention_mask: Optional[torch.Tensor]):
    logits = torch.matmul(q, k.transpose(-2, -1)) * scale
    qlen, kvlen = q.shape[-2], k.shape[-2]
    if attention_mask is not None:
        logits = logits + attention_mask
    elif causal:
        cm = torch.triu(torch.full((qlen, kvlen), torch.finfo(logits.dtype).min,
                                   device=q.device, dtype=logits.dtype),
                        diagonal=kvlen - qlen + 1)
        logits = logits + cm
    if window > 0:
        iq = torch.arange(qlen, device=q.device).unsqueeze(1)
        ik = torch.arange(kvlen, device=q.device).unsqueeze(0)
        dist = ik - iq
        valid = (dist >= 0) & (dist < window)
        logits = logits + torch.zeros(qlen, kvlen, device=q.device, dtype=logits.dtype).masked_fill(
            ~valid, float("-inf"))
    return logits


def diff_attention(q1, q2, k, v, lam, window: int = 0, causal: bool = True,
                   scale: Optional[float] = None, attention_mask: Optional[torch.Tensor] = None):
    """(softmax(Q1 K^T s + M) - lam softmax(Q2 K^T s + M)) V / (1 - lam + 1e-8).

    Inputs bshd; k/v may carry a prefix (cache): queries align to the last positions.
    The sliding-window mask follows the reference exactly (distance measured as
    key_index - query_index without the cache offset, reference ``kda_diff.py:875-886``)."""
    H, hd = q1.shape[2], q1.shape[3]
    groups = H // k.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    kx = _expand_kv(k, groups).transpose(1, 2)
    vx = _expand_kv(v, groups).transpose(1, 2)
    l1 = _masked_logits(q1.transpose(1, 2), kx, scale, window, causal, 0, attention_mask)
    l2 = _masked_logits(q2.transpose(1, 2), kx, scale, window, causal, 0, attention_mask)
    lam4 = lam.view(1, H, 1, 1).to(l1.dtype)
    w = (F.softmax(l1, -1) - lam4 * F.softmax(l2, -1)) / (1.0 - lam4 + 1e-8)
    return torch.matmul(w, vx).transpose(1, 2)


def sdpa_attention(q, k, v, window: int = 0, attention_mask: Optional[torch.Tensor] = None,
                   dropout_p: float = 0.0):
    """GQA softmax attention with the reference's masking rules (``attention.py:157-181``)."""
    H = q.shape[2]
    groups = H // k.shape[2]
    qt = q.transpose(1, 2)
    kt = _expand_kv(k, groups).transpose(1, 2)
    vt = _expand_kv(v, groups).transpose(1, 2)
    qlen, kvlen = qt.shape[-2], kt.shape[-2]
    mask = attention_mask
    if window > 0:
        iq = torch.arange(qlen, device=q.device).unsqueeze(1)
        ik = torch.arange(kvlen, device=q.device).unsqueeze(0)
        dist = ik - iq
        valid = (dist >= 0) & (dist < window)
        sw = torch.zeros(qlen, kvlen, device=q.device, dtype=q.dtype).masked_fill(~valid, float("-inf"))
        if mask is not None:
            if mask.dtype == torch.bool:
                mask = mask.float().masked_fill(~mask, float("-inf"))
            mask = torch.minimum(mask, sw)
        else:
            mask = sw
    if mask is not None:
        o = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask, dropout_p=dropout_p)
    else:
        o = F.scaled_dot_product_attention(qt, kt, vt, dropout_p=dropout_p, is_causal=True)
    return o.transpose(1, 2)


# ---------------------------------------------------------------------------------------------
# MoE
# ---------------------------------------------------------------------------------------------

def router_topk(scores: torch.Tensor, k: int):
    vals, idx = torch.topk(scores, k, dim=-1)
    return F.softmax(vals, dim=-1), idx


def moe_routed(x, idx, gates, w_gate, w_up, w_down):
    """sum_k gate_k * down_e(silu(gate_e x) * up_e x) over the top-k experts e = idx[:, k].

    x: (T, d); idx, gates: (T, k); w_gate/w_up: (E, I, d); w_down: (E, d, I)."""
    T, d = x.shape
    E = w_gate.shape[0]
    out = torch.zeros(T, d, dtype=x.dtype, device=x.device)
    for e in range(E):
        hit = idx == e
        rows = hit.any(-1)
        if not bool(rows.any()):
            continue
        tok = rows.nonzero(as_tuple=True)[0]
        slot = hit[rows].float().argmax(-1)
        xe = x[tok]
        h = F.silu(xe @ w_gate[e].t().to(x.dtype)) * (xe @ w_up[e].t().to(x.dtype))
        ye = h @ w_down[e].t().to(x.dtype)
        out.index_add_(0, tok, ye * gates[tok, slot].unsqueeze(-1).to(ye.dtype))
    return out


def moe_expert_outputs(x, idx, w_gate, w_up, w_down):
    """Unweighted per-slot expert outputs (T, k, d) (reference ``communicative_moe.py:341-391``)."""
    T, k = idx.shape
    out = torch.zeros(T, k, x.shape[1], dtype=x.dtype, device=x.device)
    for e in range(w_gate.shape[0]):
        tok, slot = (idx == e).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        xe = x[tok]
        h = F.silu(xe @ w_gate[e].t().to(x.dtype)) * (xe @ w_up[e].t().to(x.dtype))
        out[tok, slot] = h @ w_down[e].t().to(x.dtype)
    return out


# ---------------------------------------------------------------------------------------------
# loss
# ---------------------------------------------------------------------------------------------

def linear_cross_entropy(h: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                         ignore_index: int = -100) -> torch.Tensor:
    """mean CE of softmax(h W^T) against labels over non-ignored rows.  h (T, d), W (V, d)."""
    logits = F.linear(h, weight.to(h.dtype))
    return F.cross_entropy(logits.float() if logits.dtype != torch.float32 else logits,
                           labels, ignore_index=ignore_index)


def _band_mask(S, Skv, lo, hi, device, dtype):
    iq = torch.arange(S, device=device).unsqueeze(1) + (Skv - S)
    ik = torch.arange(Skv, device=device).unsqueeze(0)
    dist = ik - iq
    ok = (dist >= lo) & (dist <= hi)
    return torch.zeros(S, Skv, device=device, dtype=dtype).masked_fill(~ok, float("-inf"))


def attention_band(q, k, v, lo, hi, scale=None):
    """GQA softmax attention over keys with lo <= key - query position <= hi (bshd)."""
    groups = q.shape[2] // k.shape[2]
    qt = q.transpose(1, 2).float()
    kt = _expand_kv(k, groups).transpose(1, 2).float()
    vt = _expand_kv(v, groups).transpose(1, 2).float()
    s = (qt @ kt.transpose(-1, -2)) * (q.shape[-1] ** -0.5 if scale is None else scale)
    s = s + _band_mask(q.shape[1], k.shape[1], lo, hi, q.device, s.dtype)
    p = torch.softmax(s, -1).nan_to_num(0.0)
    return (p @ vt).transpose(1, 2).to(q.dtype)


def diff_attention_band(q1, q2, k, v, lam, lo, hi, scale=None):
    o1 = attention_band(q1, k, v, lo, hi, scale)
    o2 = attention_band(q2, k, v, lo, hi, scale)
    lam4 = lam.view(1, 1, -1, 1).to(o1.dtype)
    return (o1 - lam4 * o2) / (1.0 - lam4 + 1e-8)
