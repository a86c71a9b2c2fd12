"""Micro-benchmarks of the native kernels at the shapes of the ultra-7b bench workload.

    python -m mamformer_b200.utils.kernel_bench --op gemm [--iters 20]
    python -m mamformer_b200.utils.kernel_bench --op scan --once     # one launch (profiler capture)

Each case builds its inputs once on the GPU, warms up, and times ``--iters`` launches with CUDA
events on the launching stream (synchronised on both sides).  Inputs are larger than the 126 MB
L2 where the kernel is memory-bound; for the GEMMs the operands are re-read from L2 by design.
The report gives the achieved rate and its fraction of the measured peaks
(``MEASURED_PEAKS.json``: copy bandwidth, cuBLAS bf16 GEMM throughput).  ``--once`` runs one
warm-up and exactly one launch of the case, for a profiler that captures a single kernel.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"]
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0


def case_gemm(d=4096, V=128000, T=4096):
    """CE logits GEMM: (T, d) x (V, d)^T -> (T, V) bf16."""
    from mamformer_b200.ops import gemm
    h = torch.randn(T, d, device="cuda").bfloat16()
    W = torch.randn(V, d, device="cuda").bfloat16() * 0.02
    out = torch.empty(T, V, device="cuda", dtype=torch.bfloat16)
    return (lambda: gemm.mm(h, W, out=out)), 2.0 * T * V * d, (T * d + V * d + T * V) * 2


def case_grouped(E=128, k=8, T=4096, d=4096, I=576):
    """MoE up-projection: grouped-M GEMM over 128 experts (balanced)."""
    from mamformer_b200.ops import gemm
    from mamformer_b200.ops.moe import plan
    idx = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)])
    pos, seg, tile_off, _, rows = plan(idx, E)
    x = torch.randn(rows, d, device="cuda").bfloat16()
    w = torch.randn(E, I, d, device="cuda").bfloat16() * 0.02
    out = torch.empty(rows, I, device="cuda", dtype=torch.bfloat16)
    return (lambda: gemm.grouped_mm(x, w, seg, tile_off, out=out)), 2.0 * T * k * I * d, (rows * d + E * I * d + rows * I) * 2


def case_wgrad(E=128, k=8, T=16384, d=4096, I=576):
    """MoE weight gradient: grouped-K GEMM accumulated into the fp32 optimizer buffer (the
    epilogue's bulk tensor reduce-add), micro-batch of 4 x 4096 tokens, 128 experts."""
    from mamformer_b200.ops import gemm
    from mamformer_b200.ops.moe import plan
    idx = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)])
    pos, seg, tile_off, _, rows = plan(idx, E)
    dy = torch.randn(rows, I, device="cuda").bfloat16()
    x = torch.randn(rows, d, device="cuda").bfloat16()
    dw = torch.zeros(E, I, d, device="cuda")
    return (lambda: gemm.grouped_wgrad(dy, x, seg, dw, accumulate=True)), 2.0 * T * k * I * d, \
        (rows * (I + d)) * 2 + E * I * d * 4 * 2


def case_scan(B=1, S=4096, D=8192, N=128, backward=False):
    """Selective scan (Mamba block of ultra-7b: d_inner 8192, d_state 128), fused gate."""
    from mamformer_b200.ops.native import _C
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(B, S, D, device="cuda", generator=g).bfloat16()
    dt = (torch.randn(B, S, D, device="cuda", generator=g) * 0.5 - 2).bfloat16()
    A = torch.log(torch.linspace(0.5, 8, N, device="cuda"))
    Bm = torch.randn(B, S, N, device="cuda", generator=g).bfloat16()
    Cm = torch.randn(B, S, N, device="cuda", generator=g).bfloat16()
    Dv = torch.ones(D, device="cuda")
    z = torch.randn(B, S, D, device="cuda", generator=g).bfloat16()
    y, hs, ck, fin = _C.selective_scan_fwd(x, dt, A, Bm, Cm, Dv, z, None, True, True, False)
    io = (4 * B * S * D + 2 * B * S * N) * 2
    if not backward:
        return (lambda: _C.selective_scan_fwd(x, dt, A, Bm, Cm, Dv, z, None, True, True, False)), 0.0, io
    dy = torch.randn_like(x)
    dhs = torch.randn_like(hs) if hs is not None else None
    return (lambda: _C.selective_scan_bwd(x, dt, A, Bm, Cm, Dv, z, ck, dy, dhs, True)), 0.0, 2 * io


def case_linear_attn(B=1, S=4096, H=32, G=8, hd=128, backward=False):
    from mamformer_b200.ops.native import _C
    mk = lambda h: (torch.randn(B, S, h, hd, device="cuda") * 0.5).bfloat16()
    q1, q2, k, v = mk(H), mk(H), mk(G), mk(G)
    lam = torch.full((H,), 0.5, device="cuda")
    out, Sst, zst = _C.linear_attn_fwd(q1, q2, k, v, lam, hd)
    C = 64
    flops = 2.0 * B * H * S * (2 * C * hd + 2 * C * hd + 2 * hd * hd) * 2
    io = (3 * B * S * H * hd + 2 * B * S * G * hd) * 2
    if not backward:
        return (lambda: _C.linear_attn_fwd(q1, q2, k, v, lam, hd)), flops, io
    dout = torch.randn_like(out)
    return (lambda: _C.linear_attn_bwd(q1, q2, k, v, lam, hd, Sst, zst, dout)), 2.5 * flops, 2 * io


def case_ce(T=4096, d=4096, V=128000):
    """Fused linear + cross-entropy forward and backward (recompute), tied embedding."""
    from mamformer_b200.ops import linear_ce
    h = (torch.randn(T, d, device="cuda") * 0.5).bfloat16().requires_grad_()
    W = (torch.randn(V, d, device="cuda") * 0.02).bfloat16().requires_grad_()
    W.main_grad = torch.zeros(V, d, device="cuda")
    lab = torch.randint(0, V, (T,), device="cuda")

    def run():
        loss = linear_ce.linear_cross_entropy(h, W, lab)
        loss.backward()
    return run, 4 * 2.0 * T * V * d, 0


def case_moe(T=4096, d=4096, E=128, k=8, I=576):
    """Routed experts forward + backward on one GPU (dispatch, 3 grouped GEMMs, combine)."""
    from mamformer_b200.ops import moe
    x = (torch.randn(T, d, device="cuda") * 0.5).bfloat16().requires_grad_()
    idx = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)])
    gates = torch.softmax(torch.randn(T, k, device="cuda"), -1).requires_grad_()
    ws = [(torch.randn(*s, device="cuda") * 0.02).bfloat16().requires_grad_() for s in ((E, I, d), (E, I, d), (E, d, I))]
    for w in ws:
        w.main_grad = torch.zeros(w.shape, device="cuda")

    def run():
        out = moe.routed(x, idx, gates, *ws)
        out.backward(torch.ones_like(out))
    return run, 3 * 3 * 2.0 * T * k * d * I, 0


def case_adamw(n=1 << 28):
    """Fused AdamW over a 2^28-element fp32 segment with a bf16 copy (the optimizer step)."""
    from mamformer_b200.ops.native import _C
    p, g, m, v = (torch.randn(n, device="cuda") for _ in range(4))
    v.abs_()
    low = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    scale = torch.ones(1, device="cuda")
    return (lambda: _C.adamw_step(p, g, m, v, low, 1e-4, 0.9, 0.95, 1e-8, 0.1, 1, scale)), 0.0, n * (4 * 7 + 2)


def case_flash_attn(B=1, S=4096, H=32, G=8, hd=128, backward=False):
    """Causal GQA softmax attention of the ultra-7b full-attention layer (32 query / 8 KV heads)."""
    from mamformer_b200.ops.native import _C
    mk = lambda h: (torch.randn(B, S, h, hd, device="cuda") * 0.5).bfloat16()
    q, k, v = mk(H), mk(G), mk(G)
    lo, hi, scale = -(1 << 30), 0, hd ** -0.5
    flops = 4.0 * B * H * S * S * hd / 2          # causal: half of the S x S scores
    if not backward:
        return (lambda: _C.flash_attn_fwd(q, k, v, lo, hi, scale)), flops, 0
    out, lse = _C.flash_attn_fwd(q, k, v, lo, hi, scale)
    dout = torch.randn_like(out)
    return (lambda: _C.flash_attn_bwd(q, k, v, out, lse, dout, lo, hi, scale)), 2.5 * flops, 0


def case_flash_tc(B=1, S=4096, H=32, G=8, hd=128, diff=False):
    """tcgen05 flash forward (csrc/flash_tc.cu), causal, 32 query / 8 KV heads: GQA head pairs, or
    the differential form (two query tensors, one shared K / V stream, lambda combine)."""
    from mamformer_b200.ops.native import _C
    mk = lambda h: (torch.randn(B, S, h, hd, device="cuda") * 0.5).bfloat16()  # noqa: E731
    q, q2, k, v = mk(H), mk(H), mk(G), mk(G)
    lo, hi, scale = -(1 << 30), 0, hd ** -0.5
    flops = 4.0 * B * H * S * S * hd / 2 * (2 if diff else 1)
    if diff:
        lam = torch.full((H,), 0.5, device="cuda")
        return (lambda: _C.flash_tc_fwd(q, q2, k, v, lam, lo, hi, scale)), flops, 0
    return (lambda: _C.flash_tc_fwd(q, None, k, v, None, lo, hi, scale)), flops, 0


def case_flash_tc_bwd(B=1, S=4096, H=32, G=8, hd=128, diff=False):
    """tcgen05 flash backward (csrc/flash_tc_bwd.cu), causal, 32 query / 8 KV heads; the
    differential form runs both maps in one launch (shared K / V, dK / dV summed in TMEM).
    FLOPs: 2.5 x the forward's (S^T, dP^T, dV, dK, dQ products vs S and PV)."""
    from mamformer_b200.ops.native import _C
    mk = lambda h: (torch.randn(B, S, h, hd, device="cuda") * 0.5).bfloat16()  # noqa: E731
    q, q2, k, v = mk(H), mk(H), mk(G), mk(G)
    lo, hi, scale = -(1 << 30), 0, hd ** -0.5
    flops = 2.5 * 4.0 * B * H * S * S * hd / 2 * (2 if diff else 1)
    if diff:
        lam = torch.full((H,), 0.5, device="cuda")
        out, o1, o2, l1, l2, _ = _C.flash_tc_fwd(q, q2, k, v, lam, lo, hi, scale)
        dout = torch.randn_like(out)
        coef = torch.stack([1 / (1 - lam), -lam / (1 - lam)])
        return (lambda: _C.flash_tc_bwd(q, q2, k, v, o1, o2, l1, l2, dout, coef, lo, hi, scale)), flops, 0
    out, lse = _C.flash_tc_fwd(q, None, k, v, None, lo, hi, scale)
    dout = torch.randn_like(out)
    return (lambda: _C.flash_tc_bwd(q, None, k, v, out, None, lse, None, dout, None, lo, hi, scale)), flops, 0


def case_router(T=4096, E=128, k=8):
    """Router top-k + softmax over the selected scores + per-expert histogram."""
    from mamformer_b200.ops.native import _C
    scores = torch.randn(T, E, device="cuda")
    return (lambda: _C.router_topk(scores, k)), 0.0, T * E * 4 + T * k * 12


def case_rmsnorm(T=16384, d=4096, backward=False):
    """RMSNorm over 4 micro-batch sequences of 4096 tokens at d_model 4096 (bf16 in / out)."""
    from mamformer_b200.ops.native import _C
    x = torch.randn(T, d, device="cuda").bfloat16()
    w = torch.ones(d, device="cuda")
    if not backward:
        return (lambda: _C.rmsnorm_fwd(x, w, 1e-6)), 0.0, 2 * T * d * 2 + T * 4
    _, rstd = _C.rmsnorm_fwd(x, w, 1e-6)
    dy = torch.randn_like(x)
    return (lambda: _C.rmsnorm_bwd(x, w, dy, rstd)), 0.0, 3 * T * d * 2 + T * 4


def case_swiglu(T=16384, I=4608, backward=False):
    """SwiGLU of the two shared experts (intermediate 2 x 2304) over 16384 tokens."""
    from mamformer_b200.ops.native import _C
    g, u = (torch.randn(T, I, device="cuda").bfloat16() for _ in range(2))
    if not backward:
        return (lambda: _C.swiglu_fwd(g, u)), 0.0, 3 * T * I * 2
    dy = torch.randn_like(g)
    return (lambda: _C.swiglu_bwd(g, u, dy)), 0.0, 5 * T * I * 2


def case_rope(B=4, S=4096, H=32, hd=128):
    """Rotary embedding of the 32 query heads (fp32 cos / sin tables of S x hd/2)."""
    from mamformer_b200.ops.native import _C
    x = torch.randn(B, S, H, hd, device="cuda").bfloat16()
    ang = torch.arange(S, device="cuda")[:, None] * torch.rand(hd // 2, device="cuda")[None]
    c, s = ang.cos(), ang.sin()
    return (lambda: _C.rope_apply(x, c, s, False)), 0.0, 2 * x.numel() * 2 + 2 * c.numel() * 4


def case_conv(B=4, S=4096, C=8192, K=4, backward=False):
    """Causal depthwise conv (width 4) + SiLU of the Mamba block, d_inner 8192."""
    from mamformer_b200.ops.native import _C
    x = torch.randn(B, S, C, device="cuda").bfloat16()
    w = torch.randn(C, K, device="cuda") * 0.3
    if not backward:
        return (lambda: _C.conv_silu_fwd(x, w)), 0.0, 2 * x.numel() * 2
    dy = torch.randn_like(x)
    return (lambda: _C.conv_silu_bwd(x, w, dy)), 0.0, 3 * x.numel() * 2


def case_groupnorm(B=4, S=4096, H=32, hd=128, backward=False):
    """Per-head GroupNorm of the KDA-Diff output (32 heads of 128 per token)."""
    from mamformer_b200.ops.native import _C
    x = torch.randn(B, S, H * hd, device="cuda").bfloat16()
    w, b = torch.ones(H * hd, device="cuda"), torch.zeros(H * hd, device="cuda")
    if not backward:
        return (lambda: _C.head_groupnorm_fwd(x, H, w, b, 1e-5)), 0.0, 2 * x.numel() * 2
    _, mr = _C.head_groupnorm_fwd(x, H, w, b, 1e-5)
    dy = torch.randn_like(x)
    return (lambda: _C.head_groupnorm_bwd(x, H, w, mr, dy)), 0.0, 3 * x.numel() * 2


CASES = {"gemm": case_gemm, "grouped": case_grouped, "wgrad": case_wgrad, "scan": case_scan,
         "scan_bwd": lambda: case_scan(backward=True), "linear_attn": case_linear_attn,
         "linear_attn_bwd": lambda: case_linear_attn(backward=True), "ce": case_ce, "moe": case_moe,
         "adamw": case_adamw, "flash_attn": case_flash_attn,
         "flash_attn_bwd": lambda: case_flash_attn(backward=True), "router": case_router,
         "flash_tc": case_flash_tc, "flash_tc_diff": lambda: case_flash_tc(diff=True),
         "flash_tc_bwd": case_flash_tc_bwd, "flash_tc_diff_bwd": lambda: case_flash_tc_bwd(diff=True),
         "rmsnorm": case_rmsnorm, "rmsnorm_bwd": lambda: case_rmsnorm(backward=True),
         "swiglu": case_swiglu, "swiglu_bwd": lambda: case_swiglu(backward=True), "rope": case_rope,
         "conv": case_conv, "conv_bwd": lambda: case_conv(backward=True), "groupnorm": case_groupnorm,
         "groupnorm_bwd": lambda: case_groupnorm(backward=True)}


def run(op: str, iters: int = 20, once: bool = False) -> dict:
    fn, flops, nbytes = CASES[op]()
    fn()
    torch.cuda.synchronize()
    if once:
        fn()
        torch.cuda.synchronize()
        return {"op": op, "launched": 1}
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    hbm, tf = _peaks()
    out = {"op": op, "ms": round(ms, 4)}
    if flops:
        out["tflops"] = round(flops / ms / 1e9, 1)
        out["frac_of_measured_bf16"] = round(flops / ms / 1e9 / tf, 3)
    if nbytes:
        out["gbs"] = round(nbytes / ms / 1e6, 1)
        out["frac_of_measured_hbm"] = round(nbytes / ms / 1e6 / hbm, 3)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--op", default="all", choices=["all"] + list(CASES))
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--once", action="store_true")
    a = ap.parse_args(argv)
    for op in (CASES if a.op == "all" else [a.op]):
        print(json.dumps(run(op, a.iters, a.once)), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
