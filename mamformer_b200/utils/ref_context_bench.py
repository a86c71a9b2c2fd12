"""The reference's own eager hot ops next to this framework's kernels, at the benchmark shapes.

    python -m mamformer_b200.utils.ref_context_bench [--op all|scan|diff_attn|moe] [--ref-dir baseline/_ref]

Context for the headline number, not the benchmark's reference arm: the reference's stock GPU
path stops in its Triton linear-attention kernel, so its full training step has no B200 time;
its other hot ops still run, and each is timed here through the reference's own functions and
modules (imported unmodified from the installed copy) against the op this framework runs in
their place, forward + backward, bf16 autocast for the reference as its training script uses.

* scan      - ``mamformer/layers/mamba2.py`` ``selective_scan`` (Python loop over time,
              ``mamba2.py:109-116``) vs the native selective-scan kernels; d_inner 8192,
              d_state 128, batch 1.  The reference loop runs on a shorter sequence (256 steps:
              its activations grow with S) and both are reported per token.
* diff_attn - ``FullDiffAttention`` (two materialised S x S maps, ``kda_diff.py:826-862``) vs this
              framework's module of the same name (flash kernels); d_model 4096, 32 / 8 heads,
              head_dim 128, latent 512, causal window 4096, batch 1.
* moe       - ``DeepSeekMoE`` (Python loop over 128 experts, ``moe.py:310-332``) vs this
              framework's module (native routing plan + grouped tcgen05 GEMMs); d_model 4096,
              2 shared experts of 2304, 128 routed of 576, top-8.

CUDA events on the current stream, warm-up first, synchronise on both sides.  One JSON line per
op: ``ref_ms``, ``ours_ms`` (per token where the sequence lengths differ), ``speedup``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _time(fn, iters=3, warmup=1):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def _ref_import(ref_dir):
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    sys.dont_write_bytecode = True
    import mamformer  # noqa: F401  (the reference package)
    return mamformer


def case_scan(ref_dir, seq=4096, ref_seq=256, D=8192, N=128):
    _ref_import(ref_dir)
    from mamformer.layers.mamba2 import selective_scan as ref_scan
    from mamformer_b200 import ops

    def inputs(S):
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(1, S, D, device="cuda", generator=g).bfloat16().requires_grad_()
        dt = torch.nn.functional.softplus(torch.randn(1, S, D, device="cuda", generator=g) * 0.5 - 2) \
            .bfloat16().requires_grad_()
        A = torch.log(torch.linspace(0.5, 8, N, device="cuda")).requires_grad_()
        Bm = torch.randn(1, S, N, device="cuda", generator=g).bfloat16().requires_grad_()
        Cm = torch.randn(1, S, N, device="cuda", generator=g).bfloat16().requires_grad_()
        Dv = torch.ones(D, device="cuda").requires_grad_()
        return x, dt, A, Bm, Cm, Dv

    ri = inputs(ref_seq)

    def ref_step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y, hs = ref_scan(*ri, return_h_states=True)
        (y.float().sum() + hs.float().sum()).backward()

    oi = inputs(seq)

    def our_step():
        y, hs = ops.selective_scan(*oi, return_h_states=True)
        (y.float().sum() + hs.float().sum()).backward()

    r = _time(ref_step, iters=1, warmup=1)
    o = _time(our_step)
    return {"op": "scan", "shape": f"B=1 d_inner={D} d_state={N}", "ref_seq": ref_seq, "our_seq": seq,
            "ref_ms_per_token": round(r / ref_seq, 5), "ours_ms_per_token": round(o / seq, 5),
            "speedup": round((r / ref_seq) / (o / seq), 1)}


def case_diff_attn(ref_dir, seq=4096):
    _ref_import(ref_dir)
    from mamformer.layers.kda_diff import FullDiffAttention as RefFDA
    from mamformer_b200.models.kda_diff import FullDiffAttention as OurFDA
    kw = dict(d_model=4096, n_heads=32, n_kv_heads=8, head_dim=128, latent_dim=512, sliding_window=4096,
              use_state_injection=False)
    torch.manual_seed(0)
    ref = RefFDA(**kw).cuda()
    ours = OurFDA(**kw).cuda()
    from mamformer_b200.utils.precision import to_compute_dtype
    to_compute_dtype(ours, torch.bfloat16)             # matrices bf16, vectors fp32, as in training
    from mamformer_b200.ops.linear import use_native_linear
    use_native_linear(ours)
    x = (torch.randn(1, seq, 4096, device="cuda") * 0.5).requires_grad_()
    xb = x.detach().bfloat16().requires_grad_()

    def ref_step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = ref(x)[0]
        out.float().sum().backward()

    def our_step():
        ours(xb)[0].float().sum().backward()

    r = _time(ref_step, iters=2, warmup=1)
    o = _time(our_step)
    return {"op": "diff_attn", "shape": f"B=1 S={seq} d=4096 heads 32/8 hd 128", "ref_ms": round(r, 3),
            "ours_ms": round(o, 3), "speedup": round(r / o, 1),
            "note": "reference window mask with the causal mask leaves the diagonal; both run it"}


def case_moe(ref_dir, tokens=4096):
    _ref_import(ref_dir)
    from mamformer.layers.moe import DeepSeekMoE as RefMoE
    from mamformer_b200.models.moe import DeepSeekMoE as OurMoE
    args = (4096, 2, 2304, 128, 8, 576)
    torch.manual_seed(0)
    ref = RefMoE(*args).cuda()
    ours = OurMoE(*args).cuda()
    from mamformer_b200.utils.precision import to_compute_dtype
    to_compute_dtype(ours, torch.bfloat16)
    from mamformer_b200.ops.linear import use_native_linear
    use_native_linear(ours)
    x = (torch.randn(1, tokens, 4096, device="cuda") * 0.5).requires_grad_()
    xb = x.detach().bfloat16().requires_grad_()

    def ref_step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = ref(x)[0]
        out.float().sum().backward()

    def our_step():
        ours(xb)[0].float().sum().backward()

    r = _time(ref_step, iters=2, warmup=1)
    o = _time(our_step)
    return {"op": "moe", "shape": f"T={tokens} d=4096 E=128 top-8 I=576 + 2 shared x 2304", "ref_ms": round(r, 3),
            "ours_ms": round(o, 3), "speedup": round(r / o, 1)}


CASES = {"scan": case_scan, "diff_attn": case_diff_attn, "moe": case_moe}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--op", default="all", choices=["all"] + list(CASES))
    ap.add_argument("--ref-dir", default=os.path.join(ROOT, "baseline", "_ref"))
    a = ap.parse_args(argv)
    if not os.path.isdir(os.path.join(a.ref_dir, "mamformer")):
        print(json.dumps({"unavailable": f"reference package not found under {a.ref_dir}"}))
        return
    for op in (CASES if a.op == "all" else [a.op]):
        try:
            print(json.dumps(CASES[op](a.ref_dir)), flush=True)
        except torch.cuda.OutOfMemoryError as exc:
            print(json.dumps({"op": op, "reference_oom": str(exc).splitlines()[0][:200]}), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
