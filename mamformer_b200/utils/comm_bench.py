"""Multi-GPU benchmarks of the fused compute + collective paths, as fractions of their roofline.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m mamformer_b200.utils.comm_bench [--op all|ag_gemm|gemm_rs|dp_allreduce|ep_moe]

Every case runs on all ranks with CUDA events on the launching stream (barrier and synchronise on
both sides, warm-up first); the reported time is the MAX over ranks.  Roofline per case = the
slower of (its FLOPs at the measured bf16 GEMM peak) and (the bytes that must cross NVLink into
one GPU at the measured peer-copy bandwidth, 770 GB/s per direction).  Each fused path is
compared with the same work done as NCCL collective + this repository's GEMM (the unfused
baseline).

* ag_gemm  - sequence-parallel column GEMM on all-gathered row shards: "pull" (copy-engine pulls
             of the peers' shards overlapped with the local-shard GEMM) and "kernel" (the
             tcgen05 GEMM's TMA producer reads the peers' shards).  NVLink bytes in:
             (P-1)/P * T * K * 2.
* gemm_rs  - row GEMM + reduce-scatter of the partial products: "pull" (other ranks' row blocks
             first, then copy-engine pulls of the peers' partials overlapped with the own-rows
             GEMM) and "kernel" (epilogue stores into the owners' staging slots + local sum).
             NVLink bytes: (P-1)/P * T * N * 2.
* dp_allreduce - 64 MiB fp32 gradient bucket summed over symmetric memory, two-shot:
             "kernel" (reduce-scatter and all-gather by SM P2P loads) and "pull" (copy-engine
             pulls, in-place adds by the slice owner).  NVLink bytes in: 2 (P-1)/P * n * 4.
* ep_moe   - expert-parallel MoE layer forward + backward (T tokens per rank, top-k routing,
             128 experts sharded over P ranks) with the NVLink peer-memory transport vs NCCL
             all-to-all.  Roofline: expert GEMM FLOPs vs dispatch + combine bytes.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0     # measured peer copy, GB/s per direction per GPU


def _peak_tflops() -> float:
    from mamformer_b200.utils.kernel_bench import _peaks
    return _peaks()[1]


def _time(fn, iters: int = 10, warmup: int = 3) -> float:
    """Per-iteration milliseconds, max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    return float(t.item())


def _report(name, ms_fused, ms_base, flops, link_bytes, extra=None):
    peak = _peak_tflops()
    t_roof = max(flops / (peak * 1e12), link_bytes / (LINK_GBS * 1e9)) * 1e3
    out = {"op": name, "world": dist.get_world_size(), "fused_ms": round(ms_fused, 4),
           "baseline_nccl_ms": round(ms_base, 4) if ms_base is not None else None,
           "roofline_ms": round(t_roof, 4), "frac_of_roofline": round(t_roof / ms_fused, 3),
           "tflops": round(flops / ms_fused / 1e9, 1) if flops else None,
           "link_gbs": round(link_bytes / ms_fused / 1e6, 1) if link_bytes else None}
    if extra:
        out.update(extra)
    if dist.get_rank() == 0:
        print(json.dumps(out), flush=True)


def case_ag_gemm(T=16384, K=4096, N=4096):
    from mamformer_b200.ops import gemm
    from mamformer_b200.parallel import tp_fused
    P, r = dist.get_world_size(), dist.get_rank()
    g = torch.Generator(device="cuda").manual_seed(r)
    x = (torch.randn(T // P, K, device="cuda", generator=g) * 0.5).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    full = torch.empty(T, K, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)

    def base():
        dist.all_gather_into_tensor(full, x)
        gemm.mm(full, w, out=out)
    mb = _time(base)
    for impl in ("pull", "kernel"):
        ms = _time(lambda: tp_fused.ag_gemm(x, w, dist.group.WORLD, impl=impl))
        _report("ag_gemm", ms, mb, 2.0 * T * N * K, (P - 1) / P * T * K * 2,
                {"impl": impl, "T": T, "K": K, "N": N})


def case_gemm_rs(T=16384, K=4096, N=4096):
    from mamformer_b200.ops import gemm
    from mamformer_b200.parallel import tp_fused
    P, r = dist.get_world_size(), dist.get_rank()
    g = torch.Generator(device="cuda").manual_seed(r)
    y = (torch.randn(T, K, device="cuda", generator=g) * 0.5).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    part = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
    mine = torch.empty(T // P, N, device="cuda", dtype=torch.bfloat16)

    def base():
        gemm.mm(y, w, out=part)
        dist.reduce_scatter_tensor(mine, part)
    mb = _time(base)
    for impl in ("pull", "kernel"):
        ms = _time(lambda: tp_fused.gemm_rs(y, w, dist.group.WORLD, impl=impl))
        _report("gemm_rs", ms, mb, 2.0 * T * N * K, (P - 1) / P * T * N * 2,
                {"impl": impl, "T": T, "K": K, "N": N})


def case_dp_allreduce(mib=64):
    import torch.distributed._symmetric_memory as symm
    from mamformer_b200.ops._ext import require_native
    from mamformer_b200.optim import _DP_SLOT0
    C = require_native()
    P, r = dist.get_world_size(), dist.get_rank()
    n = mib * (1 << 20) // 4
    buf = symm.empty(n, dtype=torch.float32, device="cuda")
    buf.normal_()
    h = symm.rendezvous(buf, dist.group.WORLD)
    plain = torch.randn(n, device="cuda")
    state = {"epoch": 0}

    def barrier():
        state["epoch"] += 1
        C.ep_barrier(h.signal_pad_ptrs, r, state["epoch"], _DP_SLOT0)

    def fused():
        barrier()
        C.dp_reduce_scatter(h.buffer_ptrs, r, 0, n, 1.0, False)
        barrier()
        C.dp_all_gather(h.buffer_ptrs, r, 0, n)
        barrier()
    from mamformer_b200.optim import dp_pull_allreduce
    tmp = {}
    mb = _time(lambda: dist.all_reduce(plain))
    ms = _time(fused)
    _report("dp_allreduce", ms, mb, 0.0, 2 * (P - 1) / P * n * 4,
            {"impl": "kernel", "MiB": mib, "comm_error": int(C.comm_error())})
    ms = _time(lambda: dp_pull_allreduce(h, buf, 0, n, barrier, tmp))
    _report("dp_allreduce", ms, mb, 0.0, 2 * (P - 1) / P * n * 4,
            {"impl": "pull", "MiB": mib, "comm_error": int(C.comm_error())})


def case_ep_moe(T=8192, d=4096, E=128, k=8, I=576):
    import copy
    from mamformer_b200.models.moe import DeepSeekMoE
    from mamformer_b200.parallel.expert_parallel import ExpertParallelGroup, shard_experts_ep
    P, r = dist.get_world_size(), dist.get_rank()
    torch.manual_seed(0)
    base = DeepSeekMoE(d, n_shared_experts=1, shared_expert_dim=I, n_routed_experts=E, top_k=k,
                       routed_expert_dim=I).cuda().bfloat16()
    g = torch.Generator(device="cuda").manual_seed(100 + r)
    x = (torch.randn(1, T, d, device="cuda", generator=g) * 0.5).bfloat16().requires_grad_()
    dy = torch.randn(1, T, d, device="cuda", generator=g).bfloat16()
    epg = ExpertParallelGroup(group=dist.group.WORLD)
    res = {}
    for backend in ("p2p", "nccl"):
        m = copy.deepcopy(base)
        shard_experts_ep(m, epg, backend=backend)

        def step():
            y, _ = m(x)
            y.backward(dy)
            for p_ in m.parameters():
                p_.grad = None
            x.grad = None
        res[backend] = _time(step, iters=5)
        m.ep_engine.check_error()
    flops = 3 * 3 * 2.0 * T * (k + 1) * d * I             # 3 GEMMs per expert (k routed + 1 shared), fwd + 2 bwd
    link = 2 * 2 * (P - 1) / P * T * k * d * 2            # dispatch + combine, fwd and bwd
    _report("ep_moe", res["p2p"], res["nccl"], flops, link, {"T_per_rank": T, "d": d, "E": E, "k": k, "I": I})


CASES = {"ag_gemm": case_ag_gemm, "gemm_rs": case_gemm_rs, "dp_allreduce": case_dp_allreduce, "ep_moe": case_ep_moe}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--op", default="all", choices=["all"] + list(CASES))
    a = ap.parse_args(argv)
    import datetime
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    try:
        for op in (CASES if a.op == "all" else [a.op]):
            CASES[op]()
            torch.cuda.empty_cache()
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
