"""Parallel runtime on CPU: gloo ranks in child processes, each checking its shard of the
gradients (and the loss) against the unsharded single-process model."""
import socket

import pytest
import torch
import torch.multiprocessing as mp

import _dist_workers as W


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spawn(fn, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=W._run, args=(fn, r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, msg = q.get(timeout=600)
        res[r] = msg
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    bad = {r: m for r, m in res.items() if m != "ok"}
    assert not bad, "\n".join(f"rank {r}:\n{m}" for r, m in bad.items())


def test_parallel_config_layout():
    from mamformer_b200.parallel import ParallelConfig
    pc = ParallelConfig(dp_size=2, tp_size=2, pp_size=1, ep_size=2)
    assert pc.world_size == 8
    for r in range(8):
        assert pc.get_global_rank(*pc.get_4d_rank(r)) == r
    assert pc.get_4d_rank(5) == (1, 0, 0, 1)
    assert pc.group_members(("ep",))[0] == [0, 1]
    assert pc.group_members(("tp",))[0] == [0, 2]
    assert pc.group_members(("dp", "ep"))[0] == [0, 1, 4, 5]
    with pytest.raises(ValueError):
        ParallelConfig(tp_size=3).validate(3)


def test_pipeline_split_and_bubble():
    from mamformer_b200.parallel.pipeline_parallel import bubble_fraction, split_layers
    assert split_layers(10, 4) == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert bubble_fraction(4, 12) == pytest.approx(3 / 15)


def test_data_parallel_matches_single_process():
    _spawn(W.dp_worker, 2)


def test_zero1_sharded_optimizer_matches_unsharded():
    _spawn(W.dp_zero_worker, 2)


def test_zero1_bucket_reduction_reaches_every_slice_owner():
    _spawn(W.zero_reduce_worker, 3)


def test_expert_parallel_matches_single_process():
    _spawn(W.ep_worker, 2)


def test_tensor_parallel_matches_single_process():
    _spawn(W.tp_worker, 2)


def test_pipeline_parallel_matches_single_process():
    _spawn(W.pp_worker, 2)


def test_diagnostics_cpu():
    from mamformer_b200.parallel import LoadBalanceAnalyzer, ParallelismMonitor
    lb = LoadBalanceAnalyzer(1, 4)
    lb.update(0, torch.tensor([100, 0, 0, 0]))
    assert any("COLLAPSE" in w for w in lb.get_warnings())
    mon = ParallelismMonitor(n_layers=1, n_experts=4, use_cuda=False)
    mon.start_step()
    mon.comm_start("all_reduce", 1 << 20)
    mon.comm_end("all_reduce")
    st = mon.end_step(1, 2.0, 1000)
    assert st.loss == 2.0 and "communication" in mon.get_full_report()
    mon.reset()


def test_p2p_transport_selection_cpu():
    """The peer-memory gradient transport is chosen only for CUDA groups of 2..8 ranks; on CPU
    (or a single rank) the optimizer keeps ordinary buffers and the NCCL/gloo all-reduce."""
    from mamformer_b200.optim import _p2p_ok
    assert not _p2p_ok("nccl", object(), "cuda")
    assert not _p2p_ok("p2p", None, "cuda")
    assert not _p2p_ok("p2p", object(), "cpu")


def test_fused_tp_path_selection_cpu():
    """The fused GEMM -> reduce-scatter TP path applies only to CUDA bf16 operands whose token
    count splits into whole 128-row shards; CPU tensors keep the collective path."""
    from mamformer_b200.parallel.tensor_parallel import _fused_ok
    x = torch.zeros(512, 64, dtype=torch.bfloat16)
    w = torch.zeros(32, 64, dtype=torch.bfloat16)
    assert not _fused_ok(x, w, None)
    assert not _fused_ok(x, w, object())          # CPU tensors: never fused


def test_dp_slice_bounds_partition():
    """Each rank's slice of a gradient bucket is whole 16-byte words, the slices tile the bucket
    exactly, and the Python bounds (copy-engine form) match the native kernels' slicing."""
    from mamformer_b200.optim import dp_slice_bounds
    try:
        import mamformer_b200._C as C
    except ImportError:
        C = None
    for lo, hi in ((0, 4), (64, 64 + 4096), (128, 128 + 1000), (0, 262144)):
        for P in (2, 3, 4, 8):
            covered = []
            for q in range(P):
                s0, s1 = dp_slice_bounds(lo, hi, P, q)
                assert s0 % 4 == 0 and lo <= s0 <= s1 <= hi
                covered.extend(range(s0, s1))
                if C is not None:
                    sl = C.dp_slice(lo, hi, P)
                    assert s0 == min(hi, lo + q * sl)
            assert covered == list(range(lo, hi))


def test_ep_engine_capacity_and_overflow_bookkeeping():
    """Host side of the expert-parallel capacity protocol: buffer sizes, when a step can
    overflow, and what a detected overflow does (restore the routing state, raise the factor)."""
    import types
    from mamformer_b200.parallel.expert_parallel import EPEngine, ExpertParallelGroup
    eng = EPEngine(ExpertParallelGroup(ep_size=8, ep_rank=3), capacity_factor=2.0)
    assert eng.can_overflow
    assert eng.capacity(1000, 16) == 3072                     # ceil(2 * 1000) + 64 * 16 -> 128-aligned
    assert not EPEngine(ExpertParallelGroup(ep_size=2, ep_rank=0), capacity_factor=2.0).can_overflow
    assert EPEngine(ExpertParallelGroup(ep_size=4, ep_rank=0), capacity_factor=8.0).capacity(1000, 16) == \
        (4 * 1000 + 64 * 16 + 127) // 128 * 128                # never more than P * T * k rows needed
    bias = torch.tensor([0.5, -0.5])
    eng._snapshot = [(bias, torch.tensor([0.0, 0.0]))]
    eng._stage = types.SimpleNamespace(rows_x=1000)
    eng._status_event = types.SimpleNamespace(synchronize=lambda: None)
    eng._status_host = torch.tensor([0, 1234], dtype=torch.int32)
    assert not eng.step_overflowed() and eng.capacity_factor == 2.0
    eng._status_host = torch.tensor([1, 5000], dtype=torch.int32)
    assert eng.step_overflowed()
    assert torch.equal(bias, torch.zeros(2))                  # routing state of the step restored
    assert eng.capacity_factor == 6.25 and eng.overflow_steps == 1
