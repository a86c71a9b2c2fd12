"""Parallel runtime on 2+ GPUs (NCCL, one process per GPU; skipped with fewer GPUs)."""
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spawn(fn, world, timeout=240):
    import os
    import queue
    import _gpu_dist_workers as W
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=W._run, args=(getattr(W, fn), r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, msg = q.get(timeout=timeout)
            res[r] = msg
    except queue.Empty:
        res.update({r: "no result (rank exited or timed out)" for r in range(world) if r not in res})
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    bad = {r: m for r, m in res.items() if m != "ok"}
    assert not bad, "\n".join(f"rank {r}:\n{m}" for r, m in bad.items())


def _worlds(*sizes):
    """World sizes of a multi-GPU test: every one this box has GPUs for (2 and up), optionally
    restricted by MAMF_TEST_WORLDS (e.g. "8")."""
    import os
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    only = {int(x) for x in os.environ.get("MAMF_TEST_WORLDS", "").split(",") if x.strip()}
    out = []
    for w in sizes:
        skip = n < w or (bool(only) and w not in only)
        out.append(pytest.param(w, marks=pytest.mark.skipif(skip, reason=f"needs {w} GPUs / not selected")))
    return out


ALL = _worlds(2, 4, 8)


@pytest.mark.parametrize("world", ALL)
def test_data_parallel_trainer(world):
    _spawn("dp_trainer_worker", world)


@pytest.mark.parametrize("world", ALL)
def test_data_parallel_p2p_transport(world):
    """Copy-engine pull form: replicas bitwise equal, gradients equal to NCCL's (rel 1e-5)."""
    _spawn("dp_p2p_worker", world)


@pytest.mark.parametrize("world", ALL)
def test_data_parallel_kernel_transport(world):
    _spawn("dp_pull_worker", world)


@pytest.mark.parametrize("world", _worlds(2))
def test_data_parallel_nvls_transport(world):
    _spawn("dp_nvls_worker", world)


@pytest.mark.parametrize("world", ALL)
def test_expert_parallel_moe(world):
    _spawn("ep_moe_worker", world)


@pytest.mark.parametrize("world", ALL)
def test_expert_parallel_capacity_overflow_reruns_the_step(world):
    _spawn("ep_capacity_rerun_worker", world)


@pytest.mark.parametrize("world", _worlds(2, 8))
def test_tp_fused_gemms(world):
    _spawn("tp_fused_worker", world)


@pytest.mark.parametrize("world", _worlds(2))
def test_tp_model_fused_matches_unfused(world):
    _spawn("tp_model_fused_worker", world)
