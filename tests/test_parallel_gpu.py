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


needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs 2 GPUs")


@needs2
def test_data_parallel_trainer_two_gpus():
    _spawn("dp_trainer_worker", 2)


@needs2
def test_data_parallel_p2p_transport_two_gpus():
    _spawn("dp_p2p_worker", 2)


@needs2
def test_data_parallel_kernel_transport_two_gpus():
    _spawn("dp_pull_worker", 2)


@needs2
def test_data_parallel_nvls_transport_two_gpus():
    _spawn("dp_nvls_worker", 2)


@needs2
def test_expert_parallel_moe_two_gpus():
    _spawn("ep_moe_worker", 2)


@needs2
def test_tp_fused_gemms_two_gpus():
    _spawn("tp_fused_worker", 2)


@needs2
def test_tp_model_fused_matches_unfused_two_gpus():
    _spawn("tp_model_fused_worker", 2)
