"""Failure detection and recovery on the host: heartbeats across gloo ranks, NaN skip and
checkpoint rollback (skipping a truncated checkpoint), non-finite gradient skip."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from mamformer_b200 import MamformerConfig, MamformerForCausalLM
from mamformer_b200.engine import TrainConfig, Trainer
from mamformer_b200.fault import FaultPolicy, Heartbeat, RankFailureError, ResilientTrainer


def _trainer():
    torch.manual_seed(0)
    return Trainer(MamformerForCausalLM(MamformerConfig.from_preset("debug")),
                   TrainConfig(learning_rate=1e-3, warmup_steps=1, micro_batch=2, compute_dtype=torch.float32))


def test_nan_skip_and_rollback(tmp_path):
    from mamformer_b200.checkpoint import save_checkpoint
    tr = _trainer()
    rt = ResilientTrainer(tr, FaultPolicy(max_consecutive_nan=3, checkpoint_dir=str(tmp_path)))
    ids = torch.randint(0, 1000, (2, 16))
    assert rt.train_step(ids) is not None
    save_checkpoint(str(tmp_path / "checkpoint_step_1.pt"), tr.model, tr.optimizer, tr.scheduler, step=1)
    good = {n: p.detach().clone() for n, p in tr.model.named_parameters()}
    # a newer checkpoint that is truncated (unreadable) must be skipped
    (tmp_path / "checkpoint_step_2.pt").write_bytes(b"not a checkpoint")
    w = tr.model.model.embed_tokens.weight
    with torch.no_grad():
        w.fill_(float("nan"))
    for _ in range(3):
        assert rt.train_step(ids) is None
    assert tr.skipped_steps == 3
    assert any("skip unreadable checkpoint checkpoint_step_2.pt" in e for e in rt.events)
    assert any("rolled back to checkpoint_step_1.pt" in e for e in rt.events)
    for n, p in tr.model.named_parameters():
        assert torch.equal(p.detach(), good[n]), n
    assert rt.train_step(ids) is not None


def test_nonfinite_grad_skip():
    tr = _trainer()
    ids = torch.randint(0, 1000, (2, 16))
    before = {n: p.detach().clone() for n, p in tr.model.named_parameters()}
    h = tr.model.model.norm.weight.register_hook(lambda g: g * float("inf"))
    tr.train_step(ids, sync_loss=True, check_grads=True)
    h.remove()
    assert tr.skipped_steps == 1
    for n, p in tr.model.named_parameters():
        assert torch.equal(p.detach(), before[n]), n


def _flush(q):
    """os._exit skips the queue's feeder thread: hand the pending items to the pipe first."""
    q.close()
    q.join_thread()


def _hb_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    result, code = None, 0
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        hb = Heartbeat(stale_after_s=5.0)
        hb.beat(0)
        dist.barrier()
        if rank == 1:
            hb.report_failure("simulated: data loader crashed")
            dist.barrier()
            os._exit(0)            # leaves without further collectives
        dist.barrier()
        try:
            hb.check()
            result = "no failure detected"
        except RankFailureError as e:
            result = "ok" if "rank 1 failed" in str(e) else str(e)
        # stale detection: rank 1's beat is old relative to a clock far in the future
        try:
            hb.check(now=1e12)
        except RankFailureError:
            pass
    except Exception as e:
        result, code = repr(e), 1
    q.put((rank, result))
    _flush(q)
    os._exit(code)


def test_heartbeat_detects_failed_rank():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_hb_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    r, msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert (r, msg) == (0, "ok")
