"""Worker bodies for the multi-GPU tests (NCCL, one process per GPU)."""
import copy
import os
import traceback

import torch
import torch.distributed as dist


def _run(fn, rank, world, port, out):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        import datetime
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=datetime.timedelta(seconds=120))
        fn(rank, world)
        out.put((rank, "ok"))
    except Exception:
        out.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def ep_moe_worker(rank, world):
    """Expert-parallel MoE layer (both transports) against the unsharded layer on one GPU."""
    from mamformer_b200.models.moe import DeepSeekMoE
    from mamformer_b200.parallel.expert_parallel import ExpertParallelGroup, shard_experts_ep
    torch.manual_seed(0)
    base = DeepSeekMoE(128, n_shared_experts=1, shared_expert_dim=128, n_routed_experts=8, top_k=2,
                       routed_expert_dim=64).cuda().bfloat16().eval()
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    x = torch.randn(2, 192, 128, device="cuda", generator=g).bfloat16()
    ref = copy.deepcopy(base)
    xr = x.clone().requires_grad_()
    yr, _ = ref(xr)
    dy = torch.randn(yr.shape, device="cuda", generator=g).bfloat16()
    yr.backward(dy)
    ref_w = {n: p.grad.float().clone() for n, p in ref.named_parameters() if n.startswith("routed_")}
    for n in ref_w:
        dist.all_reduce(ref_w[n])                      # owners see every rank's tokens
    epg = ExpertParallelGroup(group=dist.group.WORLD)
    for backend in ("p2p", "nccl"):
        m = copy.deepcopy(base)
        shard_experts_ep(m, epg, backend=backend)
        xe = x.clone().requires_grad_()
        ye, _ = m(xe)
        assert _rel(ye, yr) < 2e-2, (backend, "out", _rel(ye, yr))
        ye.backward(dy)
        assert _rel(xe.grad, xr.grad) < 3e-2, (backend, "dx", _rel(xe.grad, xr.grad))
        s, e = epg.get_expert_range(8)
        for n, p in m.named_parameters():
            if n in ref_w:
                assert _rel(p.grad, ref_w[n][s:e]) < 3e-2, (backend, n, _rel(p.grad, ref_w[n][s:e]))
        m.ep_engine.check_error()
    torch.cuda.synchronize()


def _tiny_moe_model():
    from mamformer_b200.config import MamformerConfig
    from mamformer_b200.models.model import MamformerForCausalLM
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    d = MamformerConfig.from_yaml(os.path.join(root, "configs", "ultra-7b.yaml")).to_dict()
    d.update(d_model=256, n_heads=2, n_kv_heads=1, head_dim=128, n_layers=2, vocab_size=512,
             interleave_fusion_layers=[1], interleave_last_layers_dense=1, moe_n_routed_experts=16,
             moe_top_k=4, moe_expert_intermediate_dim=64, moe_shared_expert_intermediate_dim=128,
             kda_diff_kernel_dim=128, kda_diff_latent_dim=64, d_ff=512, mtp_enabled=False)
    torch.manual_seed(0)
    return MamformerForCausalLM(MamformerConfig.from_dict(d)).cuda()


def ep_capacity_rerun_worker(rank, world):
    """Expert parallelism with a deliberately small capacity: steps whose routing overflows an
    owner are discarded and rerun with a larger capacity, so the result is bitwise equal to a
    run whose capacity can never overflow."""
    from mamformer_b200.engine import TrainConfig, Trainer
    from mamformer_b200.parallel.expert_parallel import ExpertParallelGroup, shard_experts_ep
    g = torch.Generator().manual_seed(7 + rank)
    ids = [torch.randint(0, 512, (2, 128), generator=g).cuda() for _ in range(3)]
    results = []
    for cf in (float(world), 0.3):
        model = _tiny_moe_model()
        shard_experts_ep(model, ExpertParallelGroup(group=dist.group.WORLD), backend="p2p", capacity_factor=cf)
        tr = Trainer(model, TrainConfig(learning_rate=1e-3, warmup_steps=1, micro_batch=1), dp_group=dist.group.WORLD,
                     expert_dp_group=None, ep_group=dist.group.WORLD)
        losses = [tr.train_step(x, sync_loss=True) for x in ids]
        eng = model._mamf_ep_engine
        results.append((losses, {n: p.detach().clone() for n, p in model.named_parameters()}, eng.overflow_steps))
        del tr, model
    (l_big, p_big, o_big), (l_small, p_small, o_small) = results
    assert o_big == 0 and o_small >= 1, (o_big, o_small)
    # The capacity only sizes buffers, so the routed computation is the same; what differs run to
    # run is the order of the float atomics in the scan backward (dA, dD), which can flip the
    # sign of a near-zero AdamW update: parameters agree to 2 * lr per step.
    for a, b in zip(l_big, l_small):
        assert abs(a - b) <= 1e-5 * abs(a), (l_big, l_small)
    for n in p_big:
        diff = (p_big[n].float() - p_small[n].float()).abs().max().item()
        assert diff <= 2 * 1e-3 * len(ids) + 1e-6, (n, diff)
    torch.cuda.synchronize()


def dp_trainer_worker(rank, world):
    """Bucketed, overlapped data-parallel gradient sums on NCCL: the reduced gradients equal a
    single-GPU step on the concatenated batch, and every rank ends with the same parameters.
    (Parameters after one AdamW step are not compared with the single-GPU run: the first step
    moves every element by lr * sign(g), so a near-zero gradient element whose sign differs by
    rounding changes the result by 2 lr.)"""
    from mamformer_b200 import MamformerConfig, MamformerForCausalLM
    from mamformer_b200.engine import Trainer, TrainConfig
    cfg = MamformerConfig.from_preset("debug")
    tc = TrainConfig(learning_rate=1e-3, warmup_steps=1, micro_batch=1)
    torch.manual_seed(0)
    ref = Trainer(MamformerForCausalLM(cfg).cuda(), tc)
    ids = torch.randint(0, cfg.vocab_size, (world, 128), generator=torch.Generator().manual_seed(5)).cuda()
    ref.train_step(ids, sync_loss=True)
    torch.manual_seed(0)
    tr = Trainer(MamformerForCausalLM(cfg).cuda(), tc, dp_group=dist.group.WORLD, bucket_mb=1.0)
    tr.train_step(ids[rank:rank + 1], sync_loss=True)
    torch.cuda.synchronize()
    bad = []
    for (n, p), (_, q) in zip(tr.model.named_parameters(), ref.model.named_parameters()):
        other = p.detach().clone()
        dist.broadcast(other, 0)                   # every rank takes every collective first
        og = p.main_grad.clone()
        dist.broadcast(og, 0)
        if not torch.equal(other, p.detach()):
            bad.append(f"{n}: replicas differ by {(other.float() - p.detach().float()).abs().max().item():.3e}, "
                       f"grads by {(og - p.main_grad).abs().max().item():.3e} (|g| max {og.abs().max().item():.3e}, "
                       f"dtype {p.dtype}, numel {p.numel()})")
        g, gr = p.main_grad / world, q.main_grad   # the DP buffer holds sum_r dL_r/dtheta
        if gr.norm() > 1e-6 and _rel(g, gr) > 3e-2:
            bad.append(f"{n}: grad rel {_rel(g, gr):.3e}")
    assert not bad, bad


def dp_p2p_worker(rank, world, nvls=False):
    """Data-parallel gradient sums by the NVLink kernels (symmetric-memory gradient buffers):
    reduced gradients equal the single-GPU batch gradient, replicas stay bitwise equal over two
    steps, and the result matches the NCCL transport."""
    import os as _os
    from mamformer_b200 import MamformerConfig, MamformerForCausalLM
    from mamformer_b200.engine import Trainer, TrainConfig
    _os.environ["MAMF_DP_NVLS"] = "1" if nvls else "0"
    cfg = MamformerConfig.from_preset("debug")
    tc = TrainConfig(learning_rate=1e-3, warmup_steps=1, micro_batch=1)
    ids = torch.randint(0, cfg.vocab_size, (2, world, 128), generator=torch.Generator().manual_seed(5)).cuda()
    torch.manual_seed(0)
    ref = Trainer(MamformerForCausalLM(cfg).cuda(), tc)
    torch.manual_seed(0)
    nc = Trainer(MamformerForCausalLM(cfg).cuda(), tc, dp_group=dist.group.WORLD, bucket_mb=1.0)
    torch.manual_seed(0)
    tr = Trainer(MamformerForCausalLM(cfg).cuda(), tc, dp_group=dist.group.WORLD, bucket_mb=1.0,
                 dp_transport="p2p")
    assert any(seg.symm is not None for _, seg in tr.optimizer.segments), "no symmetric gradient segment"
    bad = []
    for step in range(2):
        ref.train_step(ids[step], sync_loss=True)
        nc.train_step(ids[step, rank:rank + 1], sync_loss=True)
        tr.train_step(ids[step, rank:rank + 1], sync_loss=True)
        torch.cuda.synchronize()
        for (n, p), (_, q), (_, u) in zip(tr.model.named_parameters(), ref.model.named_parameters(),
                                          nc.model.named_parameters()):
            other = p.detach().clone()
            dist.broadcast(other, 0)
            if not torch.equal(other, p.detach()):
                bad.append(f"step {step} {n}: replicas differ")
            if step == 0:
                g, gr = p.main_grad / world, q.main_grad
                if gr.norm() > 1e-6 and _rel(g, gr) > 3e-2:
                    bad.append(f"{n}: grad rel {_rel(g, gr):.3e}")
                if _rel(p.main_grad, u.main_grad) > 1e-5:
                    bad.append(f"{n}: p2p vs nccl grad rel {_rel(p.main_grad, u.main_grad):.3e}")
    from mamformer_b200.fault import check_device_status
    check_device_status()
    assert not bad, bad[:10]


def dp_nvls_worker(rank, world):
    dp_p2p_worker(rank, world, nvls=True)


def dp_pull_worker(rank, world):
    """The SM-load ("kernel") form of the peer-memory gradient all-reduce (the copy-engine
    "pull" form is the default that dp_p2p_worker exercises)."""
    import mamformer_b200.optim as O
    O._DP_IMPL = "kernel"
    try:
        dp_p2p_worker(rank, world)
    finally:
        O._DP_IMPL = "pull"


def tp_fused_worker(rank, world):
    """Fused all-gather->GEMM and GEMM->reduce-scatter (and their autograd) against NCCL + torch."""
    from mamformer_b200.parallel import tp_fused
    g = dist.group.WORLD
    torch.manual_seed(0)
    T, K, N = 512 * world, 1024, 768
    rows = T // world
    x_full = (torch.randn(T, K, device="cuda") * 0.5).bfloat16()
    W = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    x_loc = x_full[rank * rows:(rank + 1) * rows].contiguous()
    y = tp_fused.ag_gemm(x_loc, W, g)
    want = (x_full.float() @ W.float().t())
    assert _rel(y, want) < 1e-2, _rel(y, want)
    # reduce-scatter: every rank holds a different partial product
    parts = [(torch.randn(T, K, device="cuda", generator=torch.Generator(device="cuda").manual_seed(10 + r)) * 0.5).bfloat16()
             for r in range(world)]
    z = tp_fused.gemm_rs(parts[rank], W, g)
    full = sum(p_.float() @ W.float().t() for p_ in parts)
    assert _rel(z, full[rank * rows:(rank + 1) * rows]) < 1e-2
    # autograd through the sequence-parallel SwiGLU against the unsharded FFN
    d, ff = 256, 512
    torch.manual_seed(1)
    wg, wu, wd = (torch.randn(ff, d, device="cuda") * 0.05, torch.randn(ff, d, device="cuda") * 0.05,
                  torch.randn(d, ff, device="cuda") * 0.05)
    m = tp_fused.SequenceParallelSwiGLU(d, ff, g).cuda().bfloat16()
    sl = slice(rank * ff // world, (rank + 1) * ff // world)
    with torch.no_grad():
        m.gate_proj.weight.copy_(wg[sl]); m.up_proj.weight.copy_(wu[sl]); m.down_proj.weight.copy_(wd[:, sl])
    xs = (torch.randn(T, d, device="cuda", generator=torch.Generator(device="cuda").manual_seed(3)) * 0.5).bfloat16()
    xl = xs[rank * rows:(rank + 1) * rows].clone().requires_grad_()
    out = m(xl)
    xr = xs.float().clone().requires_grad_()
    ref = (torch.nn.functional.silu(xr @ wg.t()) * (xr @ wu.t())) @ wd.t()
    assert _rel(out, ref[rank * rows:(rank + 1) * rows]) < 2e-2
    go = torch.randn(T, d, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
    out.backward(go[rank * rows:(rank + 1) * rows].bfloat16())
    ref.backward(go)
    assert _rel(xl.grad, xr.grad[rank * rows:(rank + 1) * rows]) < 3e-2
    torch.cuda.synchronize()


def tp_model_fused_worker(rank, world):
    """Model-level tensor parallelism on CUDA/bf16: the path with GEMM -> reduce-scatter fused
    kernels gives the same loss and gradients as the NCCL all-reduce path."""
    from mamformer_b200 import MamformerConfig, MamformerForCausalLM
    from mamformer_b200.config import InterleaveConfig, KDADiffConfig, MambaConfig, MoEConfig, MTPConfig
    from mamformer_b200.engine import Trainer, TrainConfig
    from mamformer_b200.parallel import DistributedCoordinator, ParallelConfig, tp_fused
    from mamformer_b200.parallel.tensor_parallel import ColumnParallelLinear, RowParallelLinear
    cfg = MamformerConfig(
        d_model=256, n_layers=4, n_heads=4, n_kv_heads=2, head_dim=64, d_ff=512, vocab_size=512,
        max_seq_len=256, mamba=MambaConfig(expand=2, d_state=64, d_conv=4),
        moe=MoEConfig(enabled=False), kda_diff=KDADiffConfig(enabled=True, kernel_dim=64, latent_dim=64),
        mtp=MTPConfig(enabled=True, depth=1, loss_weight=0.3),
        interleave=InterleaveConfig(enabled=True, pattern="cross_layer", attn_every_k=2, first_layer_attn=False,
                                    last_layers_dense=0, fusion_layers=[3]))
    ids = torch.randint(0, 512, (2, 128), generator=torch.Generator().manual_seed(3)).cuda()
    coord = DistributedCoordinator(ParallelConfig(tp_size=world)).initialize()
    res = {}
    for fused in (True, False):
        torch.manual_seed(0)
        model = coord.shard_model(MamformerForCausalLM(cfg).cuda())
        for m in model.modules():
            if isinstance(m, (ColumnParallelLinear, RowParallelLinear)):
                m.fused = fused
        tr = Trainer(model, TrainConfig(learning_rate=1e-3, warmup_steps=1, micro_batch=2))
        n_ws = len(tp_fused._WS)
        loss = tr.train_step(ids, sync_loss=True)
        torch.cuda.synchronize()
        if fused:
            assert len(tp_fused._WS) > 0, "fused TP path not taken"
        res[fused] = (loss, {n: p.main_grad.float().clone() for n, p in tr.model.named_parameters()})
    (lf, gf), (lu, gu) = res[True], res[False]
    assert abs(lf - lu) < 2e-2 * abs(lu), (lf, lu)
    bad = [f"{n}: {_rel(gf[n], gu[n]):.3e}" for n in gu if gu[n].norm() > 1e-6 and _rel(gf[n], gu[n]) > 5e-2]
    assert not bad, bad[:10]
