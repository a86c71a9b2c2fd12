"""Native MoE (grouped tcgen05 GEMMs) and fused linear-CE vs the PyTorch reference."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from mamformer_b200.ops import reference as ref  # noqa: E402


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp(min=1e-6)).item()


def _moe_case(T=300, d=128, E=8, k=2, I=64, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, d, device="cuda", generator=g).bfloat16()
    scores = torch.randn(T, E, device="cuda", generator=g)
    vals, idx = torch.topk(scores, k)
    gates = torch.softmax(vals, -1)
    w = [(0.05 * torch.randn(*s, device="cuda", generator=g)).bfloat16() for s in ((E, I, d), (E, I, d), (E, d, I))]
    return x, gates, idx, w


def test_moe_routed_matches_reference():
    from mamformer_b200.ops import moe
    x, gates, idx, (wg, wu, wd) = _moe_case()
    leaves = [t.clone().requires_grad_() for t in (x, gates, wg, wu, wd)]
    out = moe.routed(leaves[0], idx, leaves[1], *leaves[2:])
    dout = torch.randn_like(out)
    (out.float() * dout.float()).sum().backward()
    rl = [t.detach().float().clone().requires_grad_() for t in (x, gates, wg, wu, wd)]
    ro = ref.moe_routed(rl[0], idx, rl[1], *rl[2:])
    (ro * dout.float()).sum().backward()
    assert _rel(out, ro) < 2e-2
    for name, a, b in zip(["dx", "dgates", "dwg", "dwu", "dwd"], leaves, rl):
        assert _rel(a.grad, b.grad) < 3e-2, name


def test_moe_weight_grads_go_to_main_grad():
    from mamformer_b200.ops import moe
    x, gates, idx, (wg, wu, wd) = _moe_case(seed=1)
    params = [torch.nn.Parameter(t) for t in (wg, wu, wd)]
    for p in params:
        p.main_grad = torch.full(p.shape, 0.5, device="cuda")
    out = moe.routed(x, idx, gates, *params)
    out.float().sum().backward()
    rl = [t.detach().float().clone().requires_grad_() for t in (wg, wu, wd)]
    ref.moe_routed(x.float(), idx, gates, *rl).sum().backward()
    for p, r in zip(params, rl):
        assert p.grad is None
        assert _rel(p.main_grad - 0.5, r.grad) < 3e-2


def test_moe_expert_outputs():
    from mamformer_b200.ops import moe
    x, gates, idx, (wg, wu, wd) = _moe_case(T=100, seed=2)
    out = moe.expert_outputs(x, idx, wg, wu, wd)
    ro = ref.moe_expert_outputs(x.float(), idx, wg.float(), wu.float(), wd.float())
    assert out.shape == (100, 2, 128) and _rel(out, ro) < 2e-2


@pytest.mark.parametrize("keep", ["4", "0"])          # logits kept for the backward / recomputed
@pytest.mark.parametrize("T,V,d", [(300, 1000, 128), (2048, 32000, 256)])
def test_linear_cross_entropy(T, V, d, keep, monkeypatch):
    from mamformer_b200.ops import linear_ce
    monkeypatch.setenv("MAMF_CE_SAVE_GB", keep)
    g = torch.Generator(device="cuda").manual_seed(3)
    h = torch.randn(T, d, device="cuda", generator=g).bfloat16().requires_grad_()
    W = (0.05 * torch.randn(V, d, device="cuda", generator=g)).bfloat16().requires_grad_()
    labels = torch.randint(0, V, (T,), device="cuda", generator=g)
    labels[::7] = -100
    loss = linear_ce.linear_cross_entropy(h, W, labels)
    (3.0 * loss).backward()
    hr = h.detach().clone().requires_grad_()
    Wr = W.detach().clone().requires_grad_()
    logits = (hr.float() @ Wr.float().t()).bfloat16().float()
    lr = F.cross_entropy(logits, labels, ignore_index=-100)
    (3.0 * lr).backward()
    assert abs(loss.item() - lr.item()) < 2e-3 * lr.item()
    assert _rel(h.grad, hr.grad) < 3e-2
    assert _rel(W.grad, Wr.grad) < 3e-2


@pytest.mark.parametrize("T,E,k", [(1000, 128, 8), (77, 16, 4), (64, 256, 2)])
def test_router_topk_and_histogram(T, E, k):
    from mamformer_b200.ops import native
    g = torch.Generator(device="cuda").manual_seed(7)
    s = torch.randn(T, E, device="cuda", generator=g).requires_grad_()
    gates, idx = native.router_topk(s, k)
    sr = s.detach().clone().requires_grad_()
    vr, ir = torch.topk(sr, k, dim=-1)
    gr = torch.softmax(vr, -1)
    assert torch.equal(idx, ir)
    assert torch.allclose(gates, gr, atol=1e-5, rtol=1e-5)
    dg = torch.randn(T, k, device="cuda", generator=g)
    gates.backward(dg)
    gr.backward(dg)
    assert torch.allclose(s.grad, sr.grad, atol=1e-5, rtol=1e-4)
    h = native.expert_histogram(idx, E)
    assert torch.equal(h, torch.bincount(idx.flatten(), minlength=E))
