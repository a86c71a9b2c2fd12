"""tcgen05 GEMM (dense, grouped-M, grouped-K) vs fp32 torch.matmul on the same bf16 inputs."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from mamformer_b200.ops import gemm  # noqa: E402


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp(min=1e-6)).item()


def _bf(*shape, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, device="cuda", generator=g).bfloat16()


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 512, 256), (304, 200, 136), (1024, 4096, 4096),
                                   (384, 576, 512), (256, 1152, 256), (200, 400, 128)])
def test_dense_tn(M, N, K):
    a, b = _bf(M, K, seed=1), _bf(N, K, seed=2)
    out = gemm.mm(a, b)
    torch.cuda.synchronize()
    gemm.check_error()
    assert _rel(out, a.float() @ b.float().t()) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (200, 320, 192), (256, 576, 128)])
def test_dense_nn(M, N, K):
    a, b = _bf(M, K, seed=3), _bf(K, N, seed=4)
    out = gemm.mm_nn(a, b, out_dtype=torch.float32)
    torch.cuda.synchronize()
    gemm.check_error()
    assert _rel(out, a.float() @ b.float()) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 128, 192), (512, 576, 384), (300, 72, 136)])
def test_dense_wgrad_accumulate(M, N, K):
    dy, x = _bf(M, N, seed=5), _bf(M, K, seed=6)
    out = torch.randn(N, K, device="cuda")
    ref = out + dy.float().t() @ x.float()
    gemm.mm_tn_acc(dy, x, out, accumulate=True)
    torch.cuda.synchronize()
    gemm.check_error()
    assert _rel(out, ref) < 1e-2


def _segments(counts, align=64):
    seg = [0]
    for c in counts:
        seg.append(seg[-1] + (c + align - 1) // align * align)
    return seg


@pytest.mark.parametrize("N", [256, 576])
def test_grouped_m_and_k(N):
    """N = 576 (the MoE expert width) runs the 192-wide tile."""
    counts = [70, 0, 256, 5, 130, 64]
    G, K = len(counts), 192
    seg = _segments(counts)
    Mt = seg[-1]
    x = torch.zeros(Mt, K, device="cuda").bfloat16()
    for g, c in enumerate(counts):
        if c:
            x[seg[g]:seg[g] + c] = _bf(c, K, seed=10 + g)
    w = _bf(G, N, K, seed=7)
    seg_t = torch.tensor(seg, device="cuda", dtype=torch.int32)
    to = gemm.tile_offsets(seg_t)
    y = gemm.grouped_mm(x, w, seg_t, to)
    wt = _bf(G, K, N, seed=8)
    y2 = gemm.grouped_mm_nn(x, wt, seg_t, to, out_dtype=torch.float32)
    dy = torch.zeros(Mt, N, device="cuda").bfloat16()
    for g, c in enumerate(counts):
        if c:
            dy[seg[g]:seg[g] + c] = _bf(c, N, seed=30 + g)
    dw0 = torch.randn(G, N, K, device="cuda")
    dw = dw0.clone()
    gemm.grouped_wgrad(dy, x, seg_t, dw, accumulate=True)
    torch.cuda.synchronize()
    gemm.check_error()
    for g, c in enumerate(counts):
        rows = slice(seg[g], seg[g] + c)
        if c:
            assert _rel(y[rows], x[rows].float() @ w[g].float().t()) < 1e-2, g
            assert _rel(y2[rows], x[rows].float() @ wt[g].float()) < 1e-2, g
            assert _rel(dw[g], dw0[g] + dy[rows].float().t() @ x[rows].float()) < 1e-2, g
        else:
            assert torch.equal(dw[g], dw0[g])


@pytest.mark.parametrize("M,K,N,bias", [(4096, 1024, 512, False), (300, 256, 72, True)])
def test_fused_linear_matches_torch(M, K, N, bias):
    import torch.nn as nn
    from mamformer_b200.ops.linear import FusedLinear, use_native_linear
    torch.manual_seed(0)
    ref = nn.Linear(K, N, bias=bias).cuda().bfloat16()
    mod = nn.Linear(K, N, bias=bias).cuda().bfloat16()
    mod.load_state_dict(ref.state_dict())
    assert use_native_linear(mod) == 1 and isinstance(mod, FusedLinear)  # the root module itself
    x = torch.randn(M, K, device="cuda").bfloat16()
    xr, xn = x.clone().requires_grad_(), x.clone().requires_grad_()
    yr, yn = ref(xr), mod(xn)
    assert (yn.float() - yr.float()).norm() / yr.float().norm() < 1e-2
    g = torch.randn_like(yr)
    yr.backward(g)
    yn.backward(g)
    for a, b in ((xn.grad, xr.grad), (mod.weight.grad, ref.weight.grad)):
        assert (a.float() - b.float()).norm() / b.float().norm() < 2e-2
    mod.weight.main_grad = torch.zeros(N, K, device="cuda")
    mod.weight.grad = None
    mod(xn).backward(g)
    assert mod.weight.grad is None
    assert (mod.weight.main_grad - ref.weight.grad.float()).norm() / ref.weight.grad.float().norm() < 2e-2
