"""Native chunked KDA-Diff linear attention against the fp32 PyTorch form of the same operator."""
import pytest
import torch

from mamformer_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("B,S,H,G,hd,K", [(2, 200, 8, 2, 64, 64), (1, 256, 4, 4, 128, 128), (1, 130, 4, 1, 128, 64),
                                          (1, 1024, 8, 2, 128, 128), (2, 330, 8, 2, 128, 128)])
def test_linear_diff_attention_fwd_bwd(B, S, H, G, hd, K):
    from mamformer_b200.ops import native
    torch.manual_seed(0)
    dev = "cuda"
    mk = lambda h: (torch.randn(B, S, h, hd, device=dev) * 0.5).bfloat16()
    q1, q2, k, v = mk(H), mk(H), mk(G), mk(G)
    lam = torch.sigmoid(torch.randn(H, device=dev)).clamp(max=0.99)
    ins = [t.clone().requires_grad_() for t in (q1, q2, k, v)]
    lam_n = lam.clone().requires_grad_()
    out = native.linear_diff_attention(*ins, lam_n, K)
    assert out.dtype == torch.bfloat16
    ins_r = [t.float().clone().requires_grad_() for t in (q1, q2, k, v)]
    lam_r = lam.clone().requires_grad_()
    want = ref.linear_diff_attention_fp32(*ins_r, lam_r, K)
    assert _rel(out, want) < 1e-2, _rel(out, want)
    g = torch.randn_like(want)
    out.backward(g.bfloat16())
    want.backward(g)
    for a, b, n in zip(ins + [lam_n], ins_r + [lam_r], ("q1", "q2", "k", "v", "lam")):
        assert _rel(a.grad, b.grad) < 2e-2, (n, _rel(a.grad, b.grad))
