"""Native flash attention (GQA, band masks) and differential attention against fp32 PyTorch."""
import pytest
import torch

from mamformer_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
BIG = 1 << 30


def _rel(a, b):
    # relative error, with an absolute floor for gradients that are analytically ~0 (e.g. dq of a
    # diagonal-only band, where dS = P (dP - D) cancels exactly)
    floor = 1e-2 * b.numel() ** 0.5
    return ((a.float() - b.float()).norm() / max(b.float().norm().item(), floor)).item()


@pytest.mark.parametrize("B,S,H,G,hd,lo,hi", [
    (2, 200, 8, 2, 64, -BIG, 0),          # causal, ragged length
    (1, 256, 4, 4, 128, -BIG, 0),
    (1, 300, 8, 2, 128, -63, 0),          # causal sliding window 64
    (1, 190, 4, 1, 128, 0, 31),           # reference GQA window quirk (keys at / after the query)
    (1, 128, 4, 2, 64, 0, 0),             # diagonal only
])
def test_flash_attention_fwd_bwd(B, S, H, G, hd, lo, hi):
    from mamformer_b200.ops import native
    torch.manual_seed(0)
    mk = lambda h: torch.randn(B, S, h, hd, device="cuda").bfloat16()
    q, k, v = mk(H), mk(G), mk(G)
    ins = [t.clone().requires_grad_() for t in (q, k, v)]
    out = native.flash_attention(*ins, lo=lo, hi=hi)
    ins_r = [t.float().clone().requires_grad_() for t in (q, k, v)]
    want = ref.attention_band(*ins_r, lo, hi)
    assert _rel(out, want) < 1e-2, _rel(out, want)
    g = torch.randn_like(want)
    out.backward(g.bfloat16())
    want.backward(g)
    for a, b, n in zip(ins, ins_r, "qkv"):
        assert _rel(a.grad, b.grad) < 2e-2, (n, _rel(a.grad, b.grad))


def test_diff_attention_native():
    from mamformer_b200.ops import native
    torch.manual_seed(1)
    B, S, H, G, hd = 1, 256, 4, 2, 128
    q1, q2 = (torch.randn(B, S, H, hd, device="cuda").bfloat16() for _ in range(2))
    k, v = (torch.randn(B, S, G, hd, device="cuda").bfloat16() for _ in range(2))
    lam = torch.tensor([0.2, 0.5, 0.7, 0.9], device="cuda", requires_grad=True)
    out = native.diff_attention(q1, q2, k, v, lam, -BIG, 0)
    want = ref.diff_attention_band(q1.float(), q2.float(), k.float(), v.float(), lam, -BIG, 0)
    assert _rel(out, want) < 2e-2
    out.float().sum().backward()
    assert lam.grad is not None and torch.isfinite(lam.grad).all()
