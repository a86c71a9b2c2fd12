"""tcgen05 flash-attention forward (csrc/flash_tc.cu) against fp32 PyTorch references of the same
op: differential attention (output and the gradients dq1, dq2, dk, dv, d lambda, whose backward
runs the flash backward kernels on the saved per-map outputs / log-sum-exps) and GQA head pairs,
for causal, windowed and look-ahead bands, ragged sequence lengths and several KV groupings."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from mamformer_b200.ops import reference as ref  # noqa: E402

BIG = 1 << 30


def _rel(a, b, floor=1e-6):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp(min=floor)).item()


# Gradient comparisons use an absolute floor: with the one-key diagonal band the exact dq / dk
# are zero (softmax over a single key has no gradient), and only rounding noise is left.
GFLOOR = 0.05


def _qkv(B, S, H, G, seed, Skv=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    Skv = S if Skv is None else Skv
    mk = lambda *s: (torch.randn(*s, device="cuda", generator=g) * 0.7).bfloat16()  # noqa: E731
    return mk(B, S, H, 128), mk(B, S, H, 128), mk(B, Skv, G, 128), mk(B, Skv, G, 128)


BANDS = [(-BIG, 0), (-255, 0), (0, 200), (0, 0)]


@pytest.mark.parametrize("B,S,H,G", [(1, 256, 4, 2), (2, 300, 8, 2), (1, 130, 2, 1)])
@pytest.mark.parametrize("band", BANDS)
def test_diff_forward_and_grads_match_fp32(B, S, H, G, band):
    from mamformer_b200.ops import native
    lo, hi = band
    q1, q2, k, v = _qkv(B, S, H, G, seed=S + H)
    lam = torch.linspace(0.2, 0.8, H, device="cuda")
    leaves = [t.clone().requires_grad_() for t in (q1, q2, k, v, lam)]
    out = native._DiffFlashTC.apply(*leaves[:4], leaves[4], lo, hi, 128 ** -0.5)
    import mamformer_b200._C as C
    assert C.flash_tc_error() == 0
    rl = [t.detach().float().clone().requires_grad_() for t in (q1, q2, k, v, lam)]
    want = ref.diff_attention_band(*rl[:4], rl[4], lo, hi)
    assert _rel(out, want) < 2e-2, _rel(out, want)
    dout = torch.randn_like(want)
    (out.float() * dout).sum().backward()
    (want * dout).sum().backward()
    # d lambda sums dout . (o1 - o2) / (1 - lam)^2: o1 - o2 is a small difference of two averages
    # formed with bf16 probabilities (as in any flash kernel), so it carries a few % of error
    tols = {"dq1": 3e-2, "dq2": 3e-2, "dk": 3e-2, "dv": 3e-2, "dlam": 6e-2}
    for name, a, b in zip(["dq1", "dq2", "dk", "dv", "dlam"], leaves, rl):
        assert _rel(a.grad, b.grad, GFLOOR) < tols[name], (name, _rel(a.grad, b.grad, GFLOOR))


@pytest.mark.parametrize("B,S,H,G", [(1, 256, 4, 2), (2, 333, 8, 2), (1, 512, 8, 1)])
@pytest.mark.parametrize("band", BANDS)
def test_gqa_pair_forward_and_grads_match_fp32(B, S, H, G, band):
    from mamformer_b200.ops import native
    lo, hi = band
    q, _, k, v = _qkv(B, S, H, G, seed=7 * S + H)
    leaves = [t.clone().requires_grad_() for t in (q, k, v)]
    out = native._FlashTCPair.apply(*leaves, lo, hi, 128 ** -0.5)
    rl = [t.detach().float().clone().requires_grad_() for t in (q, k, v)]
    want = ref.attention_band(*rl, lo, hi)
    assert _rel(out, want) < 2e-2, _rel(out, want)
    dout = torch.randn_like(want)
    (out.float() * dout).sum().backward()
    (want * dout).sum().backward()
    for name, a, b in zip(["dq", "dk", "dv"], leaves, rl):
        assert _rel(a.grad, b.grad, GFLOOR) < 3e-2, (name, _rel(a.grad, b.grad, GFLOOR))


def test_rows_without_keys_give_zero_and_infinite_lse():
    import mamformer_b200._C as C
    q1, q2, k, v = _qkv(1, 128, 2, 1, seed=3)
    lam = torch.full((2,), 0.5, device="cuda")
    # band entirely after the sequence end: no query row has a key
    out, o1, o2, lse1, lse2, od = C.flash_tc_fwd(q1, q2, k, v, lam, 1000, 2000, 128 ** -0.5)
    torch.cuda.synchronize()
    assert C.flash_tc_error() == 0
    assert torch.count_nonzero(out) == 0 and torch.isinf(lse1).all() and torch.isinf(lse2).all()


def test_model_level_diff_attention_uses_the_tcgen05_forward():
    """ops.diff_attention at head_dim 128 takes the tcgen05 path and matches the two-pass path."""
    from mamformer_b200.ops import native
    q1, q2, k, v = _qkv(1, 256, 4, 2, seed=11)
    lam = torch.full((4,), 0.4, device="cuda")
    a = native.diff_attention(q1, q2, k, v, lam, -BIG, 0)
    o1 = native.flash_attention(q1, k, v, -BIG, 0)
    o2 = native.flash_attention(q2, k, v, -BIG, 0)
    b = (o1.float() - 0.4 * o2.float()) / (1 - 0.4 + 1e-8)
    assert _rel(a, b) < 2e-2
