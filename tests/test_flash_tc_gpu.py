"""tcgen05 flash attention (forward csrc/flash_tc.cu, backward csrc/flash_tc_bwd.cu) against fp32
PyTorch references of the same op: differential attention (output and the gradients dq1, dq2, dk,
dv, d lambda; one backward launch over both maps with the per-head dout factors applied inside the
kernel), GQA head pairs and single heads, for causal, windowed and look-ahead bands, ragged
sequence lengths, key sequences longer than the queries and several KV groupings."""

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
    assert C.flash_tc_bwd_error() == 0


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
    import mamformer_b200._C as C
    assert C.flash_tc_bwd_error() == 0


@pytest.mark.parametrize("B,S,Skv,H,G", [(1, 200, 200, 6, 2), (2, 190, 320, 4, 4), (1, 64, 64, 3, 1)])
@pytest.mark.parametrize("band", BANDS)
def test_single_head_backward_matches_fp32(B, S, Skv, H, G, band):
    """Odd query heads per KV head (the mma.sync forward) and keys longer than the queries
    (queries aligned to the end of the keys): gradients from the tcgen05 backward."""
    from mamformer_b200.ops import native
    import mamformer_b200._C as C
    lo, hi = band
    q, _, k, v = _qkv(B, S, H, G, seed=S + 3 * Skv + H, Skv=Skv)
    leaves = [t.clone().requires_grad_() for t in (q, k, v)]
    out = native._FlashAttn.apply(*leaves, lo, hi, 128 ** -0.5)
    rl = [t.detach().float().clone().requires_grad_() for t in (q, k, v)]
    want = ref.attention_band(*rl, lo, hi)
    assert _rel(out, want) < 2e-2, _rel(out, want)
    dout = torch.randn_like(want)
    (out.float() * dout).sum().backward()
    (want * dout).sum().backward()
    for name, a, b in zip(["dq", "dk", "dv"], leaves, rl):
        assert _rel(a.grad, b.grad, GFLOOR) < 3e-2, (name, _rel(a.grad, b.grad, GFLOOR))
    assert C.flash_tc_bwd_error() == 0


def test_backward_of_rows_without_keys_is_zero():
    import mamformer_b200._C as C
    q, _, k, v = _qkv(1, 128, 2, 1, seed=5)
    q2 = torch.cat([q, q], 2)                      # two query heads on one KV head (pair mode)
    out, lse = C.flash_tc_fwd(q2, None, k, v, None, 1000, 2000, 128 ** -0.5)
    dq, dk, dv = C.flash_tc_bwd(q2, None, k, v, out, None, lse, None, torch.randn_like(out), None, 1000, 2000,
                                128 ** -0.5)
    torch.cuda.synchronize()
    assert C.flash_tc_bwd_error() == 0
    assert torch.count_nonzero(dq) == 0 and torch.count_nonzero(dk) == 0 and torch.count_nonzero(dv) == 0


def test_diff_backward_matches_two_single_map_backwards():
    """The fused two-map backward equals the sum of two single-map tcgen05 backwards run with
    dO1 = c1 dout and dO2 = c2 dout (to bf16 rounding of the dout factors)."""
    import mamformer_b200._C as C
    q1, q2, k, v = _qkv(2, 320, 8, 2, seed=21)
    lam = torch.linspace(0.1, 0.7, 8, device="cuda")
    lo, hi, sc = -BIG, 0, 128 ** -0.5
    out, o1, o2, lse1, lse2, od = C.flash_tc_fwd(q1, q2, k, v, lam, lo, hi, sc)
    dout = torch.randn_like(out)
    den = 1.0 / (1.0 - lam + 1e-8)
    coef = torch.stack([den, -lam * den])
    dq1, dq2, dk, dv = C.flash_tc_bwd(q1, q2, k, v, o1, o2, lse1, lse2, dout, coef, lo, hi, sc)
    do1 = (dout.float() * den.view(1, 1, -1, 1)).bfloat16()
    do2 = (dout.float() * (-lam * den).view(1, 1, -1, 1)).bfloat16()
    a1, ak1, av1 = C.flash_tc_bwd(q1, None, k, v, o1, None, lse1, None, do1, None, lo, hi, sc)
    a2, ak2, av2 = C.flash_tc_bwd(q2, None, k, v, o2, None, lse2, None, do2, None, lo, hi, sc)
    torch.cuda.synchronize()
    assert C.flash_tc_bwd_error() == 0
    assert _rel(dq1, a1, GFLOOR) < 2e-2 and _rel(dq2, a2, GFLOOR) < 2e-2
    assert _rel(dk, ak1.float() + ak2.float(), GFLOOR) < 2e-2
    assert _rel(dv, av1.float() + av2.float(), GFLOOR) < 2e-2


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
