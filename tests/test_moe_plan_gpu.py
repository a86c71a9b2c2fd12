"""Device-side MoE routing plans (``csrc/moe_rows.cu``): the counting sort against the eager
sort, and the expert-parallel layout / positions / row pull with P ranks emulated in one process
(every "rank" is a buffer on this GPU, so no barrier or peer memory is involved; the count
exchange itself runs in the multi-GPU tests)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _skewed_idx(T, k, E, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    # skewed scores so some experts get many rows and some none
    bias = torch.linspace(-3, 3, E, device="cuda")
    scores = torch.randn(T, E, device="cuda", generator=g) + bias
    scores[:, E // 3] = -1e9                               # one expert never chosen
    return torch.topk(scores, k).indices


@pytest.mark.parametrize("T,k,E", [(1000, 8, 128), (4096, 2, 16), (7, 3, 5), (33000, 8, 256)])
def test_native_sort_plan_matches_eager(T, k, E):
    from mamformer_b200.ops.moe import plan, plan_eager
    idx = _skewed_idx(T, k, E, seed=T)
    pos, seg, tile_off, counts, rows = plan(idx, E)
    pos_e, seg_e, tile_e, counts_e = plan_eager(idx.reshape(-1).long(), E)
    assert torch.equal(pos, pos_e)
    assert torch.equal(seg.cpu(), seg_e.cpu())
    assert torch.equal(tile_off.cpu(), tile_e.cpu())
    assert torch.equal(counts.long().cpu(), counts_e.cpu())
    assert int(seg[-1]) <= rows


def test_bias_update_kernel_matches_eager_bitwise():
    from mamformer_b200.models.moe import _update_expert_bias
    E, T, k = 128, 16384, 8
    counts = torch.randint(0, 3 * T * k // E, (E,), device="cuda")
    b1 = torch.randn(E, device="cuda") * 1e-3
    e1 = torch.rand(E, device="cuda") / E
    b2, e2 = b1.clone(), e1.clone()
    _update_expert_bias(counts, T, E, k, 0.001, b1, e1)                     # native
    with torch.no_grad():                                                   # eager float32 ops
        load = counts.float() / (T * k + 1e-8)
        b2 -= 0.001 * torch.sign(load - 1.0 / E)
        e2.mul_(0.99).add_(0.01 * load)
    assert torch.equal(b1, b2) and torch.equal(e1, e2)


def _emulated_ep(P, El, T, k, d, cap_factor, seed=0):
    """Run sort -> stage -> layout -> positions -> pull for P emulated ranks; return what each
    owner pulled and the expected rows."""
    import mamformer_b200._C as C
    E = P * El
    Q = T * k
    xs = [torch.randn(T, d, device="cuda").bfloat16() for _ in range(P)]
    idxs = [_skewed_idx(T, k, E, seed + 17 * r).reshape(-1).long().contiguous() for r in range(P)]
    sorts = [C.moe_sort_plan(i, E, False) for i in idxs]                   # srow, counts, start
    stages = []
    for r in range(P):
        st = torch.empty(Q, d, device="cuda", dtype=torch.bfloat16)
        C.moe_scatter_rows(st, sorts[r][0], xs[r], k)
        stages.append(st)
    Cmat = torch.stack([s[1] for s in sorts]).contiguous()                 # (P, E) int32
    cap = (int(min(P, cap_factor) * Q) + 64 * El + 127) // 128 * 128
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    pulled, plans, positions = [], [], []
    for me in range(P):
        plan = torch.empty(C.ep_plan_size(P, El), dtype=torch.int32, device="cuda")
        C.ep_layout(Cmat, me, cap, plan, status)
        xp = torch.full((cap, d), float("nan"), device="cuda", dtype=torch.bfloat16)
        C.ep_pull_rows(xp, [s.data_ptr() for s in stages], d, Q, plan, P)
        pos = torch.empty(Q, dtype=torch.int64, device="cuda")
        owner = torch.empty(Q, dtype=torch.int32, device="cuda")
        C.ep_positions(idxs[me], sorts[me][0], sorts[me][2], plan, P, cap, pos, owner)
        pulled.append(xp)
        plans.append(plan)
        positions.append((pos, owner))
    return xs, idxs, Cmat, cap, status, pulled, plans, positions


def test_ep_layout_pull_and_positions_emulated():
    P, El, T, k, d = 4, 8, 300, 4, 64
    xs, idxs, Cmat, cap, status, pulled, plans, positions = _emulated_ep(P, El, T, k, d, cap_factor=P)
    assert int(status[0]) == 0
    E = P * El
    Cc = Cmat.cpu()
    for me in range(P):
        plan = plans[me].cpu()
        seg = plan[: El + 1]
        xp = pulled[me]
        # expected: per local expert, rows of sender 0, 1, ... in assignment order, then zero pad
        for le in range(El):
            e = me * El + le
            rows = []
            for s in range(P):
                q = (idxs[s] == e).nonzero().flatten()
                rows.append(xs[s][q // k])
            want = torch.cat(rows) if rows else xs[0][:0]
            n = want.shape[0]
            assert n == int(Cc[:, e].sum())
            got = xp[int(seg[le]): int(seg[le + 1])]
            assert got.shape[0] == (n + 63) // 64 * 64
            assert torch.equal(got[:n], want)
            assert torch.count_nonzero(got[n:]) == 0
        tiles = plan[El + 1: 2 * El + 2]
        want_tiles = torch.cat([torch.zeros(1, dtype=torch.int64),
                                torch.cumsum((seg[1:] - seg[:-1] + 127) // 128, 0)])
        assert torch.equal(tiles.long(), want_tiles)
    # every assignment's row sits at pos[q] of its owner's buffer
    for r in range(P):
        pos, owner = positions[r]
        for o in range(P):
            sel = (owner == o).nonzero().flatten()
            assert torch.equal(pulled[o][pos[sel]], xs[r][sel // k])
        assert torch.equal(owner.long(), idxs[r] // El)


def test_ep_layout_flags_an_owner_over_capacity():
    P, El, T, k, d = 4, 4, 256, 8, 64
    # capacity factor 1 with skewed routing: the busiest owner needs more rows than T*k + pads
    xs, idxs, Cmat, cap, status, pulled, plans, positions = _emulated_ep(P, El, T, k, d, cap_factor=1.0)
    need = max(int(sum(((int(Cmat[:, o * El + le].sum()) + 63) // 64 * 64) for le in range(El))) for o in range(P))
    assert need > cap
    assert int(status[0]) == 1 and int(status[1]) == need
    for me in range(P):
        assert int(plans[me][El]) <= cap                    # clamped: every access stays in bounds
        pos, _ = positions[me]
        assert int(pos.max()) < cap
