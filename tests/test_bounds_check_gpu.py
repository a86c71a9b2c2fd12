"""The bounds-checked build of the index-driven kernels (module ``mamformer_b200._C_check``):
an index outside its buffer is recorded in the file's error word and skipped, never accessed.

Every out-of-range index used here still lands inside a larger allocation that the tested
buffer is a view of, so even a missing guard could not touch memory outside this process's
tensors; the test then sees the stray write instead."""

import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


def _check():
    return importlib.import_module("mamformer_b200._C_check")


def test_main_module_is_unchecked_and_check_module_is_checked():
    import mamformer_b200._C as C
    assert not C.bounds_check_built()
    assert _check().bounds_check_built()


def test_scatter_rows_skips_and_records_a_bad_row():
    C = _check()
    C.bounds_error_moe_rows()                                   # clear
    big = torch.zeros(64, 128, device="cuda", dtype=torch.bfloat16)
    dst = big[:32]
    src = torch.randn(4, 128, device="cuda").bfloat16()
    idx = torch.tensor([0, 5, 40, 3], device="cuda")
    C.moe_scatter_rows(dst, idx, src, 1)
    torch.cuda.synchronize()
    assert C.bounds_error_moe_rows() == 1101
    assert C.bounds_error_moe_rows() == 0                       # read clears
    assert torch.equal(big[0], src[0]) and torch.equal(big[5], src[1]) and torch.equal(big[3], src[3])
    assert torch.count_nonzero(big[32:]) == 0                   # the bad row was never written


def test_combine_skips_a_row_past_its_table():
    C = _check()
    big = torch.randn(64, 64, device="cuda").bfloat16()
    rows = big[:16]
    out = torch.empty(2, 64, device="cuda", dtype=torch.bfloat16)
    pos = torch.tensor([1, 2, 3, 50], device="cuda")            # token 1's second row is out of range
    w = torch.ones(4, device="cuda")
    C.moe_combine(out, [rows.data_ptr()], 64, 16, torch.bfloat16, None, pos, w, 2, None)
    torch.cuda.synchronize()
    assert C.bounds_error_moe_rows() == 1102
    want0 = (rows[1].float() + rows[2].float()).bfloat16()
    assert torch.equal(out[0], want0)
    assert torch.equal(out[1], rows[3])                         # only the in-range row was summed


def test_cross_entropy_records_a_label_outside_the_vocabulary():
    C = _check()
    logits = torch.randn(4, 64, device="cuda").bfloat16()
    labels = torch.tensor([1, 70, -100, 3], device="cuda")
    loss = torch.empty(4, device="cuda")
    lse = torch.empty(4, device="cuda")
    C.ce_stats(logits, labels, -100, loss, lse)
    torch.cuda.synchronize()
    assert C.bounds_error_ce() == 1201
    assert loss[1].item() == 0.0 and loss[2].item() == 0.0
    want = torch.logsumexp(logits.float(), -1) - logits.float()[torch.arange(4), labels.clamp(0, 63)]
    assert abs(loss[0].item() - want[0].item()) < 1e-2


def test_ignore_index_is_not_an_error():
    C = _check()
    logits = torch.randn(2, 64, device="cuda").bfloat16()
    labels = torch.tensor([-100, 5], device="cuda")
    loss, lse = torch.empty(2, device="cuda"), torch.empty(2, device="cuda")
    C.ce_stats(logits, labels, -100, loss, lse)
    torch.cuda.synchronize()
    assert C.bounds_error_ce() == 0
