"""The allocation-free GroupNorm forward, called through its exported C symbol.

Some callers cannot allocate device memory while they run an op (custom allocator hooks,
hosts that forbid allocation after start-up, foreign runtimes that pass in buffers and a
stream only).  ``mamf_head_groupnorm_fwd_noalloc`` serves them: it takes caller-owned inputs
and outputs and keeps its statistics in a fixed array inside the library.  This test calls it
twice in a row through ctypes and compares each result with the regular GroupNorm entry point
(same kernels, so the outputs must be bitwise equal), with the statistics both in the library's
array and in caller memory, on the current and on a side stream, and against an fp32 PyTorch
group norm for head sizes that do not fill whole warps.
Kept in its own file that sorts last, so a stop-at-first-failure run has done everything else.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import mamformer_b200._C as C   # loads the extension (and torch) first
    lib = ctypes.CDLL(C.__file__)
    fn = lib.mamf_head_groupnorm_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                   ctypes.c_int, ctypes.c_void_p]
    err = lib.mamf_noalloc_last_error
    err.restype = ctypes.c_char_p
    return C, fn, err


def _call(fn, err, x, w, b, H, eps, mr=None, stream=None):
    B, S, Cdim = x.shape
    y = torch.empty_like(x)
    dtype = 1 if x.dtype == torch.bfloat16 else 0
    st = stream if stream is not None else torch.cuda.current_stream()
    rc = fn(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), None if mr is None else mr.data_ptr(),
            B, S, H, Cdim // H, eps, dtype, st.cuda_stream)
    assert rc == 0, err().decode()
    assert err() == b""
    return y


def _inputs(B, S, H, hd, dtype):
    x = (torch.randn(B, S, H * hd, device="cuda") * 2 + 0.3).to(dtype)
    w = 1 + 0.1 * torch.randn(H * hd, device="cuda")
    b = 0.1 * torch.randn(H * hd, device="cuda")
    return x, w, b


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_groupnorm_matches_regular_entry_point(dtype):
    C, fn, err = _lib()
    torch.manual_seed(0)
    cases = [(2, 300, 8, 64), (3, 70, 4, 128)]          # two calls in a row, different shapes
    for (B, S, H, hd) in cases:
        x, w, b = _inputs(B, S, H, hd, dtype)
        y = _call(fn, err, x, w, b, H, 1e-6)
        y_ref, mr_ref = C.head_groupnorm_fwd(x, H, w, b, 1e-6)
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_statistics_in_caller_memory_on_a_side_stream(dtype):
    C, fn, err = _lib()
    torch.manual_seed(1)
    side = torch.cuda.Stream()
    for (B, S, H, hd) in [(2, 130, 4, 64), (1, 64, 2, 128)]:
        x, w, b = _inputs(B, S, H, hd, dtype)
        y_ref, mr_ref = C.head_groupnorm_fwd(x, H, w, b, 1e-6)
        mr = torch.full((B * H, 2), float("nan"), device="cuda")
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            y = _call(fn, err, x, w, b, H, 1e-6, mr=mr, stream=side)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref)
        assert torch.equal(mr, mr_ref.view(B * H, 2))


@pytest.mark.parametrize("hd", [4, 100])
def test_noalloc_head_sizes_that_do_not_fill_a_warp(hd):
    """hd = 4 and 100 give stats blocks whose x extent is not a multiple of 8 before rounding;
    both entry points must still match an fp32 torch group norm."""
    C, fn, err = _lib()
    torch.manual_seed(2)
    B, S, H = 2, 77, 3
    x, w, b = _inputs(B, S, H, hd, torch.float32)
    y = _call(fn, err, x, w, b, H, 1e-6)
    y_reg, _ = C.head_groupnorm_fwd(x, H, w, b, 1e-6)
    xt = x.double().transpose(1, 2)                                # (B, C, S): groups = heads
    want = torch.nn.functional.group_norm(xt, H, w.double(), b.double(), 1e-6).transpose(1, 2)
    torch.cuda.synchronize()
    assert torch.equal(y, y_reg)
    assert (y.double() - want).abs().max().item() < 1e-4


def test_noalloc_rejects_oversized_and_out_of_range_problems():
    C, fn, err = _lib()
    x = torch.zeros(1, 64, 64, device="cuda")
    w = torch.ones(64, device="cuda")
    b = torch.zeros(64, device="cuda")
    y = torch.empty_like(x)
    st = torch.cuda.current_stream().cuda_stream
    # B*H*ceil(S/64)*3 floats: B=1024, H=512, S=64 -> 1.5M > 1M (the kernel never runs)
    rc = fn(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), None, 1024, 64, 512, 1, 1e-6, 0, st)
    assert rc == 2 and b"scratch" in err()
    rc = fn(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), None, 70000, 1, 1, 64, 1e-6, 0, st)
    assert rc == 1 and b"65535" in err()
    rc = fn(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), None, 1, 1, 2, 2 ** 31, 1e-6, 0, st)
    assert rc == 1 and b"int32" in err()
