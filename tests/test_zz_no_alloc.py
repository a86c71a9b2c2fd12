"""The allocation-free GroupNorm forward, called through its exported C symbol.

Some callers cannot allocate device memory while they run an op (custom allocator hooks,
hosts that forbid allocation after start-up, foreign runtimes that pass in buffers and a
stream only).  ``mamf_head_groupnorm_fwd_noalloc`` serves them: it takes caller-owned inputs
and outputs and keeps its statistics in a fixed array inside the library.  This test calls it
twice in a row through ctypes and compares each result with the regular GroupNorm entry point.
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


def _call(fn, err, x, w, b, H, eps, mr=None):
    B, S, Cdim = x.shape
    y = torch.empty_like(x)
    dtype = 1 if x.dtype == torch.bfloat16 else 0
    rc = fn(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), None if mr is None else mr.data_ptr(),
            B, S, H, Cdim // H, eps, dtype, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, err().decode()
    return y


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 3e-2)])
def test_noalloc_groupnorm_matches_regular_entry_point(dtype, tol):
    C, fn, err = _lib()
    torch.manual_seed(0)
    cases = [(2, 300, 8, 64), (3, 70, 4, 128)]          # two calls in a row, different shapes
    for (B, S, H, hd) in cases:
        x = (torch.randn(B, S, H * hd, device="cuda") * 2 + 0.3).to(dtype)
        w = 1 + 0.1 * torch.randn(H * hd, device="cuda")
        b = 0.1 * torch.randn(H * hd, device="cuda")
        y = _call(fn, err, x, w, b, H, 1e-6)
        y_ref, _ = C.head_groupnorm_fwd(x, H, w, b, 1e-6)
        torch.cuda.synchronize()
        scale = y_ref.float().abs().max().item()
        assert (y.float() - y_ref.float()).abs().max().item() <= tol * scale


def test_noalloc_rejects_oversized_problem():
    C, fn, err = _lib()
    x = torch.zeros(1, 64, 64, device="cuda")
    w = torch.ones(64, device="cuda")
    b = torch.zeros(64, device="cuda")
    y = torch.empty_like(x)
    # B*H*ceil(S/64)*3 floats: B=1024, H=512, S=64 -> 1.5M > 1M (the kernel never runs)
    rc = fn(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), None, 1024, 64, 512, 1, 1e-6, 0,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 2 and b"scratch" in err()
