"""Bounded in-kernel waits: a barrier whose peer never arrives times out (~2 s), records an
error code and returns; the host raises CommTimeoutError and the GPU stays usable."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_barrier_timeout_is_reported_not_hung():
    from mamformer_b200.fault import CommTimeoutError, check_device_status
    from mamformer_b200.ops._ext import require_native
    C = require_native()
    check_device_status()
    mine = torch.zeros(512, dtype=torch.int32, device="cuda")
    fake_peer = torch.zeros(512, dtype=torch.int32, device="cuda")     # nobody writes rank 1's flag
    C.ep_barrier([mine.data_ptr(), fake_peer.data_ptr()], 0, 1, 0)
    torch.cuda.synchronize()
    with pytest.raises(CommTimeoutError):
        check_device_status()
    check_device_status()                                              # cleared
    x = torch.randn(1024, device="cuda")
    assert torch.isfinite((x @ x).reshape(1)).all()                    # context still usable
