"""Failure detection without a GPU fault: a kernel whose barrier nobody completes
gives up after a short budget, reports the timeout through the status word, and
the context stays usable."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout(cuda_ok):
    from kernelswift_b200 import _lib, ops

    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.ks_selftest_wait_timeout(50_000_000, stream), "selftest")  # 50 ms
    with pytest.raises(_lib.KsError) as e:
        ops.device_status()
    assert e.value.code == _lib.KS_ERR_DEVICE
    ops.device_status()  # cleared
    x = torch.randn(1, 64, 4, 4, device="cuda")
    y = ops.sinkhorn(x, 3, 1e-6)
    ops.device_status()
    assert torch.isfinite(y).all()
