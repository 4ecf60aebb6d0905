"""Sinkhorn kernel vs the golden fixtures and the oracle (baseline/sinkhorn.py:13-19)."""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden
from oracle import ks_oracle as O

SK = sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN, "sk_*.npz")))
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", SK)
def test_golden(cuda_ok, name):
    from kernelswift_b200 import ops

    d = load_golden(name)
    out = ops.sinkhorn(torch.from_numpy(d["x"]).cuda(), int(d["repeat"]), float(d["eps"]))
    ops.device_status()
    np.testing.assert_allclose(out.cpu().numpy(), d["out"], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("shape,repeat", [
    ((8, 4096, 4, 4), 20),     # C1
    ((2, 32768, 8, 8), 20),    # the Sinkhorn stage of C5
    ((3, 7, 5, 5), 10),
    ((1, 129, 2, 2), 3),
    ((1, 5, 16, 16), 20),
    ((2, 3, 33, 33), 2),
    ((1, 1, 1, 1), 5),
    ((4, 33, 4, 4), 0),
])
def test_vs_oracle(cuda_ok, shape, repeat):
    from kernelswift_b200 import ops

    x = torch.randn(*shape, generator=torch.Generator().manual_seed(sum(shape)))
    out = ops.sinkhorn(x.cuda(), repeat, 1e-6)
    ops.device_status()
    ref = O.sinkhorn(x.numpy(), repeat, 1e-6)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=1e-6)
    # the reference harness tolerance
    assert torch.allclose(out.cpu(), torch.from_numpy(ref), rtol=1e-2, atol=1e-2)


def test_in_place_and_repeatable(cuda_ok):
    from kernelswift_b200 import ops

    x = torch.randn(1, 1000, 4, 4, device="cuda")
    a = ops.sinkhorn(x, 20, 1e-6)
    b = ops.sinkhorn(x, 20, 1e-6)
    assert torch.equal(a, b)
    y = x.clone()
    ops.sinkhorn(y, 20, 1e-6, out=y)
    assert torch.equal(y, a)


def test_rejects_bad_input(cuda_ok):
    from kernelswift_b200 import ops

    with pytest.raises(RuntimeError):
        ops.sinkhorn(torch.randn(2, 4, 4, device="cuda").double())
    with pytest.raises(RuntimeError):
        ops.sinkhorn(torch.randn(2, 4, 5, device="cuda"))
