"""One process driving two GPUs: every op runs on cuda:0 and then on cuda:1.

The library sets each kernel's shared-memory opt-in per device (the attribute
belongs to the current device's context), so a launch on the second device must
work after the first device's.  Skipped when fewer than two GPUs are visible."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(3, 70, 8, 8, device=dev, generator=g)
    xw = torch.randn(2, 5, 12, 12, device=dev, generator=g)  # warp-per-matrix path
    q = torch.randn(1, 3, 64, 128, device=dev, generator=g).bfloat16()
    kv = torch.randn(1, 500, 128, device=dev, generator=g).bfloat16()
    idx = torch.randint(0, 500, (1, 3, 96), device=dev, generator=g).int()
    sink = torch.randn(64, device=dev, generator=g)
    qi = torch.randn(1, 96, 64, 128, device=dev, generator=g).bfloat16()
    ki = torch.randn(1, 300, 128, device=dev, generator=g).bfloat16()
    wi = (torch.rand(1, 96, 64, device=dev, generator=g) * 0.01).bfloat16()
    return x, xw, q, kv, idx, sink, qi, ki, wi


def _run(dev, args):
    from kernelswift_b200 import ops

    x, xw, q, kv, idx, sink, qi, ki, wi = args
    with torch.cuda.device(dev):
        r = (ops.sinkhorn(x, 20), ops.sinkhorn(xw, 5),
             ops.sparse_attn(q, kv, sink, idx, 128 ** -0.5),
             ops.indexer_topk(qi, ki, wi, None, 0, 300, 64, pos0=200))
        ops.device_status(dev)
    return r


def test_each_op_on_two_devices(cuda_ok):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    a0 = _case(d0, 5)
    r0 = _run(d0, a0)
    a1 = tuple(t.to(d1) for t in a0)
    r1 = _run(d1, a1)
    for x, y in zip(r0, r1):
        assert y.device == d1
        assert torch.equal(x.cpu(), y.cpu())
