"""Host-side argument checks of kernelswift_b200.ops (no GPU needed).

The kernels write through raw pointers, so a caller-supplied output or workspace
that is too small, of the wrong type, strided or on another device must be
rejected before any launch."""
import pytest
import torch

from kernelswift_b200 import ops

CPU = torch.device("cpu")


def test_out_accepts_exact_buffer():
    ops._check_out("t", torch.empty(2, 3, 4, dtype=torch.bfloat16), (2, 3, 4), torch.bfloat16, CPU)


@pytest.mark.parametrize("out,why", [
    (torch.empty(2, 3, 4, dtype=torch.int32), "must be torch.bfloat16"),        # dtype
    (torch.empty(2, 3, 3, dtype=torch.bfloat16), "shape"),                      # too small
    (torch.empty(2, 3, 5, dtype=torch.bfloat16), "shape"),                      # too large
    (torch.empty(2, 4, 3, dtype=torch.bfloat16).transpose(1, 2), "contiguous"),  # strided view
    (torch.empty(2, 3, 4, dtype=torch.bfloat16, device="meta"), "must be on"),  # device
    ("not a tensor", "must be a tensor"),
])
def test_out_rejects(out, why):
    with pytest.raises(RuntimeError, match=why):
        ops._check_out("t", out, (2, 3, 4), torch.bfloat16, CPU)


def test_int64_request_rejects_int32_out():
    with pytest.raises(RuntimeError, match="int64"):
        ops._check_out("indexer", torch.empty(1, 4, 8, dtype=torch.int32), (1, 4, 8), torch.int64, CPU)


def test_workspace_sized_in_bytes():
    ops._check_workspace("t", torch.empty(256, dtype=torch.uint8), 256, CPU)
    ops._check_workspace("t", torch.empty(64, dtype=torch.float32), 256, CPU)  # 256 bytes
    with pytest.raises(RuntimeError, match="bytes needed"):
        ops._check_workspace("t", torch.empty(63, dtype=torch.float32), 256, CPU)


@pytest.mark.parametrize("ws,why", [
    (torch.empty(512, dtype=torch.uint8)[::2], "contiguous"),
    (torch.empty(256, dtype=torch.uint8, device="meta"), "must be on"),
    (None, "must be a tensor"),
])
def test_workspace_rejects(ws, why):
    with pytest.raises(RuntimeError, match=why):
        ops._check_workspace("t", ws, 256, CPU)


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: every op raises on host tensors."""
    x = torch.randn(4, 4, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.sinkhorn(x, 3)
    q = torch.randn(1, 2, 16, 128).bfloat16()
    kv = torch.randn(1, 8, 128).bfloat16()
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.sparse_attn(q, kv, torch.zeros(16), torch.zeros(1, 2, 4, dtype=torch.int32), 0.1)
