"""Sinkhorn drop-in: ``ModelNew`` with the interface of KernelSwift's
baseline/sinkhorn.py (constructor ``(repeat=10, eps=1e-6)``, ``forward(x)``,
``get_inputs``, ``get_init_inputs``), running the sm_100a kernel of
libks_b200.so.  Usable directly by the reference's harness
(benchmarks/ks/auto_bench.py --v1_file <this file>): every statement the
harness's AST filter drops is inside a function.
"""
import torch
import torch.nn as nn


def _ops():
    import os
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    from kernelswift_b200 import ops

    return ops


class Model(nn.Module):
    """Sinkhorn normalisation (baseline/sinkhorn.py:5-19) on the B200 kernel."""

    def __init__(self, repeat: int = 10, eps: float = 1e-6):
        super().__init__()
        self.repeat = repeat
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _ops().sinkhorn(x, self.repeat, self.eps)


class ModelNew(Model):
    pass


n0 = 1
n1 = 1024
mhc = 4


def get_inputs():
    x = torch.randn(n0, n1, mhc, mhc, dtype=torch.float32)
    return [x]


def get_init_inputs():
    return []
