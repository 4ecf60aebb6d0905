"""SparseAttention drop-in: ``ModelNew`` with the interface of KernelSwift's
baseline/sparse_attention.py (constructor ``(n_heads, head_dim)``, parameter
``attn_sink``, ``forward(q, kv, topk_idxs)``, ``get_inputs``,
``get_init_inputs``), running the tcgen05 kernel of libks_b200.so.
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


class ModelNew(nn.Module):
    """Top-k sparse MQA attention with sinks (baseline/sparse_attention.py:45-65)."""

    def __init__(self, n_heads: int, head_dim: int):
        super().__init__()
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.softmax_scale = head_dim ** -0.5
        self.attn_sink = nn.Parameter(torch.zeros(n_heads, dtype=torch.float32))

    def forward(self, q: torch.Tensor, kv: torch.Tensor, topk_idxs: torch.Tensor) -> torch.Tensor:
        return _ops().sparse_attn(q, kv, self.attn_sink, topk_idxs, self.softmax_scale)


batch_size = 8
seq_len = 2600
n_kv = 32
n_heads = 64
head_dim = 128
topk = 16


def get_inputs():
    q = torch.randn(batch_size, seq_len, n_heads, head_dim, dtype=torch.bfloat16)
    kv = torch.randn(batch_size, n_kv, head_dim, dtype=torch.bfloat16)
    topk_idxs = torch.randint(0, n_kv, (batch_size, seq_len, topk), dtype=torch.int32)
    return [q, kv, topk_idxs]


def get_init_inputs():
    return [n_heads, head_dim]
