"""The reference's forwards restated in torch — TEST AND BASELINE INFRASTRUCTURE ONLY.

The reference's operators are PyTorch modules (baseline/sinkhorn.py,
baseline/sparse_attention.py, baseline/indexer.py of TtitiO/KernelSwift).  The
reference checkout does not travel to the GPU box, so these functions restate
their forward arithmetic with the same torch operations in the same order.  They
serve two purposes:

* the v0 side of the reference harness's comparison in tests/harness.py (run on
  the GPU, as auto_bench.py would run baseline/*.py there);
* the reference CPU implementation timed by bench.py (`cpu_baseline`,
  `--impl reference`): torch's CPU kernels on the host cores, which is what
  running baseline/*.py on the CPU executes.

They are pinned by tests/test_harness_cpu.py: built and run in the harness's
order at seed 42 they reproduce the reference modules' own outputs
(tests/golden/hx_*.npz, made by tests/golden/make_golden.py from baseline/*.py).
The numpy oracle (ks_oracle.py) remains the parity checker of the CUDA path.
Nothing under kernelswift_b200/ imports this module.
"""
from __future__ import annotations

import torch


def sinkhorn(x: torch.Tensor, repeat: int, eps: float) -> torch.Tensor:
    """baseline/sinkhorn.py:13-19."""
    y = x.softmax(-1) + eps
    y = y / (y.sum(-2, keepdim=True) + eps)
    for _ in range(repeat - 1):
        y = y / (y.sum(-1, keepdim=True) + eps)
        y = y / (y.sum(-2, keepdim=True) + eps)
    return y


def sparse_attn(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor,
                topk_idxs: torch.Tensor, softmax_scale: float) -> torch.Tensor:
    """baseline/sparse_attention.py:5-42: gather the selected kv rows (invalid ones
    zeroed), fp32 scores, -inf on invalid entries, softmax with the sink in the
    denominator, fp32 weighted sum, cast back to q's dtype."""
    B, M, H, D = q.shape
    K = topk_idxs.shape[-1]
    ok = topk_idxs >= 0
    rows = topk_idxs.clamp_min(0).long()
    bidx = torch.arange(B, device=q.device)[:, None, None].expand(B, M, K)
    g = kv[bidx, rows].masked_fill(~ok.unsqueeze(-1), 0.0)
    s = torch.einsum("bmhd,bmtd->bmht", q.float(), g.float()) * softmax_scale
    s = s.masked_fill(~ok.unsqueeze(2), float("-inf"))
    sink = attn_sink.float().view(1, 1, H, 1)
    z = torch.maximum(torch.amax(s, dim=-1, keepdim=True), sink)
    e = torch.exp(s - z).masked_fill(~ok.unsqueeze(2), 0.0)
    w = e / (e.sum(dim=-1, keepdim=True) + torch.exp(sink - z))
    return torch.einsum("bmht,bmtd->bmhd", w, g.float()).to(q.dtype)


def rope_inplace(x: torch.Tensor, freqs_cis: torch.Tensor) -> None:
    """baseline/indexer.py:114-129: rotate interleaved pairs of x (a view of
    [B, S, H, rd]) by the complex factors of its rows, in fp32, copied back."""
    cx = torch.view_as_complex(x.float().unflatten(-1, (-1, 2)))
    f = freqs_cis.view(1, cx.size(1), 1, cx.size(-1))
    x.copy_(torch.view_as_real(cx * f).flatten(-2))


def indexer_after_projections(q: torch.Tensor, weights: torch.Tensor, kv_cache: torch.Tensor,
                              freqs_cis: torch.Tensor, rope_dim: int, topk: int, ratio: int,
                              start_pos: int, offset: int, s0: int = 0):
    """baseline/indexer.py:171-205 after the two projections: q bf16 [B,S,H,D]
    (rotated in place), weights bf16 [B,S,H], kv_cache [B, >= end_pos//ratio, D],
    freqs_cis [S, rope_dim/2] complex (the rows' positions).  `s0` is the sequence
    position of row 0 when the rows are a slice of a prefill (start_pos == 0): it
    enters the causal mask (:187-191, :199-201) the way the rows' own positions do
    in the whole call.  Returns (indices int64 [B,S,k], masked bf16 scores)."""
    B, S = q.shape[:2]
    end_pos = start_pos + s0 + S
    rope_inplace(q[..., -rope_dim:], freqs_cis)
    sc = torch.einsum("bshd,btd->bsht", q, kv_cache[:B, : end_pos // ratio])
    sc = (sc.relu_() * weights.unsqueeze(-1)).sum(dim=2)
    if start_pos == 0:
        keys = torch.arange(end_pos // ratio, device=q.device).repeat(S, 1)
        lim = torch.arange(s0 + 1, s0 + S + 1, device=q.device).unsqueeze(1) // ratio
        sc += torch.where(keys >= lim, float("-inf"), 0.0)
    idx = sc.topk(min(topk, end_pos // ratio), dim=-1)[1]
    if start_pos == 0:
        lim = torch.arange(s0 + 1, s0 + S + 1, device=q.device).unsqueeze(1) // ratio
        return torch.where(idx >= lim, -1, idx + offset), sc
    return idx + offset, sc
