"""The fused projection producer (ops.proj_rope / ks_proj_rope) vs cuBLAS and the
oracle (baseline/indexer.py:170-175, RoPE :114-129).

Gates:
  * the GEMM output (no RoPE, no scale) equals F.linear on the GPU and the
    oracle's exactly-rounded product bit for bit except rare bf16 flips from
    the fp32 accumulation order (<= 0.1 %, one bf16 ulp each);
  * RoPE and the weight scaling in the epilogue are exact: the rotated output is
    the oracle's RoPE of the kernel's own unrotated output, the scaled output is
    bf16(float(y) * scale) of it.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import bf16_from_bits, bits_from_bf16
from oracle import ks_oracle as O

pytestmark = pytest.mark.gpu


def _freqs(S, rd, pos0=0):
    inv = 1.0 / (10000.0 ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))
    ang = torch.outer(torch.arange(pos0, pos0 + S, dtype=torch.float32), inv)
    return torch.stack([ang.cos(), ang.sin()], -1).contiguous()


def _ulp_close(a_bits, b_bits):
    """Differing values are one bf16 rounding apart: within 2^-7 relative, or a few
    fp32 accumulation errors absolute where the exact sum is near zero."""
    a, b = O.bf16_to_f32(a_bits), O.bf16_to_f32(b_bits)
    return bool(np.all(np.abs(a - b) <= np.abs(b) * 2.0 ** -7 + 1e-5))


CASES = [
    # B, S, K, H, hd, rd
    (2, 300, 256, 16, 64, 32),      # the reference's geometry (q_lora_rank 256)
    (1, 128, 1024, 64, 128, 64),    # DSA geometry
    (1, 77, 72, 4, 128, 64),        # ragged rows, K not a multiple of 64
    (3, 40, 512, 32, 64, 16),
]


@pytest.mark.parametrize("B,S,K,H,hd,rd", CASES)
def test_proj_rope(cuda_ok, B, S, K, H, hd, rd):
    from kernelswift_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(B * 100 + S + K)
    a = torch.randn(B, S, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(H * hd, K, device="cuda", generator=g) * K ** -0.5).bfloat16()
    fr_host = _freqs(S, rd, 11)
    fr = fr_host.cuda()
    y = ops.proj_rope(a, w)
    yr = ops.proj_rope(a, w, hd, rd, fr)
    ys = ops.proj_rope(a, w, scale=0.0625 * 0.7)
    ops.device_status()
    ref = bits_from_bf16(F.linear(a, w))
    mine = bits_from_bf16(y)
    flips = mine != ref
    assert flips.mean() <= 1e-3 and _ulp_close(mine, ref), f"vs cuBLAS: {flips.mean():.2e}"
    exact = O.f32_to_bf16((a.double().cpu().numpy() @ w.double().cpu().numpy().T).astype(np.float32))
    fl = mine != exact
    assert fl.mean() <= 1e-3 and _ulp_close(mine, exact), f"vs oracle: {fl.mean():.2e}"
    # RoPE on the last rd of every head: exactly the oracle's rotation of y
    rot = O.rope_last(mine.reshape(B, S, H, hd), fr_host.numpy(), rd).reshape(B, S, H * hd)
    assert np.array_equal(bits_from_bf16(yr), rot)
    sc = O.f32_to_bf16((O.bf16_to_f32(mine) * np.float32(0.0625 * 0.7)).astype(np.float32))
    assert np.array_equal(bits_from_bf16(ys), sc)


def test_weights_projection(cuda_ok):
    """weights_proj(x) * (D^-0.5 H^-0.5): N = H columns (a 16-wide tile)."""
    from kernelswift_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(8, 260, 1024, device="cuda", generator=g).bfloat16()
    wp = (torch.randn(16, 1024, device="cuda", generator=g) * 0.03).bfloat16()
    scale = 64 ** -0.5 * 16 ** -0.5
    got = ops.proj_rope(x, wp, scale=scale)
    ops.device_status()
    ref = F.linear(x, wp) * scale
    a, b = bits_from_bf16(got), bits_from_bf16(ref)
    assert (a != b).mean() <= 2e-3 and _ulp_close(a, b)
