"""FP8 indexer kernels vs the oracle (operator contract of ks_quant_fp8_rows /
ks_indexer_fp8; the reference declares ModelArgs.dtype = "fp8" but implements no
FP8 path, so these gates rest on the oracle alone).

Gates:
  * the row quantiser: e4m3 codes and scales equal the oracle's exactly;
  * FP8 scores: equal the oracle's (exact dot products rounded once to fp32,
    then the fp32 head chain) except rare bf16 flips where the tensor cores'
    accumulation of the 128 products rounds differently; every flip is small;
  * top-k: exact, in order, on the kernel's own scores; rows whose indices differ
    from the oracle's are rows with a flip.
"""
import numpy as np
import pytest
import torch

from helpers import bf16_from_bits, bits_from_bf16
from oracle import ks_oracle as O

pytestmark = pytest.mark.gpu


def _u8(t):
    return t.contiguous().view(torch.uint8).cpu().numpy()


def test_quant_rows_bit_exact(cuda_ok):
    from kernelswift_b200 import ops

    rng = np.random.default_rng(5)
    x = (rng.standard_normal((300, 128)) * np.exp(rng.uniform(-12, 12, (300, 1)))).astype(np.float32)
    x[7] = 0.0
    x[8, :5] = [448.0, -448.0, 1e-30, -1e-30, -0.0]
    x[9] = np.float32(3e38) * np.sign(rng.standard_normal(128))
    xb = O.f32_to_bf16(x)
    x8, s = ops.quant_fp8_rows(bf16_from_bits(xb))
    ops.device_status()
    codes, ref_s = O.quant_fp8_rows(xb)
    assert np.array_equal(s.cpu().numpy(), ref_s)
    assert np.array_equal(_u8(x8), codes)
    # other row lengths (multiples of 4) and a leading batch shape
    xb2 = O.f32_to_bf16(rng.standard_normal((2, 3, 36)).astype(np.float32))
    y8, s2 = ops.quant_fp8_rows(bf16_from_bits(xb2))
    c2, r2 = O.quant_fp8_rows(xb2)
    assert np.array_equal(_u8(y8), c2) and np.array_equal(s2.cpu().numpy(), r2)


def _case(B, S, T, H, seed):
    """Quantised queries / keys the way a caller makes them: bf16 rows -> e4m3 +
    power-of-two scale per row; w = head weight x query scale (fp32)."""
    from kernelswift_b200 import ops

    rng = np.random.default_rng(seed)
    q = bf16_from_bits(O.f32_to_bf16(rng.standard_normal((B, S, H, 128)).astype(np.float32)))
    k = bf16_from_bits(O.f32_to_bf16(rng.standard_normal((B, T, 128)).astype(np.float32)))
    q8, qs = ops.quant_fp8_rows(q)
    k8, ks = ops.quant_fp8_rows(k)
    hw = torch.from_numpy(rng.uniform(-1, 1, (B, S, H)).astype(np.float32)).cuda()
    w = (hw * qs * (128 ** -0.5 * H ** -0.5)).contiguous()
    return q8, k8, w, ks


GEOMS = [
    # B, S, T, H, k, ratio, start_pos, offset, pos0
    (1, 512, 512, 64, 256, 1, 0, 0, 0),     # DSA heads, causal
    (2, 200, 50, 16, 128, 4, 0, 0, 0),      # ratio 4, T < k
    (1, 130, 300, 32, 64, 1, 170, 9, 0),    # decode-style: no mask, + offset
    (1, 256, 1024, 64, 512, 1, 0, 0, 768),  # a shard of a prefill
    (3, 33, 33, 16, 8, 1, 0, 0, 0),         # ragged S
]


@pytest.mark.parametrize("B,S,T,H,k,ratio,sp,off,pos0", GEOMS)
def test_fp8_indexer_vs_oracle(cuda_ok, B, S, T, H, k, ratio, sp, off, pos0):
    from kernelswift_b200 import ops

    q8, k8, w, ks = _case(B, S, T, H, seed=B * 7 + S + T)
    causal = sp == 0
    sc = bits_from_bf16(ops.indexer_scores_fp8(q8, k8, w, ks, T, ratio, causal, pos0))[:, :, :T]
    idx = ops.indexer_topk_fp8(q8, k8, w, ks, T, k, ratio, causal, off, pos0).cpu().numpy()
    ops.device_status()
    ref = O.indexer_scores_fp8(_u8(q8), _u8(k8), w.cpu().numpy(), ks.cpu().numpy(), causal, ratio, pos0)
    lim = O.indexer_limits(S, pos0, causal, ratio, T)
    valid = np.broadcast_to(np.arange(T)[None, None, :] < lim[None, :, None], sc.shape)
    a, r = O.bf16_to_f32(sc), O.bf16_to_f32(ref)
    flips = (a != r) & valid                       # value compare: +0 == -0
    assert flips.mean() <= 2e-3, f"score flips {flips.mean():.2e}"
    assert np.allclose(a[valid], r[valid], rtol=1e-2, atol=1e-3)
    own = np.where(valid, sc, O.NEG_INF_BF16).astype(np.uint16)
    kk = min(k, T)
    assert np.array_equal(idx, O.indexer_postprocess(O.topk_stable(own, kk), S, pos0, causal, ratio, off))
    ref_idx = O.indexer_postprocess(O.topk_stable(ref, kk), S, pos0, causal, ratio, off)
    bad_rows = np.any(idx != ref_idx, axis=-1)
    assert not np.any(bad_rows & ~np.any(flips, axis=-1))


def test_fp8_agrees_with_bf16_selection(cuda_ok):
    """The FP8 path selects nearly the same keys as the bf16 path on the same
    (un-quantised) inputs: a sanity check of scales and layout, not a parity gate."""
    from kernelswift_b200 import ops

    rng = np.random.default_rng(11)
    B, S, T, H, k = 1, 256, 2048, 64, 256
    q = bf16_from_bits(O.f32_to_bf16(rng.standard_normal((B, S, H, 128)).astype(np.float32)))
    kx = bf16_from_bits(O.f32_to_bf16(rng.standard_normal((B, T, 128)).astype(np.float32)))
    hw = torch.from_numpy(rng.uniform(0, 1, (B, S, H)).astype(np.float32)).cuda()
    scale = 128 ** -0.5 * H ** -0.5
    i16 = ops.indexer_topk(q, kx, (hw * scale).bfloat16(), None, 0, T, k, causal=False)
    q8, qs = ops.quant_fp8_rows(q)
    k8, ks = ops.quant_fp8_rows(kx)
    i8 = ops.indexer_topk_fp8(q8, k8, (hw * qs * scale).contiguous(), ks, T, k, causal=False)
    ops.device_status()
    a, b = i16.cpu().numpy(), i8.cpu().numpy()
    recall = np.mean([len(np.intersect1d(a[0, s], b[0, s])) / k for s in range(S)])
    assert recall > 0.8, recall
