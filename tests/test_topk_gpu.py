"""Top-k kernel: bit-exact against the stable oracle (value desc, index asc) with
the indexer's mask and post-processing (baseline/indexer.py:185-205)."""
import numpy as np
import pytest
import torch

from helpers import bf16_from_bits, rand_bf16_bits
from oracle import ks_oracle as O

pytestmark = pytest.mark.gpu


def oracle_topk(sc, T, k, ratio, causal, offset, pos0):
    B, S, _ = sc.shape
    s = sc[:, :, :T].copy()
    lim = O.indexer_limits(S, pos0, causal, ratio, T)
    for i in range(S):
        s[:, i, lim[i]:] = O.NEG_INF_BF16
    idx = O.topk_stable(s, min(k, T))
    return O.indexer_postprocess(idx, S, pos0, causal, ratio, offset)


CASES = [
    # B, S, T, k, ratio, causal, offset, pos0, quant
    (1, 300, 300, 64, 1, True, 0, 0, None),
    (2, 129, 1000, 128, 4, True, 5, 0, None),
    (1, 64, 777, 2048, 1, False, 100, 0, None),      # k > T: all T returned
    (1, 50, 5000, 2048, 1, False, 7, 0, 4),           # heavy ties
    (1, 96, 4096, 2048, 1, True, 0, 2000, 2),         # shard rows, ties at the threshold
    (3, 17, 65, 16, 1, True, 0, 0, 1),                # T not a multiple of 8
    (1, 8, 40000, 4096, 1, False, 0, 0, None),        # k = 4096, long rows
    (1, 4, 65536, 2048, 1, False, 0, 0, 8),           # maximum T
    # the one-warp-per-row path (T <= 2048, k <= 256) and its edges
    (2, 40, 2048, 256, 1, True, 3, 2000, 2),          # longest warp-path rows, ties
    (1, 40, 2049, 256, 1, False, 0, 0, None),         # one key past it: row kernel
    (1, 40, 1000, 257, 1, False, 0, 0, 4),            # k past it: row kernel
    (4, 33, 513, 33, 1, False, 9, 0, 1),              # k = 33 (64-wide sort), coarse ties
]


@pytest.mark.parametrize("B,S,T,k,ratio,causal,offset,pos0,quant", CASES)
@pytest.mark.parametrize("dtype", [torch.int64, torch.int32])
def test_topk_exact(cuda_ok, B, S, T, k, ratio, causal, offset, pos0, quant, dtype):
    from kernelswift_b200 import ops

    ld = (T + 7) // 8 * 8
    sc = rand_bf16_bits((B, S, ld), seed=B * 7 + S + T, scale=3.0, quant=quant)
    out = ops.topk_rows(bf16_from_bits(sc), T, k, ratio, causal, offset, pos0, dtype)
    ops.device_status()
    ref = oracle_topk(sc, T, k, ratio, causal, offset, pos0)
    got = out.cpu().numpy().astype(np.int64)
    assert got.shape == ref.shape
    bad = np.argwhere(got != ref)
    assert bad.size == 0, f"{len(bad)} mismatches, first at {bad[:3].tolist()}"


def test_all_equal_and_signed_zero(cuda_ok):
    from kernelswift_b200 import ops

    T = 1024
    sc = np.zeros((1, 3, T), np.uint16)
    sc[0, 1, ::2] = 0x8000          # -0.0 == +0.0
    sc[0, 2, 100:200] = 0x3F80      # 1.0 block, rest 0
    out = ops.topk_rows(bf16_from_bits(sc), T, 256, 1, False, 0, 0)
    ref = oracle_topk(sc, T, 256, 1, False, 0, 0)
    assert np.array_equal(out.cpu().numpy(), ref)
    assert out[0, 0].tolist() == list(range(256))


def test_dsa_prefill_shape(cuda_ok):
    """C3's geometry: 4096 causal rows over 4096 keys, k = 2048."""
    from kernelswift_b200 import ops

    T = 4096
    sc = rand_bf16_bits((1, 4096, T), seed=3, scale=2.0, quant=16)
    out = ops.topk_rows(bf16_from_bits(sc), T, 2048, 1, True, 0, 0)
    ops.device_status()
    ref = oracle_topk(sc, T, 2048, 1, True, 0, 0)
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("spread", ["narrow", "wide"])
def test_counting_and_bitonic_sort_paths(cuda_ok, spread):
    """The kernel sorts a row's selection with a stable counting sort when the
    selected keys span at most 128 bf16 values and with a bitonic sort otherwise;
    both must give the stable oracle's order.  Narrow rows mimic indexer scores
    (values in [1.5, 2.5): about 100 distinct bf16 keys, heavy ties); wide rows
    spread over many exponents, so the selection spans thousands of keys."""
    from kernelswift_b200 import ops

    B, S, T, k = 1, 64, 6000, 2048
    rng = np.random.default_rng(11 if spread == "narrow" else 12)
    if spread == "narrow":
        x = rng.uniform(1.5, 2.5, (B, S, T)).astype(np.float32)
    else:
        x = (rng.standard_normal((B, S, T)) * np.exp2(rng.integers(-20, 20, (B, S, T)))).astype(np.float32)
    sc = O.f32_to_bf16(x)
    span = len(np.unique(np.sort(sc[0, 0].view(np.int16).astype(np.int64))[-k:]))
    assert (span <= 128) == (spread == "narrow")
    for dtype in (torch.int32, torch.int64):
        out = ops.topk_rows(bf16_from_bits(sc), T, k, 1, True, 3, 4000, dtype)
        ops.device_status()
        ref = oracle_topk(sc, T, k, 1, True, 3, 4000)
        assert np.array_equal(out.cpu().numpy().astype(np.int64), ref)
