"""Pin the numpy oracle against the golden fixtures produced by the reference's
own PyTorch modules (tests/golden/make_golden.py).  CPU only."""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_golden
from oracle import ks_oracle as O

SK = sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN, "sk_*.npz")))
SA = sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN, "sa_*.npz")))
IX = sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN, "ix_*.npz")))


def test_fixture_inventory():
    assert len(SK) >= 5 and len(SA) >= 5 and len(IX) >= 4


@pytest.mark.parametrize("name", SK)
def test_sinkhorn_oracle(name):
    d = load_golden(name)
    out = O.sinkhorn(d["x"], int(d["repeat"]), float(d["eps"]))
    np.testing.assert_allclose(out, d["out"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", SA)
def test_sparse_attn_oracle(name):
    d = load_golden(name)
    out = O.sparse_attn(d["q"], d["kv"], d["sink"], d["idx"], float(d["scale"]))
    a, b = O.bf16_to_f32(out), O.bf16_to_f32(d["out"])
    assert (out == d["out"]).mean() > 0.999          # fp32 summation order only
    np.testing.assert_allclose(a, b, rtol=8e-3, atol=2e-3)  # at most ~1 bf16 ulp


@pytest.mark.parametrize("name", IX)
def test_indexer_rope_oracle(name):
    d = load_golden(name)
    rd = int(d["meta"][4])
    assert np.array_equal(O.rope_last(d["q_pre"], d["freqs"], rd), d["q_rope"])


@pytest.mark.parametrize("name", IX)
def test_indexer_score_oracle(name):
    d = load_golden(name)
    B, S, H, D, rd, k, ratio, sp, off = (int(v) for v in d["meta"])
    T = d["kv"].shape[1]
    sc = O.indexer_scores(d["q_rope"], d["kv"], d["w"], sp == 0, ratio)
    lim = O.indexer_limits(S, 0, sp == 0, ratio, T)
    valid = np.arange(T)[None, None, :] < lim[None, :, None]
    same = (sc == d["scores"]) | ~valid
    # GEMM accumulation order differs from oneDNN's: rare 1-ulp-class flips only
    assert same.mean() > 0.999
    ka = O.bf16_order_key(sc).astype(np.int64)
    kb = O.bf16_order_key(d["scores"]).astype(np.int64)
    assert np.abs(ka - kb)[np.broadcast_to(valid, ka.shape)].max() <= 16


@pytest.mark.parametrize("name", IX)
def test_indexer_topk_oracle_ties_only(name):
    """The stable oracle applied to the reference's own scores selects the same
    value sequence as the reference's torch.topk; any index difference is a
    reordering among equal scores (torch's CPU tie order is unspecified)."""
    d = load_golden(name)
    B, S, H, D, rd, k, ratio, sp, off = (int(v) for v in d["meta"])
    T = d["kv"].shape[1]
    g = d["scores"].copy()
    lim = O.indexer_limits(S, 0, sp == 0, ratio, T)
    for s in range(S):
        g[:, s, lim[s]:] = O.NEG_INF_BF16
    kk = min(k, T)
    mine = O.indexer_postprocess(O.topk_stable(g, kk), S, 0, sp == 0, ratio, off)
    ref = d["out"]
    assert mine.shape == ref.shape
    assert np.array_equal(mine < 0, ref < 0)
    key = O.bf16_order_key(g).astype(np.int64)

    def values(ix):
        raw = np.where(ix < 0, 0, ix - off)
        return np.where(ix < 0, -1, np.take_along_axis(key, raw, axis=-1))

    assert np.array_equal(values(mine), values(ref))


def test_topk_stable_tie_rule():
    # value descending, then index ascending; -0.0 == +0.0; -inf last
    vals = np.array([1.0, 2.0, 2.0, 2.0, 0.0, -0.0, -np.inf, 0.0], np.float32)
    bits = O.f32_to_bf16(vals)
    bits[5] = 0x8000
    assert O.topk_stable(bits[None], 8)[0].tolist() == [1, 2, 3, 0, 4, 5, 7, 6]


def test_bf16_round_trip():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.5, 65504.0], np.float32)
    assert np.array_equal(O.bf16_to_f32(O.f32_to_bf16(x)), O.round_bf16(x))
    # ties round to even
    assert O.f32_to_bf16(np.array([1.00390625], np.float32))[0] == 0x3F80
