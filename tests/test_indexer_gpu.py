"""Indexer kernels vs the golden fixtures and the oracle (baseline/indexer.py:161-206).

Gates:
  * RoPE + score kernel: scores equal the oracle's bit for bit except for rare
    bf16 rounding flips caused by a different fp32 accumulation order in the
    q.k GEMM (tensor cores vs the host BLAS); every flip is small.
  * top-k: the fused call's indices equal, exactly and in order, the stable
    top-k of the kernel's own scores.
  * end to end: rows whose indices differ from the oracle's are exactly rows
    whose scores carry such a flip.
"""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden
from helpers import bf16_from_bits, bits_from_bf16, rand_bf16_bits
from oracle import ks_oracle as O

IX = sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN, "ix_*.npz")))
pytestmark = pytest.mark.gpu


def run_case(q_pre, kv, w, freqs, rd, k, ratio, start_pos, offset, pos0=0):
    from kernelswift_b200 import ops

    B, S = q_pre.shape[:2]
    T = kv.shape[1]
    causal = start_pos == 0
    qg, kg, wg = bf16_from_bits(q_pre), bf16_from_bits(kv), bf16_from_bits(w)
    fg = torch.from_numpy(np.ascontiguousarray(freqs, np.float32)).cuda()
    sc = ops.indexer_scores(qg, kg, wg, fg, rd, T, ratio, causal, pos0)
    idx = ops.indexer_topk(qg, kg, wg, fg, rd, T, k, ratio, causal, offset, pos0)
    ops.device_status()
    return bits_from_bf16(sc)[:, :, :T], idx.cpu().numpy()


def check(q_pre, kv, w, freqs, rd, k, ratio, start_pos, offset, pos0=0, max_flip=1e-3):
    B, S = q_pre.shape[:2]
    T = kv.shape[1]
    causal = start_pos == 0
    sc, idx = run_case(q_pre, kv, w, freqs, rd, k, ratio, start_pos, offset, pos0)
    lim = O.indexer_limits(S, pos0, causal, ratio, T)
    valid = np.broadcast_to(np.arange(T)[None, None, :] < lim[None, :, None], sc.shape)
    ref_sc = O.indexer_scores(O.rope_last(q_pre, freqs, rd), kv, w, causal, ratio, pos0)
    flips = (sc != ref_sc) & valid
    assert flips.mean() <= max_flip, f"score flips {flips.mean():.2e}"
    # a flip moves a score by about one bf16 ulp of one head's product: small in absolute terms
    a, r = O.bf16_to_f32(sc)[valid], O.bf16_to_f32(ref_sc)[valid]
    assert np.allclose(a, r, rtol=1e-2, atol=1e-2)
    # top-k exact on the kernel's own scores
    own = sc.copy()
    own[~valid] = O.NEG_INF_BF16
    kk = min(k, T)
    exp_own = O.indexer_postprocess(O.topk_stable(own, kk), S, pos0, causal, ratio, offset)
    assert np.array_equal(idx, exp_own)
    # end to end: differences only where scores flipped
    ref_idx = O.indexer_postprocess(O.topk_stable(ref_sc, kk), S, pos0, causal, ratio, offset)
    bad_rows = np.any(idx != ref_idx, axis=-1)
    flip_rows = np.any(flips, axis=-1)
    assert not np.any(bad_rows & ~flip_rows)
    return sc, idx


@pytest.mark.parametrize("name", IX)
def test_golden(cuda_ok, name):
    d = load_golden(name)
    B, S, H, D, rd, k, ratio, sp, off = (int(v) for v in d["meta"])
    sc, idx = check(d["q_pre"], d["kv"], d["w"], d["freqs"], rd, k, ratio, sp, off)
    # vs the reference's own scores and indices (ties may reorder: value sequences equal)
    T = d["kv"].shape[1]
    lim = O.indexer_limits(S, 0, sp == 0, ratio, T)
    valid = np.broadcast_to(np.arange(T)[None, None, :] < lim[None, :, None], sc.shape)
    assert ((sc == d["scores"]) | ~valid).mean() > 0.999
    assert idx.shape == d["out"].shape and np.array_equal(idx < 0, d["out"] < 0)
    # The kernel's indices against the reference's own torch.topk output, read as
    # sequences of the reference's score values: torch's CPU tie order is
    # unspecified, so equal values may come in another index order, but the value
    # sequence must match, except in rows where the kernel's scores carry a flip.
    ref_sc = np.where(valid, d["scores"], O.NEG_INF_BF16)
    key = O.bf16_order_key(ref_sc).astype(np.int64)

    def values(ix):
        raw = np.where(ix < 0, 0, ix - off)
        return np.where(ix < 0, -1, np.take_along_axis(key, raw, axis=-1))

    differ = np.any(values(idx) != values(d["out"]), axis=-1)
    flipped = np.any((sc != d["scores"]) & valid, axis=-1)
    assert not np.any(differ & ~flipped), "index value sequences differ in rows without a flip"


GEOMS = [
    # B, S, T, H, D, rd, k, ratio, start_pos, offset, pos0
    (1, 512, 512, 64, 128, 64, 256, 1, 0, 0, 0),       # DSA heads, causal
    (2, 200, 50, 16, 64, 32, 128, 4, 0, 0, 0),         # reference geometry, ratio 4, T < k
    (1, 130, 300, 32, 128, 64, 64, 1, 170, 9, 0),      # decode-style, no mask
    (1, 256, 1024, 64, 128, 64, 512, 1, 0, 0, 768),    # a shard: rows 768..1023 of a prefill
    (3, 33, 33, 16, 128, 0, 8, 1, 0, 0, 0),            # no RoPE, ragged S
]


@pytest.mark.parametrize("B,S,T,H,D,rd,k,ratio,sp,off,pos0", GEOMS)
def test_random(cuda_ok, B, S, T, H, D, rd, k, ratio, sp, off, pos0):
    seed = B * 1000 + S + T
    q = rand_bf16_bits((B, S, H, D), seed)
    kv = rand_bf16_bits((B, T, D), seed + 1)
    rng = np.random.default_rng(seed + 2)
    w = O.f32_to_bf16((rng.uniform(-1, 1, (B, S, H)) * (D ** -0.5 * H ** -0.5)).astype(np.float32))
    pos = np.arange(pos0 + sp, pos0 + sp + S, dtype=np.float32)
    inv = 1.0 / (10000.0 ** (np.arange(0, rd, 2, dtype=np.float32) / max(rd, 1)))
    ang = np.outer(pos, inv).astype(np.float32)
    freqs = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32).reshape(S, rd // 2, 2)
    check(q, kv, w, freqs, rd, k, ratio, sp, off, pos0)


def test_shard_equals_slice_of_full_call(cuda_ok):
    """Rows computed in a shard (pos0 > 0) equal the same rows of a whole call."""
    from kernelswift_b200 import ops

    B, S, T, H, D, rd = 1, 640, 640, 64, 128, 64
    q = bf16_from_bits(rand_bf16_bits((B, S, H, D), 5))
    kv = bf16_from_bits(rand_bf16_bits((B, T, D), 6))
    w = torch.rand(B, S, H, device="cuda").bfloat16() * 0.01
    ang = torch.outer(torch.arange(S).float(), 1.0 / (10000.0 ** (torch.arange(0, rd, 2).float() / rd)))
    freqs = torch.stack([ang.cos(), ang.sin()], -1).cuda()
    full = ops.indexer_topk(q, kv, w, freqs, rd, T, 256)
    a, b = 200, 456
    part = ops.indexer_topk(q[:, a:b].contiguous(), kv, w[:, a:b].contiguous(),
                            freqs[a:b].contiguous(), rd, T, 256, pos0=a)
    ops.device_status()
    assert torch.equal(full[:, a:b], part)


def test_dsa_scale_rows(cuda_ok):
    """C3 geometry (S = T = 4096, H = 64, D = 128, k = 2048); oracle on row blocks."""
    from kernelswift_b200 import ops

    B, S, T, H, D, rd, k = 1, 4096, 4096, 64, 128, 64, 2048
    q = rand_bf16_bits((B, S, H, D), 21)
    kv = rand_bf16_bits((B, T, D), 22)
    rng = np.random.default_rng(23)
    w = O.f32_to_bf16((rng.uniform(0, 1, (B, S, H)) * (D ** -0.5 * H ** -0.5)).astype(np.float32))
    ang = np.outer(np.arange(S, dtype=np.float32),
                   1.0 / (10000.0 ** (np.arange(0, rd, 2, dtype=np.float32) / rd))).astype(np.float32)
    freqs = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
    sc, idx = run_case(q, kv, w, freqs, rd, k, 1, 0, 0)
    own = sc.copy()
    lim = O.indexer_limits(S, 0, True, 1, T)
    for s in range(S):
        own[:, s, lim[s]:] = O.NEG_INF_BF16
    assert np.array_equal(idx, O.indexer_postprocess(O.topk_stable(own, k), S, 0, True, 1, 0))
    q_rope = O.rope_last(q, freqs, rd)
    for s0 in (0, 1500, 4032):
        rows = slice(s0, s0 + 64)
        ref = O.indexer_scores(q_rope[:, rows], kv, w[:, rows], True, 1, s0)
        valid = np.arange(T)[None, None, :] < lim[rows][None, :, None]
        flips = (sc[:, rows] != ref) & valid
        assert flips.mean() < 1e-3
