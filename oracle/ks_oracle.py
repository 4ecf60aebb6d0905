"""CPU oracle for the three KernelSwift operators — TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA path.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import it; the product path in
``kernelswift_b200`` never does and has no CPU fallback.

It restates, in numpy, the reference's PyTorch modules of TtitiO/KernelSwift
(third-party arithmetic: PyTorch, pinned by the reference at 2.9.0; fixtures
were generated here with 2.11.0 CPU):

* ``sinkhorn``      <- baseline/sinkhorn.py:13-19
* ``sparse_attn``   <- baseline/sparse_attention.py:5-42
* ``rope_last``     <- baseline/indexer.py:114-129 applied as in :172
* ``indexer_scores``<- baseline/indexer.py:170-183 (+ causal mask :185-193)
* ``topk_stable`` / ``indexer_postprocess`` <- baseline/indexer.py:195-205

FP8 indexer (``e4m3_*``, ``quant_fp8_rows``, ``indexer_scores_fp8``): the
reference declares ``ModelArgs.dtype = "fp8"`` and ``scale_fmt = "ue8m0"``
(baseline/indexer.py:14-17) but its bf16 baseline never uses them and no FP8
kernel exists in the repository, so there is no reference output to pin these
against.  They restate the published e4m3 format (OCP 8-bit floating point:
1 sign, 4 exponent bits with bias 7, 3 mantissa bits, no infinities, largest
finite 448) and the operator contract stated in include/ks_b200.h; the e4m3
tables are checked exhaustively in tests/test_fp8_cpu.py.  Parity of the FP8
path is therefore "unpinned" against the reference.

The oracle is pinned against the golden fixtures in ``tests/golden`` that
``tests/golden/make_golden.py`` produced by running the reference's own modules
(see ``tests/test_oracle_golden.py``).

bf16 values travel as raw ``uint16`` bit patterns; rounding to bf16 is
round-to-nearest-even, as PyTorch's float->bfloat16 conversion.

Top-k tie rule: the reference calls ``torch.topk`` (baseline/indexer.py:196),
whose order among equal scores is unspecified (CPU torch does not keep index
order).  The oracle fixes it as value descending, then index ascending, which
is what ``torch.topk`` returns on CUDA and what the operator contract states.
``-0.0`` and ``+0.0`` compare equal, as in torch.
"""
from __future__ import annotations

import numpy as np

NEG_INF_BF16 = np.uint16(0xFF80)


# ---------------------------------------------------------------- bf16 helpers
def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    """Widen raw bf16 bits to float32 (exact)."""
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 bits, round-to-nearest-even (NaN is not expected)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_to_f32(f32_to_bf16(x))


# ---------------------------------------------------------------- Sinkhorn
def sinkhorn(x: np.ndarray, repeat: int = 10, eps: float = 1e-6) -> np.ndarray:
    """baseline/sinkhorn.py:13-19: softmax over the last dim, + eps, then column
    normalisation, then ``repeat-1`` rounds of (row, column) normalisation, each
    dividing by (sum + eps).  float32 throughout."""
    x = np.asarray(x, np.float32)
    eps = np.float32(eps)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m, dtype=np.float32)
    x = (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32) + eps
    x = (x / (x.sum(axis=-2, keepdims=True, dtype=np.float32) + eps)).astype(np.float32)
    for _ in range(repeat - 1):
        x = (x / (x.sum(axis=-1, keepdims=True, dtype=np.float32) + eps)).astype(np.float32)
        x = (x / (x.sum(axis=-2, keepdims=True, dtype=np.float32) + eps)).astype(np.float32)
    return x


# ---------------------------------------------------------------- SparseAttention
def sparse_attn(q: np.ndarray, kv: np.ndarray, sink: np.ndarray, idx: np.ndarray,
                scale: float, dv: int | None = None, rows: tuple[int, int] | None = None
                ) -> np.ndarray:
    """baseline/sparse_attention.py:5-42 on query rows ``rows=(m0, m1)`` (all rows
    by default).  q [B,M,H,D] bf16 bits, kv [B,N,D] bf16 bits, sink [H] f32,
    idx [B,M,K] int32.  Returns bf16 bits [B, m1-m0, H, dv].

    Steps (reference line numbers): valid = idx >= 0, clamp (:16-17); gather and
    zero invalid rows (:19-22); s = (q.g)*scale (:24-26); invalid -> -inf (:27);
    z = max(max_t s, sink_h) (:29-31); e = exp(s - z), invalid -> 0 (:33-34);
    den = sum e + exp(sink - z) (:35-36); out = sum_t (e/den) g (:37-41); cast (:42).
    Output columns are independent, so ``dv < D`` is ``ref[..., :dv]``."""
    B, M, H, D = q.shape
    dv = D if dv is None else dv
    m0, m1 = rows if rows is not None else (0, M)
    out = np.empty((B, m1 - m0, H, dv), np.uint16)
    sink = np.asarray(sink, np.float32)
    for b in range(B):
        kvb = bf16_to_f32(kv[b])
        for mi in range(m0, m1):
            ix = idx[b, mi].astype(np.int64)
            valid = ix >= 0
            g = kvb[np.maximum(ix, 0)]
            g[~valid] = 0.0
            qf = bf16_to_f32(q[b, mi])                          # [H, D]
            s = (qf @ g.T).astype(np.float32) * np.float32(scale)   # [H, K]
            s[:, ~valid] = -np.inf
            z = np.maximum(s.max(axis=1), sink)                 # [H]
            e = np.exp(s - z[:, None], dtype=np.float32)
            e[:, ~valid] = 0.0
            den = e.sum(axis=1, dtype=np.float32) + np.exp(sink - z, dtype=np.float32)
            w = (e / den[:, None]).astype(np.float32)
            o = (w @ g[:, :dv]).astype(np.float32)
            out[b, mi - m0] = f32_to_bf16(o)
    return out


# ---------------------------------------------------------------- Indexer
def rope_last(q_bits: np.ndarray, freqs: np.ndarray, rope_dim: int) -> np.ndarray:
    """baseline/indexer.py:114-129 applied to ``q[..., -rope_dim:]`` (:172).

    q [B,S,H,D] bf16 bits; freqs [S, rope_dim/2, 2] float32 (cos, sin) for the
    rows' positions.  Interleaved pairs (x[2j], x[2j+1]) are rotated by the
    complex factor in float32 — ``(a+bi)(c+di) = (ac-bd) + (ad+bc)i`` with each
    product and sum rounded separately — and the result is rounded back to bf16
    (the ``copy_`` into the bf16 view)."""
    out = np.array(q_bits, np.uint16, copy=True)
    D = q_bits.shape[-1]
    seg = bf16_to_f32(q_bits[..., D - rope_dim:])
    a = seg[..., 0::2]
    b = seg[..., 1::2]
    c = np.asarray(freqs[..., 0], np.float32)[None, :, None, :]
    d = np.asarray(freqs[..., 1], np.float32)[None, :, None, :]
    re = (a * c).astype(np.float32) - (b * d).astype(np.float32)
    im = (a * d).astype(np.float32) + (b * c).astype(np.float32)
    rot = np.empty_like(seg)
    rot[..., 0::2] = re
    rot[..., 1::2] = im
    out[..., D - rope_dim:] = f32_to_bf16(rot)
    return out


def indexer_limits(S: int, s0: int, causal: bool, ratio: int, T: int) -> np.ndarray:
    """Per-row count of valid keys: (s+1)//ratio for causal prefill rows
    (baseline/indexer.py:185-193, :199-202), else all T keys."""
    if causal:
        return np.minimum((np.arange(s0, s0 + S) + 1) // ratio, T)
    return np.full(S, T, np.int64)


def indexer_scores(q_rope: np.ndarray, k: np.ndarray, w: np.ndarray, causal: bool,
                   ratio: int, s0: int = 0) -> np.ndarray:
    """baseline/indexer.py:176-193 for query rows s0..s0+S-1.

    q_rope [B,S,H,D] bf16 bits (after RoPE), k [B,T,D] bf16 bits, w [B,S,H] bf16
    bits (already scaled by D^-0.5 H^-0.5 and rounded, :173-175).
    score = bf16(einsum) (:176-180); relu; bf16(score*w) (:181-182); fp32 sum over
    heads in head order, rounded to bf16 (:183); causal positions t >= (s+1)//ratio
    set to -inf (:185-193).  Returns bf16 bits [B,S,T]."""
    B, S, H, D = q_rope.shape
    T = k.shape[1]
    out = np.empty((B, S, T), np.uint16)
    lim = indexer_limits(S, s0, causal, ratio, T)
    for b in range(B):
        kf = bf16_to_f32(k[b])                                   # [T, D]
        for r0 in range(0, S, 64):
            r1 = min(S, r0 + 64)
            qf = bf16_to_f32(q_rope[b, r0:r1]).reshape(-1, D)    # [(s,h), D]
            sc = round_bf16((qf @ kf.T).astype(np.float32)).reshape(r1 - r0, H, T)
            sc = np.maximum(sc, np.float32(0.0))
            wf = bf16_to_f32(w[b, r0:r1])[:, :, None]            # [s, H, 1]
            prod = round_bf16((sc * wf).astype(np.float32))
            acc = np.zeros((r1 - r0, T), np.float32)
            for h in range(H):
                acc = (acc + prod[:, h, :]).astype(np.float32)
            res = f32_to_bf16(acc)
            for i in range(r1 - r0):
                res[i, lim[r0 + i]:] = NEG_INF_BF16
            out[b, r0:r1] = res
    return out


def bf16_order_key(bits: np.ndarray) -> np.ndarray:
    """Monotone uint16 key of a bf16 value (larger value -> larger key), with
    -0.0 folded onto +0.0 so that the two compare equal as in torch."""
    u = np.asarray(bits, np.uint16).astype(np.uint32)
    u = np.where(u == 0x8000, 0, u)
    key = np.where(u & 0x8000, (~u) & 0xFFFF, u | 0x8000)
    return key.astype(np.uint16)


def topk_stable(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest bf16 scores per row, value descending then
    index ascending (the tie rule of the contract; see module docstring).
    scores [..., T] bf16 bits -> int64 [..., k]."""
    key = 0xFFFF - bf16_order_key(scores).astype(np.int32)
    order = np.argsort(key, axis=-1, kind="stable")
    return order[..., :k].astype(np.int64)


def indexer_postprocess(idx: np.ndarray, S: int, s0: int, causal: bool, ratio: int,
                        offset: int) -> np.ndarray:
    """baseline/indexer.py:198-205: causal prefill -> index >= (s+1)//ratio
    becomes -1, else index + offset; otherwise index + offset."""
    idx = np.asarray(idx, np.int64)
    if causal:
        lim = ((np.arange(s0, s0 + S) + 1) // ratio)[None, :, None]
        return np.where(idx >= lim, -1, idx + offset)
    return idx + offset


def indexer_forward(q_pre: np.ndarray, k: np.ndarray, w: np.ndarray, freqs: np.ndarray,
                    rope_dim: int, topk: int, ratio: int, start_pos: int, offset: int,
                    s0: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Operator part of baseline/indexer.py:161-206 after the two projections:
    RoPE, scores, mask, top-k, post-process.  Rows s0.. of a prefill call
    (start_pos == 0) or the whole decode call.  Returns (indices int64, scores)."""
    B, S = q_pre.shape[:2]
    T = k.shape[1]
    causal = start_pos == 0
    q = rope_last(q_pre, freqs, rope_dim)
    sc = indexer_scores(q, k, w, causal, ratio, s0)
    kk = min(topk, T)
    idx = topk_stable(sc, kk)
    return indexer_postprocess(idx, S, s0, causal, ratio, offset), sc


# ---------------------------------------------------------------- FP8 (e4m3) indexer
def _e4m3_table() -> np.ndarray:
    """float32 value of every e4m3 code (NaN for 0x7F and 0xFF)."""
    v = np.empty(256, np.float32)
    for c in range(256):
        sgn = -1.0 if c & 0x80 else 1.0
        e, m = (c >> 3) & 0xF, c & 7
        if e == 0xF and m == 7:
            v[c] = np.nan
        elif e == 0:
            v[c] = sgn * (m / 8.0) * 2.0 ** -6
        else:
            v[c] = sgn * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return v


E4M3 = _e4m3_table()
_POS = E4M3[:0x7F]          # codes 0x00..0x7E: +0 .. 448, increasing


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    return E4M3[np.asarray(codes, np.uint8)]


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3 codes, round to nearest (ties to the even code) and
    saturation to +-448 (the cvt.rn.satfinite rule); the sign of zero is kept."""
    x = np.asarray(x, np.float32)
    a = np.abs(x)
    hi = np.clip(np.searchsorted(_POS, a, side="left"), 0, len(_POS) - 1)  # first >= a
    lo = np.maximum(hi - 1, 0)
    d_lo = a - _POS[lo]
    d_hi = _POS[hi] - a
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(a >= _POS[-1], len(_POS) - 1, code)  # saturate
    return (code | np.where(np.signbit(x), 0x80, 0)).astype(np.uint8)


def quant_fp8_rows(x_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Rows of bf16 bits [..., D] -> (e4m3 codes [..., D], fp32 scales [...]):
    scale = smallest power of two >= max(amax, 1e-4) / 448, codes of x / scale."""
    x = bf16_to_f32(x_bits)
    amax = np.maximum(np.abs(x).max(axis=-1), np.float32(1e-4)).astype(np.float32)
    v = (amax / np.float32(448.0)).astype(np.float32)
    m, e = np.frexp(v)                               # v = m * 2^e, m in [0.5, 1)
    s = np.where(m == 0.5, v, np.ldexp(np.float32(1.0), e)).astype(np.float32)
    return e4m3_encode((x / s[..., None]).astype(np.float32)), s


def indexer_scores_fp8(q8: np.ndarray, k8: np.ndarray, w: np.ndarray, k_scale: np.ndarray,
                       causal: bool, ratio: int, s0: int = 0) -> np.ndarray:
    """FP8 indexer scores (operator contract of ks_indexer_fp8) for rows s0..:
    bf16( k_scale[t] * sum_h fp32(relu(dot_h) * w_h) ) with the head sum in fp32,
    heads in order, and the causal mask of baseline/indexer.py:185-193.
    q8 [B,S,H,D] and k8 [B,T,D] e4m3 codes, w [B,S,H] fp32, k_scale [B,T] fp32.
    The dot products are exact (float64) rounded once to fp32."""
    B, S, H, D = q8.shape
    T = k8.shape[1]
    out = np.empty((B, S, T), np.uint16)
    lim = indexer_limits(S, s0, causal, ratio, T)
    for b in range(B):
        kf = e4m3_decode(k8[b]).astype(np.float64)          # [T, D]
        for r0 in range(0, S, 16):
            r1 = min(S, r0 + 16)
            qf = e4m3_decode(q8[b, r0:r1]).astype(np.float64).reshape(-1, D)
            dot = (qf @ kf.T).astype(np.float32).reshape(r1 - r0, H, T)
            rel = np.maximum(dot, np.float32(0.0))
            acc = np.zeros((r1 - r0, T), np.float32)
            wf = np.asarray(w[b, r0:r1], np.float32)
            for h in range(H):
                acc = (acc + (rel[:, h, :] * wf[:, h:h + 1]).astype(np.float32)).astype(np.float32)
            res = f32_to_bf16((acc * np.asarray(k_scale[b], np.float32)[None, :]).astype(np.float32))
            for i in range(r1 - r0):
                res[i, lim[r0 + i]:] = NEG_INF_BF16
            out[b, r0:r1] = res
    return out
