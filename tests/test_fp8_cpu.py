"""The FP8 oracle's e4m3 tables and quantisation rule, on the CPU.

e4m3 (OCP 8-bit float, "fn" variant): 1 sign, 4 exponent bits (bias 7), 3
mantissa bits, no infinities, 0x7F / 0xFF are NaN, largest finite 448.  torch's
float8_e4m3fn implements the same format, so its conversions are an independent
check of the oracle's tables (torch rounds to nearest even but does not
saturate, so only values within range are compared)."""
import numpy as np
import torch

from oracle import ks_oracle as O


def test_decode_table_matches_torch():
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    ref = codes.view(torch.float8_e4m3fn).float().numpy()
    mine = O.E4M3
    assert np.array_equal(np.isnan(ref), np.isnan(mine))
    ok = ~np.isnan(ref)
    assert np.array_equal(ref[ok], mine[ok])
    assert mine[0x7E] == 448.0 and mine[0x01] == 2.0 ** -9


def test_encode_round_trips_every_finite_code():
    codes = np.array([c for c in range(256) if c not in (0x7F, 0xFF)], np.uint8)
    assert np.array_equal(O.e4m3_encode(O.e4m3_decode(codes)), codes)


def test_encode_matches_torch_in_range():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000) * s for s in (1e-3, 0.1, 1, 30, 200)])
    x = np.clip(x, -448, 448).astype(np.float32)
    # midpoints between neighbouring codes exercise ties-to-even
    pos = O.E4M3[:0x7F].astype(np.float64)
    mids = ((pos[1:] + pos[:-1]) / 2).astype(np.float32)
    x = np.concatenate([x, mids, -mids]).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_encode(x), ref)


def test_encode_saturates():
    x = np.array([448.0, 460.0, 464.0, 1e6, np.float32(3e38), -1e6], np.float32)
    assert O.e4m3_encode(x).tolist() == [0x7E, 0x7E, 0x7E, 0x7E, 0x7E, 0xFE]


def test_quant_rows_scale_is_power_of_two_and_bounds_error():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((64, 128)) * np.exp(rng.uniform(-8, 8, (64, 1)))).astype(np.float32)
    x[3] = 0.0
    xb = O.f32_to_bf16(x)
    codes, s = O.quant_fp8_rows(xb)
    m, _ = np.frexp(s)
    assert np.all(m == 0.5)                                  # powers of two
    xf = O.bf16_to_f32(xb)
    amax = np.maximum(np.abs(xf).max(-1), 1e-4)
    assert np.all(s >= amax / 448) and np.all(s < 2 * amax / 448 * (1 + 1e-6))
    deq = O.e4m3_decode(codes) * s[:, None]
    assert np.all(np.abs(deq - xf) <= np.maximum(np.abs(xf) * 2 ** -4, s[:, None] * 2 ** -10))
    assert np.all(codes[3] == 0) and s[3] == np.float32(2.0 ** np.ceil(np.log2(1e-4 / 448)))
