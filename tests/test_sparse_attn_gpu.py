"""SparseAttention kernel vs the golden fixtures and the oracle
(baseline/sparse_attention.py:5-42).  Float outputs: the harness tolerance
atol = rtol = 1e-2, plus a tighter check on the mean error."""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden
from helpers import bf16_from_bits, bits_from_bf16
from oracle import ks_oracle as O

SA = sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN, "sa_*.npz")))
pytestmark = pytest.mark.gpu


def assert_close(got_bits, ref_bits):
    a = O.bf16_to_f32(got_bits).astype(np.float64)
    r = O.bf16_to_f32(ref_bits).astype(np.float64)
    assert np.all(np.isfinite(a))
    assert np.allclose(a, r, atol=1e-2, rtol=1e-2), f"max abs diff {np.abs(a - r).max():.3e}"
    assert np.abs(a - r).mean() < 2e-3


@pytest.mark.parametrize("name", SA)
def test_golden(cuda_ok, name):
    from kernelswift_b200 import ops

    d = load_golden(name)
    out = ops.sparse_attn(bf16_from_bits(d["q"]), bf16_from_bits(d["kv"]),
                          torch.from_numpy(d["sink"]).cuda(), torch.from_numpy(d["idx"]).cuda(),
                          float(d["scale"]))
    ops.device_status()
    assert_close(bits_from_bf16(out), d["out"])


def make_case(B, M, H, D, N, K, seed, mode="perm", sink="randn"):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, M, H, D, generator=g).bfloat16()
    kv = torch.randn(B, N, D, generator=g).bfloat16()
    if mode == "perm":
        idx = torch.stack([torch.stack([torch.randperm(N, generator=g)[:K] for _ in range(M)])
                           for _ in range(B)]).int()
    else:
        idx = torch.randint(-N // 4, N, (B, M, K), generator=g).int()  # duplicates and -1s
        idx[idx < 0] = -1
    s = torch.randn(H, generator=g) if sink == "randn" else torch.zeros(H)
    return q, kv, s, idx


CASES = [
    # B, M, H, D, N, K, dv, mode
    (1, 128, 16, 128, 4096, 512, 128, "perm"),     # C2
    (2, 5, 128, 576, 2048, 512, 512, "perm"),      # MLA heads, dv = 512 of D = 576
    (1, 7, 128, 576, 1000, 100, 512, "mixed"),     # ragged K, duplicates, -1
    (1, 6, 64, 128, 32, 16, 128, "mixed"),         # reference geometry
    (3, 3, 24, 192, 300, 130, 192, "perm"),        # odd H, dv not a multiple of 128
    (1, 4, 128, 256, 777, 64, 64, "mixed"),        # dv = 64
]


@pytest.mark.parametrize("B,M,H,D,N,K,dv,mode", CASES)
def test_vs_oracle(cuda_ok, B, M, H, D, N, K, dv, mode):
    from kernelswift_b200 import ops

    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=B * 100 + M + H + K, mode=mode)
    out = ops.sparse_attn(q.cuda(), kv.cuda(), s.cuda(), idx.cuda(), D ** -0.5, dv)
    ops.device_status()
    ref = O.sparse_attn(bits_from_bf16(q), bits_from_bf16(kv), s.numpy(), idx.numpy(), D ** -0.5, dv)
    assert_close(bits_from_bf16(out), ref)


def test_column_slice(cuda_ok):
    """dv_begin > 0 (the second pass of a D = 576 output) equals those columns of a full call."""
    from kernelswift_b200 import _lib, ops

    B, M, H, D, N, K = 1, 3, 128, 576, 512, 128
    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=9)
    q, kv, s, idx = q.cuda(), kv.cuda(), s.cuda(), idx.cuda()
    full = ops.sparse_attn(q, kv, s, idx, D ** -0.5)  # 576 columns: 512 + 64
    part = torch.empty(B, M, H, 64, dtype=torch.bfloat16, device="cuda")
    _lib.check(_lib.lib().ks_sparse_attn(q.data_ptr(), kv.data_ptr(), s.data_ptr(), idx.data_ptr(),
                                         part.data_ptr(), B, M, H, D, N, K, 512, 64, D ** -0.5,
                                         torch.cuda.current_stream().cuda_stream), "sa")
    ops.device_status()
    assert torch.equal(full[..., 512:], part)
    ref = O.sparse_attn(bits_from_bf16(q), bits_from_bf16(kv), s.cpu().numpy(), idx.cpu().numpy(), D ** -0.5)
    assert_close(bits_from_bf16(full), ref)


def test_edge_rows(cuda_ok):
    """All-invalid rows give 0; a single repeated row gives that row; sinks weigh in."""
    from kernelswift_b200 import ops

    B, M, H, D, N, K = 1, 4, 16, 128, 64, 96
    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=3)
    idx[0, 0] = -1
    idx[0, 1] = 5
    idx[0, 2, 1:] = -1
    out = ops.sparse_attn(q.cuda(), kv.cuda(), torch.full((H,), -1e4).cuda(), idx.cuda(), D ** -0.5)
    ops.device_status()
    o = out.float().cpu()
    assert torch.all(o[0, 0] == 0)
    assert torch.allclose(o[0, 1], kv[0, 5].float().expand(H, D), atol=1e-2, rtol=1e-2)
    assert torch.allclose(o[0, 2], kv[0, idx[0, 2, 0]].float().expand(H, D), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("D,dv", [(576, 512), (128, 128)])
def test_trailing_invalid_blocks(cuda_ok, D, dv):
    """Rows whose indices are valid only in a prefix (the indexer's output for early
    causal rows: -1 after the first s + 1 entries).  The kernel stops after the last
    256-key block holding a valid index; prefixes ending on, just before and just after
    block boundaries, a single entry and none must match the oracle."""
    from kernelswift_b200 import ops

    B, H, N, K = 1, 128 if D == 576 else 16, 3000, 1024
    lens = [0, 1, 255, 256, 257, 511, 512, 700, 1023, 1024]
    M = len(lens)
    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=21)
    for m, n in enumerate(lens):
        idx[0, m, n:] = -1
    out = ops.sparse_attn(q.cuda(), kv.cuda(), s.cuda(), idx.cuda(), D ** -0.5, dv)
    ops.device_status()
    ref = O.sparse_attn(bits_from_bf16(q), bits_from_bf16(kv), s.numpy(), idx.numpy(), D ** -0.5, dv)
    assert_close(bits_from_bf16(out), ref)
    assert torch.all(out[0, 0].float() == 0)


def test_mla_scale_rows(cuda_ok):
    """C4 geometry (4, 4096, 128, 576), N = 32768, K = 2048, dv = 512, causal-valid
    indices; the oracle checks a sample of rows."""
    from kernelswift_b200 import ops

    B, M, H, D, N, K, dv = 4, 4096, 128, 576, 32768, 2048, 512
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, M, H, D, device="cuda", generator=g).bfloat16()
    kv = torch.randn(B, N, D, device="cuda", generator=g).bfloat16()
    pos = N - M + torch.arange(M, device="cuda")
    r = torch.rand(B, M, K, device="cuda", generator=g)
    idx = (r * (pos[None, :, None] + 1).float()).long().clamp_max(N - 1).int()
    sink = torch.zeros(H, device="cuda")
    out = ops.sparse_attn(q, kv, sink, idx, D ** -0.5, dv)
    ops.device_status()
    rows = [0, 1, 2047, 4095]
    for b in (0, 3):
        qb = bits_from_bf16(q[b:b + 1, rows])
        ib = idx[b:b + 1, rows].cpu().numpy()
        ref = O.sparse_attn(qb, bits_from_bf16(kv[b:b + 1]), sink.cpu().numpy(), ib, D ** -0.5, dv)
        assert_close(bits_from_bf16(out[b:b + 1, rows]), ref)


@pytest.mark.parametrize("B,M,H,D,N,K,dv,mode", [
    CASES[0],                                   # D = 128: room for 9 ring slots, 5 used
    CASES[4],                                   # D = 192: room for 8
    (2, 16, 128, 192, 4096, 1024, 192, "perm"),  # four key blocks per query
])
def test_repeatable(cuda_ok, B, M, H, D, N, K, dv, mode):
    """Repeated calls give bit-identical results.  Guards the ring sizing: with a
    slot count that is not a multiple of the gather groups, a group could pass its
    "slot empty" parity wait two phases early and overwrite a chunk in use, which
    shows up as run-to-run differences."""
    from kernelswift_b200 import ops

    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=7 + D + K, mode=mode)
    q, kv, s, idx = q.cuda(), kv.cuda(), s.cuda(), idx.cuda()
    outs = [ops.sparse_attn(q, kv, s, idx, D ** -0.5, dv) for _ in range(4)]
    ops.device_status()
    for o in outs[1:]:
        assert torch.equal(outs[0], o)
    ref = O.sparse_attn(bits_from_bf16(q), bits_from_bf16(kv), s.cpu().numpy(), idx.cpu().numpy(), D ** -0.5, dv)
    assert_close(bits_from_bf16(outs[0]), ref)


def test_out_of_range_index_reported(cuda_ok):
    """An index >= N (the reference's gather raises on it,
    baseline/sparse_attention.py:19-21) is skipped like -1 and reported as a bounds
    error by the status check, without faulting; the status is cleared once read."""
    from kernelswift_b200 import _lib, ops

    B, M, H, D, N, K = 1, 3, 16, 128, 200, 64
    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=31)
    bad = idx.clone()
    bad[0, 1, 5] = N          # just past the table
    bad[0, 2, 0] = N + 12345  # far past it
    out = ops.sparse_attn(q.cuda(), kv.cuda(), s.cuda(), bad.cuda(), D ** -0.5)
    with pytest.raises(_lib.KsError) as e:
        ops.device_status()
    assert e.value.code == _lib.KS_ERR_DEVICE and "table size" in str(e.value)
    ops.device_status()  # cleared
    masked = bad.clone()
    masked[masked >= N] = -1
    ref = O.sparse_attn(bits_from_bf16(q), bits_from_bf16(kv), s.numpy(), masked.numpy(), D ** -0.5)
    assert_close(bits_from_bf16(out), ref)
    # in-range calls leave the status clean
    ops.sparse_attn(q.cuda(), kv.cuda(), s.cuda(), idx.cuda(), D ** -0.5)
    ops.device_status()


@pytest.mark.parametrize("K", [100, 300, 700])  # one, two and three 256-key blocks
def test_persistent_token_sequences(cuda_ok, K):
    """More tokens than resident CTA pairs (300 tokens over at most 74 pairs), so each
    pair runs several tokens in a row with the ring, barrier phases and S / P buffers
    carried across them.  Block counts 1, 2 and 3 take the three ring layouts at a
    token boundary; duplicates, -1 entries and fully masked rows check that no
    running max, sum or output leaks from one token into the next."""
    from kernelswift_b200 import ops

    B, M, H, D, N, dv = 2, 150, 128, 128, 2000, 128
    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=31 + K, mode="mixed")
    idx[0, 7] = -1          # nothing valid
    idx[1, 80, 1:] = -1     # a single valid key
    idx[1, 149] = 17        # one key repeated K times
    out = ops.sparse_attn(q.cuda(), kv.cuda(), s.cuda(), idx.cuda(), D ** -0.5, dv)
    ops.device_status()
    ref = O.sparse_attn(bits_from_bf16(q), bits_from_bf16(kv), s.numpy(), idx.numpy(), D ** -0.5, dv)
    assert_close(bits_from_bf16(out), ref)
    again = ops.sparse_attn(q.cuda(), kv.cuda(), s.cuda(), idx.cuda(), D ** -0.5, dv)
    assert torch.equal(out, again)


@pytest.mark.parametrize("B,M,H,D,N,K,dv_begin,dv", [
    (3, 13, 16, 128, 500, 32, 0, 128),    # 8 tokens per tile, tiles across batches
    (2, 9, 32, 256, 300, 20, 64, 192),    # 4 tokens per tile, a column slice
    (1, 7, 128, 256, 777, 64, 0, 256),    # one token per tile, the longest rows
    (1, 5, 64, 128, 300, 16, 64, 64),     # TMA-stored tiles, the last half full, a column slice
])
def test_tiny_rows(cuda_ok, B, M, H, D, N, K, dv_begin, dv):
    """Index rows of at most 64 keys: 128 / H tokens share one 128-row tile, each
    row keeping its own token's keys.  Duplicates, -1 entries, fully masked rows
    and output column slices against the oracle; the output tiles are stored by
    TMA, the last one clipped where it runs past the last token."""
    from kernelswift_b200 import _lib, ops

    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=41 + H + K, mode="mixed")
    idx[0, 1] = -1
    idx[-1, -1, 1:] = idx[-1, -1, 0]
    out = torch.empty(B, M, H, dv, dtype=torch.bfloat16, device="cuda")
    qc, kvc, sc, ic = q.cuda(), kv.cuda(), s.cuda(), idx.cuda()
    _lib.check(_lib.lib().ks_sparse_attn(qc.data_ptr(), kvc.data_ptr(), sc.data_ptr(), ic.data_ptr(),
                                    out.data_ptr(), B, M, H, D, N, K, dv_begin, dv, D ** -0.5,
                                    torch.cuda.current_stream().cuda_stream), "ks_sparse_attn")
    ops.device_status()
    ref = O.sparse_attn(bits_from_bf16(q), bits_from_bf16(kv), s.numpy(), idx.numpy(), D ** -0.5,
                        dv_begin + dv)[..., dv_begin:]
    assert_close(bits_from_bf16(out), ref)


@pytest.mark.parametrize("B,M,H,D,N,K,dv_begin,dv", [
    (1, 9, 16, 128, 900, 300, 0, 128),     # three tiles: the 512-thread form, slots past K
    (2, 5, 64, 256, 1000, 512, 0, 256),    # four full tiles, 64 heads, the widest output
    (1, 6, 32, 192, 500, 200, 64, 128),    # two tiles, a column slice
    (3, 4, 24, 128, 3000, 129, 0, 128),    # a single key in the second tile
])
def test_multi_tile_rows(cuda_ok, B, M, H, D, N, K, dv_begin, dv):
    """Index rows of 129-512 keys with at most 64 heads (the few-heads kernel, one
    warp group per 128-key tile, per-head maxima and sums combined across the
    groups).  Rows with nothing valid, with keys in the first tile only, with the
    first tile empty and with one key repeated against the oracle; repeated calls
    bit-identical."""
    from kernelswift_b200 import _lib, ops

    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=51 + H + K, mode="mixed")
    idx[0, 0] = -1
    idx[0, 1, 128:] = -1
    idx[0, 2, :128] = -1
    idx[-1, -1, :] = idx[-1, -1, 0]
    qc, kvc, sc, ic = q.cuda(), kv.cuda(), s.cuda(), idx.cuda()

    def call():
        out = torch.empty(B, M, H, dv, dtype=torch.bfloat16, device="cuda")
        _lib.check(_lib.lib().ks_sparse_attn(qc.data_ptr(), kvc.data_ptr(), sc.data_ptr(), ic.data_ptr(),
                                             out.data_ptr(), B, M, H, D, N, K, dv_begin, dv, D ** -0.5,
                                             torch.cuda.current_stream().cuda_stream), "ks_sparse_attn")
        return out

    out = call()
    ops.device_status()
    ref = O.sparse_attn(bits_from_bf16(q), bits_from_bf16(kv), s.numpy(), idx.numpy(), D ** -0.5,
                        dv_begin + dv)[..., dv_begin:]
    assert_close(bits_from_bf16(out), ref)
    assert torch.all(out[0, 0].float() == 0)  # nothing valid: the sink alone, zeros out
    for _ in range(3):
        assert torch.equal(out, call())


def test_tiny_out_of_range_index_reported(cuda_ok):
    """The short-row kernel (128 / H tokens per tile) skips an index >= N like -1 and
    reports it as a bounds error, as the other attention kernels do."""
    from kernelswift_b200 import _lib, ops

    B, M, H, D, N, K = 2, 5, 64, 128, 300, 16
    q, kv, s, idx = make_case(B, M, H, D, N, K, seed=61)
    bad = idx.clone()
    bad[1, 3, 7] = N
    out = ops.sparse_attn(q.cuda(), kv.cuda(), s.cuda(), bad.cuda(), D ** -0.5)
    with pytest.raises(_lib.KsError) as e:
        ops.device_status()
    assert e.value.code == _lib.KS_ERR_DEVICE and "table size" in str(e.value)
    ops.device_status()  # cleared
    masked = bad.clone()
    masked[masked >= N] = -1
    ref = O.sparse_attn(bits_from_bf16(q), bits_from_bf16(kv), s.numpy(), masked.numpy(), D ** -0.5)
    assert_close(bits_from_bf16(out), ref)
