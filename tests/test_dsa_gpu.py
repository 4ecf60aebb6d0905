"""The DSA step (indexer -> int32 top-k -> sparse attention) through ``ops.dsa``
at the headline configuration C5, checked against the oracle on row blocks.

C5: B = 2, S = T = 32768, indexer H = 64, D = 128, RoPE on the last 64 dims,
top-2048, causal prefill (baseline/indexer.py:170-205); its int32 indices feed
sparse attention with H = 128, D = 576, dv = 512 over the same rows
(baseline/sparse_attention.py:5-42).  The rows are split the way bench.py splits
them over two ranks (zigzag: (0, 8192) + (24576, 32768) and (8192, 24576)), so
the calls start at pos0 = 0, 8192 and 24576.  Inputs are seeded on the device.

Gates per checked block of rows:
  * scores (read from the call's workspace) equal the oracle's bit for bit except
    rare bf16 flips from the GEMM's fp32 accumulation order (<= 0.1 %, small);
  * indices equal, exactly and in order, the stable top-k of the kernel's own
    scores, with -1 past each row's causal limit;
  * rows whose indices differ from the oracle's are rows with a score flip;
  * attention on those kernel-produced indices (early rows are mostly -1)
    matches the oracle within the harness tolerance.
"""
import numpy as np
import pytest
import torch

from helpers import bits_from_bf16
from oracle import ks_oracle as O

pytestmark = pytest.mark.gpu


def _freqs(a, b, rd):
    inv = 1.0 / (10000.0 ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))
    ang = torch.outer(torch.arange(a, b, dtype=torch.float32), inv)
    return torch.stack([ang.cos(), ang.sin()], -1).contiguous()


def assert_close(got_bits, ref_bits):
    a = O.bf16_to_f32(got_bits).astype(np.float64)
    r = O.bf16_to_f32(ref_bits).astype(np.float64)
    assert np.all(np.isfinite(a))
    assert np.allclose(a, r, atol=1e-2, rtol=1e-2), f"max abs diff {np.abs(a - r).max():.3e}"
    assert np.abs(a - r).mean() < 2e-3


def test_dsa_equals_the_two_ops(cuda_ok):
    """ops.dsa gives exactly what indexer_topk (int32) followed by sparse_attn gives."""
    from kernelswift_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(3)
    B, S, T, H, D, rd, k = 2, 300, 700, 64, 128, 64, 256
    Hs, Ds, dv = 32, 192, 128
    q = torch.randn(B, S, H, D, device="cuda", generator=g).bfloat16()
    kx = torch.randn(B, T, D, device="cuda", generator=g).bfloat16()
    w = (torch.rand(B, S, H, device="cuda", generator=g) * 0.01).bfloat16()
    fr = _freqs(400, 400 + S, rd).cuda()
    qs = torch.randn(B, S, Hs, Ds, device="cuda", generator=g).bfloat16()
    kv = torch.randn(B, T + 5, Ds, device="cuda", generator=g).bfloat16()
    sink = torch.randn(Hs, device="cuda", generator=g)
    out, idx = ops.dsa(q, kx, w, fr, rd, T, k, qs, kv, sink, Ds ** -0.5, dv, pos0=400, offset=5)
    idx2 = ops.indexer_topk(q, kx, w, fr, rd, T, k, pos0=400, offset=5, out_dtype=torch.int32)
    out2 = ops.sparse_attn(qs, kv, sink, idx2, Ds ** -0.5, dv)
    ops.device_status()
    assert idx.dtype == torch.int32 and torch.equal(idx, idx2)
    assert torch.equal(out, out2)
    ref = O.sparse_attn(bits_from_bf16(qs), bits_from_bf16(kv), sink.cpu().numpy(),
                        idx.cpu().numpy(), Ds ** -0.5, dv)
    assert_close(bits_from_bf16(out), ref)


def test_c5_rows(cuda_ok):
    from kernelswift_b200 import ops, shard

    B, S, H, D, rd, k = 2, 32768, 64, 128, 64, 2048
    Hs, Ds, dv = 128, 576, 512
    T = S
    g = torch.Generator(device="cuda").manual_seed(2024)
    k_ix = torch.randn(B, T, D, device="cuda", generator=g).bfloat16()
    kv = torch.randn(B, T, Ds, device="cuda", generator=g).bfloat16()
    sink = torch.zeros(Hs, device="cuda")
    ranges = shard.zigzag(S, 2, 0) + shard.zigzag(S, 2, 1)
    assert ranges == [(0, 8192), (24576, 32768), (8192, 24576)]
    ws = torch.empty(max(ops.indexer_workspace_size(B, b - a, T) for a, b in ranges),
                     dtype=torch.uint8, device="cuda")
    ld = (T + 7) // 8 * 8
    # blocks of rows checked against the oracle (each inside one call's range): the
    # first rows (mostly -1 indices), the k-th row boundary, both ends of every range
    blocks = [0, 2040, 8176, 8192, 16376, 24560, 24576, 32752]
    R, RA = 16, 6  # rows per block for the indexer, for attention
    kx_bits = bits_from_bf16(k_ix)
    kv_bits = bits_from_bf16(kv)
    n_blocks = 0
    for a, b in ranges:
        n = b - a
        q = torch.randn(B, n, H, D, device="cuda", generator=g).bfloat16()
        w = (torch.rand(B, n, H, device="cuda", generator=g) * (D ** -0.5 * H ** -0.5)).bfloat16()
        fr = _freqs(a, b, rd)
        qs = torch.randn(B, n, Hs, Ds, device="cuda", generator=g).bfloat16()
        out, idx = ops.dsa(q, k_ix, w, fr.cuda(), rd, T, k, qs, kv, sink, Ds ** -0.5, dv,
                           pos0=a, workspace=ws)
        ops.device_status()
        sc_all = ws[: B * n * ld * 2].view(torch.bfloat16).view(B, n, ld)
        for s0 in [s for s in blocks if a <= s < b]:
            r0 = s0 - a
            assert r0 + R <= n
            for bb in range(B):
                sc = bits_from_bf16(sc_all[bb, r0:r0 + R, :T])[None]
                got = idx[bb, r0:r0 + R].cpu().numpy().astype(np.int64)[None]
                q_rope = O.rope_last(bits_from_bf16(q[bb:bb + 1, r0:r0 + R]),
                                     fr[r0:r0 + R].numpy(), rd)
                ref_sc = O.indexer_scores(q_rope, kx_bits[bb:bb + 1],
                                          bits_from_bf16(w[bb:bb + 1, r0:r0 + R]), True, 1, s0)
                lim = O.indexer_limits(R, s0, True, 1, T)
                valid = np.broadcast_to(np.arange(T)[None, None, :] < lim[None, :, None], sc.shape)
                flips = (sc != ref_sc) & valid
                assert flips.mean() <= 1e-3, f"rows {s0}+: score flips {flips.mean():.2e}"
                assert np.allclose(O.bf16_to_f32(sc)[valid], O.bf16_to_f32(ref_sc)[valid],
                                   rtol=1e-2, atol=1e-2)
                own = np.where(valid, sc, O.NEG_INF_BF16).astype(np.uint16)
                exp_own = O.indexer_postprocess(O.topk_stable(own, k), R, s0, True, 1, 0)
                assert np.array_equal(got, exp_own), f"rows {s0}+ (batch {bb}): top-k"
                ref_idx = O.indexer_postprocess(O.topk_stable(ref_sc, k), R, s0, True, 1, 0)
                bad_rows = np.any(got != ref_idx, axis=-1)
                assert not np.any(bad_rows & ~np.any(flips, axis=-1))
                # attention on the kernel's own indices
                ref_o = O.sparse_attn(bits_from_bf16(qs[bb:bb + 1, r0:r0 + RA]),
                                      kv_bits[bb:bb + 1], sink.cpu().numpy(),
                                      got[:, :RA].astype(np.int32), Ds ** -0.5, dv)
                assert_close(bits_from_bf16(out[bb:bb + 1, r0:r0 + RA]), ref_o)
                n_blocks += 1
        del q, w, qs, out, idx, sc_all
    assert n_blocks == len(blocks) * B
    del ws, k_ix, kv
    torch.cuda.empty_cache()
