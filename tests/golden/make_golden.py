"""Generate the golden fixtures under tests/golden/ from the reference's own code.

This script imports the reference's PyTorch modules (``baseline/sinkhorn.py``,
``baseline/sparse_attention.py``, ``baseline/indexer.py``) from a checkout of
TtitiO/KernelSwift, runs them on CPU on small seeded inputs and stores inputs,
selected intermediates and outputs as compressed ``.npz`` files.  The fixtures
are what pins the numpy oracle in ``oracle/ks_oracle.py``: the oracle must
reproduce every stored output (bit-exactly for bf16 scores and indices, within
1e-5 for fp32 values) before it is trusted as the checker for the CUDA path.

Run it where the reference checkout exists:

    python tests/golden/make_golden.py --ref <path-to-KernelSwift-checkout>

bf16 tensors are stored as their raw uint16 bit patterns.
"""
import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load(ref, rel, name):
    spec = importlib.util.spec_from_file_location(name, os.path.join(ref, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bits(t):
    """Raw bit pattern of a bf16 tensor as uint16 numpy."""
    assert t.dtype == torch.bfloat16
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def sinkhorn_cases(ref):
    m = load(ref, "baseline/sinkhorn.py", "ref_sinkhorn")
    cases = [
        # (name, shape, repeat, eps, seed)
        ("sk_ref_default", (1, 1024, 4, 4), 10, 1e-6, 42),
        ("sk_c1_like", (2, 256, 4, 4), 20, 1e-6, 0),
        ("sk_8x8", (2, 96, 8, 8), 20, 1e-6, 1),
        ("sk_3x3_r1", (3, 5, 3, 3), 1, 1e-6, 2),
        ("sk_16x16", (1, 16, 16, 16), 20, 1e-6, 3),
        ("sk_eps_big", (1, 33, 4, 4), 3, 1e-2, 4),
    ]
    for name, shape, repeat, eps, seed in cases:
        torch.manual_seed(seed)
        x = torch.randn(*shape, dtype=torch.float32) * 2.0
        out = m.Model(repeat, eps)(x.clone())
        np.savez_compressed(os.path.join(HERE, name + ".npz"), x=x.numpy(), out=out.numpy(),
                            repeat=repeat, eps=eps)
        print(name, tuple(out.shape))


def sparse_attn_cases(ref):
    m = load(ref, "baseline/sparse_attention.py", "ref_sparse_attention")

    def run(name, B, M, H, D, N, K, seed, idx_mode, sink_mode):
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(B, M, H, D, generator=g).bfloat16()
        kv = torch.randn(B, N, D, generator=g).bfloat16()
        if idx_mode == "perm":
            idx = torch.stack([torch.stack([torch.randperm(N, generator=g)[:K] for _ in range(M)])
                               for _ in range(B)]).int()
        elif idx_mode == "randint":
            idx = torch.randint(0, N, (B, M, K), generator=g, dtype=torch.int32)
        elif idx_mode == "edge":
            idx = torch.randint(0, N, (B, M, K), generator=g, dtype=torch.int32)
            idx[0, 0, :] = 3                       # every entry the same row (count K)
            idx[0, 1, :] = torch.arange(K // 2).repeat_interleave(2).int()   # pairs (count 2)
            idx[0, 2, :] = -1                      # all invalid: output 0
            idx[0, 3, ::3] = -1                    # mixed invalid
            idx[1, 0, 1:] = -1                     # a single valid entry
            idx[1, 1, :K // 2] = -1                # invalid prefix
        elif idx_mode == "causal":
            # query m at absolute position p = N - M + m selects among [0, p]
            rows = []
            for b in range(B):
                r = []
                for mm in range(M):
                    p = N - M + mm
                    perm = torch.randperm(p + 1, generator=g)[:K]
                    if perm.numel() < K:
                        perm = torch.cat([perm, torch.full((K - perm.numel(),), -1)])
                    r.append(perm)
                rows.append(torch.stack(r))
            idx = torch.stack(rows).int()
        else:
            raise ValueError(idx_mode)
        model = m.Model(H, D)
        if sink_mode == "randn":
            with torch.no_grad():
                model.attn_sink.copy_(torch.randn(H, generator=g))
        with torch.no_grad():
            out = model(q, kv, idx)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), q=bits(q), kv=bits(kv),
                            idx=idx.numpy(), sink=model.attn_sink.detach().numpy(),
                            out=bits(out), scale=np.float32(model.softmax_scale))
        print(name, tuple(out.shape))

    run("sa_c2_like", 1, 8, 16, 128, 1024, 128, 0, "perm", "zeros")
    run("sa_edge", 2, 6, 16, 64, 64, 32, 1, "edge", "randn")
    run("sa_ref_shape", 2, 16, 64, 128, 32, 16, 2, "randint", "zeros")
    run("sa_mla_like", 1, 4, 128, 576, 512, 128, 3, "causal", "randn")
    run("sa_h128_d128", 1, 3, 128, 128, 300, 200, 4, "perm", "randn")


def indexer_cases(ref):
    m = load(ref, "baseline/indexer.py", "ref_indexer")

    def run(name, B, S, dim, H, D, rd, k, qlr, ratio, start_pos, offset, seed, ties=False,
            max_seq=None):
        max_seq = max_seq or (start_pos + S)
        args = m.ModelArgs(max_batch_size=B, max_seq_len=max_seq, dim=dim, index_n_heads=H,
                           index_head_dim=D, index_topk=k, q_lora_rank=qlr, rope_head_dim=rd)
        torch.manual_seed(seed)
        freqs = 1.0 / (10000.0 ** (torch.arange(0, rd, 2).float() / rd))
        ang = torch.outer(torch.arange(max_seq, dtype=torch.float32), freqs)
        freqs_cis = torch.polar(torch.ones_like(ang), ang)
        kv_cache = torch.randn(B, max_seq // ratio, D, dtype=torch.bfloat16)
        if ties:
            # few distinct key rows and coarse values: many equal scores per row
            kv_cache = (kv_cache * 2).round().clamp(-2, 2).bfloat16()
            kv_cache[:, 1::2] = kv_cache[:, 0::2][:, : kv_cache[:, 1::2].shape[1]]
        model = m.Model(args, freqs_cis, kv_cache, ratio)
        x = torch.randn(B, S, dim, dtype=torch.bfloat16)
        qr = torch.randn(B, S, qlr, dtype=torch.bfloat16)
        if ties:
            qr = (qr * 2).round().clamp(-2, 2).bfloat16()
        with torch.no_grad():
            out = model(x.clone(), qr.clone(), start_pos, offset)
            # Intermediates, recomputed with the reference's own modules and the same
            # op sequence as Model.forward (baseline/indexer.py:161-183).
            end_pos = start_pos + S
            q = model.wq_b(qr).unflatten(-1, (H, D))
            q_pre = q.clone()
            m.apply_rotary_emb(q[..., -rd:], freqs_cis[start_pos:end_pos])
            w = model.weights_proj(x) * (model.softmax_scale * H ** -0.5)
            sc = torch.einsum("bshd,btd->bsht", q, kv_cache[:B, : end_pos // ratio])
            sc = (sc.relu_() * w.unsqueeze(-1)).sum(dim=2)
        assert w.dtype == torch.bfloat16 and sc.dtype == torch.bfloat16
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"),
            q_pre=bits(q_pre), q_rope=bits(q), w=bits(w),
            kv=bits(kv_cache[:B, : end_pos // ratio]),
            freqs=torch.view_as_real(freqs_cis[start_pos:end_pos]).numpy(),
            scores=bits(sc), out=out.numpy(),
            meta=np.array([B, S, H, D, rd, k, ratio, start_pos, offset], np.int64))
        print(name, tuple(out.shape), out.dtype)

    # the reference's own default geometry (H=16, D=64, rd=32, ratio=4, k=128), fewer rows
    run("ix_ref_geom", 2, 256, 128, 16, 64, 32, 128, 64, 4, 0, 0, 11)
    # DSA-scale heads (H=64, D=128, rd=64, ratio=1), k < T so early rows carry -1
    run("ix_dsa_geom", 1, 192, 64, 64, 128, 64, 128, 64, 1, 0, 0, 12)
    # decode-style call: start_pos > 0, no mask, +offset
    run("ix_decode", 1, 24, 64, 64, 128, 64, 64, 64, 1, 160, 1000, 13, max_seq=184)
    # many tied scores
    run("ix_ties", 1, 128, 64, 16, 64, 32, 32, 64, 1, 0, 7, 14, ties=True)


def harness_cases(ref, seed=42):
    """Each reference Model at its own default configuration, built and run in the
    order the reference harness uses (benchmarks/ks/auto_bench.py:378-409 and
    :513-539): seed, get_init_inputs (twice, v0 then v1), Model(*init), seed,
    get_inputs, seed, forward on a clone of the inputs.  Outputs that are too large
    to store whole are kept as sampled rows plus per-row sums."""

    def seed_all():
        torch.manual_seed(seed)

    for rel, name in (("baseline/sinkhorn.py", "sinkhorn"),
                      ("baseline/sparse_attention.py", "sparse_attention"),
                      ("baseline/indexer.py", "indexer")):
        m = load(ref, rel, "ref_h_" + name)
        seed_all()
        m.get_init_inputs()
        seed_all()
        init = m.get_init_inputs()
        model = m.Model(*init)
        model.eval()
        seed_all()
        inputs = m.get_inputs()
        seed_all()
        cloned = [t.clone() if isinstance(t, torch.Tensor) else t for t in inputs]
        with torch.no_grad():
            out = model(*cloned)
        path = os.path.join(HERE, "hx_" + name + ".npz")
        if name == "sinkhorn":
            np.savez_compressed(path, out=out.numpy())
        elif name == "sparse_attention":
            B, M = out.shape[:2]
            rows = np.array([0, 1, M // 2, M - 1])
            np.savez_compressed(path, rows=rows, out_rows=bits(out[:, rows]),
                                row_sums=out.double().sum(dim=(2, 3)).numpy())
        else:
            assert out.dtype == torch.int64 and int(out.max()) < 32768
            np.savez_compressed(path, out=out.numpy().astype(np.int16))
        print("hx_" + name, tuple(out.shape), out.dtype)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path to a KernelSwift checkout")
    a = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    sinkhorn_cases(a.ref)
    sparse_attn_cases(a.ref)
    indexer_cases(a.ref)
    harness_cases(a.ref)
