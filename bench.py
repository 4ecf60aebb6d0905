"""Benchmark of the KernelSwift-B200 operators (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload dsa_e2e|c1|c2|c3|c4]
                    [--impl ours|reference]

Default workload ``dsa_e2e`` is BASELINE.json's end-to-end DSA configuration (C5):
the indexer (B=2, S=T=32768, 64 heads x 128, RoPE 64, top-2048, causal) feeding
sparse attention (128 heads, D=576, dv=512, its int32 indices), plus Sinkhorn on
(2, 32768, 8, 8) fp32 with 20 iterations.  A step is one pass of the three ops
over this rank's query rows; rows are sharded over ranks (zigzag for the causal
indexer, contiguous for the rest) with no collective on the data path, so the
total work is fixed as N grows (strong scaling).  ``value`` is query tokens per
second for the whole job (device-resident inputs, CUDA events, max over ranks);
``e2e`` adds the per-step host<->device copies of the activations (pinned
memory) through the public ops.  Inputs are seeded synthetic tensors of the
configuration's shapes and distributions (no dataset is involved).

``--impl reference`` times the reference algorithm on the host cores instead
(the reference's torch forwards restated in oracle/ks_ref_torch.py, all threads:
what baseline/*.py runs on a CPU), on bounded row samples of the same workload,
extrapolated to the full step; under torchrun only rank 0 runs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# DRAM bytes (read + write) per query token of the sparse-attention kernel at the
# H=128, D=576, dv=512, N=32768, K=2048 geometry, from an ncu capture of one full C4
# launch (dram__bytes_read.sum + dram__bytes_write.sum = 5.102e9 B for 16384 tokens,
# `ncu --metrics ... -k regex:sparse_attn -s 3 -c 1 python bench.py --workload c4`).
# The kernel's traffic grows with the tokens it
# processes (q in, out back, the kv rows of a batch from L2), so a launch's traffic
# is this figure times its tokens.
SA_DRAM_BYTES_PER_TOKEN_MLA = 5.102018560e9 / 16384


# ---------------------------------------------------------------- workloads
class Workload:
    name = ""
    metric = "tokens/s"
    dtype = "bf16"
    # True when each step first writes a buffer larger than L2: the step's time is
    # then the sum of the ops' CUDA-event spans, which leave the flush out
    flushes = False

    def __init__(self, rank, world, device):
        self.rank, self.world, self.device = rank, world, device

    # host-buffer (e2e) steps: hooks around the timed region and how copies are ordered
    def e2e_begin(self):
        pass

    def e2e_end(self):
        pass

    def e2e_note(self):
        return "copy-in, ops and copy-out in order on the current stream"

    def traffic(self, kernel):
        """DRAM bytes per step of `kernel` (scaled from an ncu capture), or None."""
        return None


def _freqs_cis(S, rd, pos0=0):
    """Complex RoPE factors of positions pos0.. (baseline/indexer.py get_init_inputs)."""
    import torch

    inv = 1.0 / (10000.0 ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))
    ang = torch.outer(torch.arange(pos0, pos0 + S, dtype=torch.float32), inv)
    return torch.polar(torch.ones_like(ang), ang)


def _freqs(S, rd, pos0=0):
    import torch

    inv = 1.0 / (10000.0 ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))
    ang = torch.outer(torch.arange(pos0, pos0 + S, dtype=torch.float32), inv)
    return torch.stack([ang.cos(), ang.sin()], -1).contiguous()


class DsaE2E(Workload):
    """C5: indexer -> sparse attention, plus Sinkhorn."""
    name = "dsa_e2e"

    def __init__(self, rank, world, device, tokens=None, B=2, S=32768, H_ix=64, D_ix=128, rd=64,
                 k=2048, H_sa=128, D_sa=576, dv=512, sk_shape=(2, 32768, 8, 8), sk_repeat=20):
        super().__init__(rank, world, device)
        S = tokens or S
        sk_shape = (sk_shape[0], tokens or sk_shape[1], sk_shape[2], sk_shape[3])
        self.B, self.S, self.H_ix, self.D_ix, self.rd, self.k = B, S, H_ix, D_ix, rd, k
        self.H_sa, self.D_sa, self.dv = H_sa, D_sa, dv
        self.sk_shape, self.sk_repeat = sk_shape, sk_repeat
        self.units = B * S  # query tokens per step, whole job
        self._host = None
        if device is None:  # host-only instance (reference arm)
            return
        import torch
        from kernelswift_b200 import ops, shard

        self.ranges = shard.zigzag(S, world, rank)
        g = torch.Generator(device=device).manual_seed(1234 + rank)
        dev = device
        # resident model state (copied once): keys, latent kv, sinks, rope tables
        self.k_ix = torch.randn(B, S, D_ix, device=dev, generator=g).bfloat16()
        self.kv = torch.randn(B, S, D_sa, device=dev, generator=g).bfloat16()
        self.sink = torch.zeros(H_sa, device=dev)
        self.freqs = [_freqs(b - a, rd, a).to(dev) for a, b in self.ranges]
        # per-step activations and outputs, one set per row range of this rank
        self.q_ix, self.w, self.q_sa, self.idx, self.out = [], [], [], [], []
        for a, b in self.ranges:
            n = b - a
            self.q_ix.append(torch.randn(B, n, H_ix, D_ix, device=dev, generator=g).bfloat16())
            self.w.append((torch.rand(B, n, H_ix, device=dev, generator=g) *
                           (D_ix ** -0.5 * H_ix ** -0.5)).bfloat16())
            self.q_sa.append(torch.randn(B, n, H_sa, D_sa, device=dev, generator=g).bfloat16())
            self.idx.append(torch.empty(B, n, k, dtype=torch.int32, device=dev))
            self.out.append(torch.empty(B, n, H_sa, dv, dtype=torch.bfloat16, device=dev))
        n_mats = sk_shape[0] * sk_shape[1]
        m0, m1 = (shard.contiguous(n_mats, world, rank) or [(0, 0)])[0]
        self.sk_x = torch.randn(m1 - m0, sk_shape[2], sk_shape[3], device=dev, generator=g)
        self.sk_out = torch.empty_like(self.sk_x)
        self.ws = torch.empty(max(ops.indexer_workspace_size(B, b - a, S) for a, b in self.ranges),
                              dtype=torch.uint8, device=dev)

    def work(self):
        return self.flops(), "tensor"

    def flops(self):
        """Algorithmic FLOPs per step on this rank (causal-valid pairs for the indexer)."""
        ix = sum(2 * self.H_ix * self.D_ix * self.B * ((a + 1 + b) * (b - a) // 2)
                 for a, b in self.ranges)
        rows = sum(b - a for a, b in self.ranges)
        sa = 2 * self.B * rows * self.H_sa * self.k * (self.D_sa + self.dv)
        return {"indexer": ix, "sparse_attn": sa}

    def run(self, timers=None):
        from kernelswift_b200 import ops

        for i, (a, b) in enumerate(self.ranges):
            with _span(timers, "indexer"):
                # rows a..b-1 of a causal prefill over all S keys (row s reads keys t <= s)
                ops.indexer_topk(self.q_ix[i], self.k_ix, self.w[i], self.freqs[i], self.rd,
                                 self.S, self.k, 1, True, 0, pos0=a, out=self.idx[i],
                                 workspace=self.ws)
            with _span(timers, "sparse_attn"):
                ops.sparse_attn(self.q_sa[i], self.kv, self.sink, self.idx[i], self.D_sa ** -0.5,
                                self.dv, out=self.out[i])
        with _span(timers, "sinkhorn"):
            ops.sinkhorn(self.sk_x, self.sk_repeat, 1e-6, out=self.sk_out)

    def launches_per_step(self):
        return 3 * len(self.ranges) + 1  # (score + top-k + attention) per range, Sinkhorn

    def traffic(self, kernel):
        if kernel != "sparse_attn" or (self.H_sa, self.D_sa, self.dv, self.k) != (128, 576, 512, 2048):
            return None
        return SA_DRAM_BYTES_PER_TOKEN_MLA * self.B * sum(b - a for a, b in self.ranges)

    def host_buffers(self):
        import torch

        def pin(t):
            return torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t)

        if self._host is None:
            self._host = {"q_ix": [pin(t) for t in self.q_ix], "w": [pin(t) for t in self.w],
                          "q_sa": [pin(t) for t in self.q_sa], "sk_x": pin(self.sk_x),
                          "out": [pin(t) for t in self.out], "idx": [pin(t) for t in self.idx],
                          "sk_out": pin(self.sk_out)}
        return self._host

    def e2e_pieces(self, rows=4096):
        """The step cut into (inputs, outputs, launch) pieces for the copy/compute
        pipeline: per row range, per batch, at most ``rows`` query rows each, plus
        the Sinkhorn matrices.  Every piece is a full public-op call on its rows."""
        from kernelswift_b200 import ops

        h = self.host_buffers()
        pieces = []
        for i, (a, b) in enumerate(self.ranges):
            for bb in range(self.B):
                for r0 in range(0, b - a, rows):
                    r1 = min(b - a, r0 + rows)

                    def sl(t, i=i, bb=bb, r0=r0, r1=r1):
                        return t[i][bb:bb + 1, r0:r1]

                    def launch(i=i, bb=bb, r0=r0, r1=r1, a=a, sl=sl):
                        # the whole indexer -> sparse attention step in one library call
                        ops.dsa(sl(self.q_ix), self.k_ix[bb:bb + 1], sl(self.w), self.freqs[i][r0:r1],
                                self.rd, self.S, self.k, sl(self.q_sa), self.kv[bb:bb + 1],
                                self.sink, self.D_sa ** -0.5, self.dv, 1, True, 0, pos0=a + r0,
                                out=sl(self.out), idx_out=sl(self.idx), workspace=self.ws)

                    ins = [(sl(self.q_ix), sl(h["q_ix"])), (sl(self.w), sl(h["w"])),
                           (sl(self.q_sa), sl(h["q_sa"]))]
                    outs = [(sl(h["out"]), sl(self.out)), (sl(h["idx"]), sl(self.idx))]
                    pieces.append((ins, outs, launch))
        pieces.append(([(self.sk_x, h["sk_x"])], [(h["sk_out"], self.sk_out)],
                       lambda: ops.sinkhorn(self.sk_x, self.sk_repeat, 1e-6, out=self.sk_out)))
        return pieces

    e2e_rows = 4096  # query rows per piece of the host-buffer pipeline

    def _pipeline(self):
        if getattr(self, "_pipe", None) is None:
            self._pipe = CopyPipeline(self.e2e_pieces(self.e2e_rows))
        return self._pipe

    def run_e2e(self):
        self._pipeline().step()

    def e2e_begin(self):
        self._pipeline().begin()

    def e2e_end(self):
        self._pipeline().end()

    def e2e_note(self):
        return (f"{len(self._pipeline().pieces)} pieces per step (<= {self.e2e_rows} query rows each): "
                "host->device copies, the ops (ops.dsa: indexer -> sparse attention in one library "
                "call; ops.sinkhorn) and device->host copies on three streams, piece by piece, so "
                "copies in both directions overlap the kernels and each other")

    def e2e_bytes(self):
        nb = lambda ts: sum(t.numel() * t.element_size() for t in ts)
        h2d = nb(self.q_ix) + nb(self.w) + nb(self.q_sa) + nb([self.sk_x])
        d2h = nb(self.out) + nb(self.idx) + nb([self.sk_out])
        return h2d, d2h

    def config(self):
        return {"workload": "C5 end-to-end DSA: indexer(B=2,S=T=32768,H=64,D=128,rope=64,top-2048,"
                            "causal) -> sparse_attn(H=128,D=576,dv=512) + sinkhorn(2,32768,8,8)x20",
                "global_batch": self.B, "seq_len": self.S, "parallelism": f"rows{self.world}",
                "sharding": "zigzag causal row ranges (indexer and attention), contiguous matrices "
                            "(sinkhorn)",
                "l2": "inputs larger than L2 (126 MB) every step"}

    # ---- CPU sample of the same workload (the reference's torch forwards, host cores)
    def cpu_sample(self, budget_rows=(16, 16, 8192)):
        import torch
        from oracle import ks_ref_torch as R

        torch.set_num_threads(os.cpu_count() or 1)
        g = torch.Generator().manual_seed(0)
        n_ix, n_sa, n_sk = budget_rows
        S, rows_per_chunk = self.S, 32
        kx = torch.randn(1, S, self.D_ix, generator=g).bfloat16()
        t_ix = 0.0
        # chunks of consecutive rows spread over the sequence: a row's cost grows
        # with its position, so the mean over evenly spread chunks is the mean row
        for s0 in np.linspace(0, S - rows_per_chunk, n_ix).astype(int):
            q = torch.randn(1, rows_per_chunk, self.H_ix, self.D_ix, generator=g).bfloat16()
            w = (torch.rand(1, rows_per_chunk, self.H_ix, generator=g) *
                 (self.D_ix ** -0.5 * self.H_ix ** -0.5)).bfloat16()
            fc = _freqs_cis(rows_per_chunk, self.rd, int(s0))
            t0 = time.perf_counter()
            R.indexer_after_projections(q, w, kx, fc, self.rd, self.k, 1, 0, 0, s0=int(s0))
            t_ix += time.perf_counter() - t0
        kv = torch.randn(1, S, self.D_sa, generator=g).bfloat16()
        q = torch.randn(1, n_sa, self.H_sa, self.D_sa, generator=g).bfloat16()
        idx = torch.stack([torch.randperm(S, generator=g)[: self.k] for _ in range(n_sa)])[None].int()
        t0 = time.perf_counter()
        R.sparse_attn(q, kv, torch.zeros(self.H_sa), idx, self.D_sa ** -0.5)
        t_sa = time.perf_counter() - t0
        x = torch.randn(n_sk, 8, 8, generator=g)
        t0 = time.perf_counter()
        R.sinkhorn(x, self.sk_repeat, 1e-6)
        t_sk = time.perf_counter() - t0
        rows = self.B * S
        n_mats = self.sk_shape[0] * self.sk_shape[1]
        t_step = (t_ix / (n_ix * rows_per_chunk) * rows + t_sa / n_sa * rows +
                  t_sk / n_sk * n_mats)
        return rows / t_step, (f"the reference's torch forwards (oracle/ks_ref_torch.py) on "
                               f"{torch.get_num_threads()} threads: {n_ix} chunks of "
                               f"{rows_per_chunk} indexer rows spread over positions 0..{S-1}, "
                               f"{n_sa} sparse-attention rows, {n_sk} Sinkhorn matrices; time "
                               f"per row extrapolated to the full step")


class SingleOp(Workload):
    """One operator at one BASELINE.json configuration (C1-C4, or C5's Sinkhorn
    stage): rows split contiguously over ranks.  `tokens` limits the query rows
    per batch (small cases for profiling)."""

    def __init__(self, rank, world, device, tokens=None):
        super().__init__(rank, world, device)
        self._host = None
        self.tokens = tokens

    def launches_per_step(self):
        return self.launches

    def host_buffers(self):
        import torch

        def pin(t):
            return torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t)

        if self._host is None:
            self._host = {"in": [pin(t) for t in self.inputs], "out": [pin(t) for t in self.outputs]}
        return self._host

    def run_e2e(self):
        h = self.host_buffers()
        for d, s in zip(self.inputs, h["in"]):
            d.copy_(s, non_blocking=True)
        self.run()
        for d, s in zip(h["out"], self.outputs):
            d.copy_(s, non_blocking=True)

    def e2e_bytes(self):
        nb = lambda ts: sum(t.numel() * t.element_size() for t in ts)
        return nb(self.inputs), nb(self.outputs)

    def config(self):
        return {"workload": self.desc, "global_batch": self.B, "seq_len": self.S,
                "parallelism": f"rows{self.world}", "sharding": "contiguous rows",
                "l2": self.l2}


class SinkhornOp(SingleOp):
    """C1 (8, 4096, 4, 4) or C5's Sinkhorn stage (2, 32768, 8, 8); repeat = 20."""

    def __init__(self, rank, world, device, tokens=None, shape=(8, 4096, 4, 4)):
        super().__init__(rank, world, device, tokens)
        self.B, self.S, self.n = shape[0], (tokens or shape[1]), shape[2]
        self.units = self.B * self.S
        self.metric = "matrices/s"
        self.dtype = "f32"
        self.desc = f"Sinkhorn fp32 ({self.B}, {self.S}, {self.n}, {self.n}), 20 iterations, eps 1e-6"
        self.l2 = ("L2 flushed before every call (256 MB write); op time = CUDA-graph replays of "
                   "(flush + op) minus replays of the flush alone")
        self.flushes = True
        self.launches = 1
        if device is None:
            return
        import torch
        from kernelswift_b200 import shard

        m0, m1 = (shard.contiguous(self.units, world, rank) or [(0, 0)])[0]
        g = torch.Generator(device=device).manual_seed(7 + rank)
        self.x = torch.randn(m1 - m0, self.n, self.n, device=device, generator=g)
        self.out = torch.empty_like(self.x)
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        self.inputs, self.outputs = [self.x], [self.out]

    def work(self):
        nbytes = 2 * self.x.numel() * 4
        return {"sinkhorn": nbytes}, "hbm"

    span_name = "sinkhorn"

    def op(self):
        from kernelswift_b200 import ops

        ops.sinkhorn(self.x, 20, 1e-6, out=self.out)

    def run(self, timers=None):
        if timers is not None:
            self.flush.zero_()  # keep each step's input out of L2
        with _span(timers, "sinkhorn"):
            self.op()

    def cpu_sample(self, budget_rows=None):
        import torch
        from oracle import ks_ref_torch as R

        torch.set_num_threads(os.cpu_count() or 1)
        n = min(self.units, 65536)
        x = torch.randn(n, self.n, self.n, generator=torch.Generator().manual_seed(0))
        t0 = time.perf_counter()
        R.sinkhorn(x, 20, 1e-6)
        dt = time.perf_counter() - t0
        return n / dt, (f"the reference's torch forward (oracle/ks_ref_torch.py) on "
                        f"{torch.get_num_threads()} threads, {n} matrices")


class SparseAttnOp(SingleOp):
    """C2 (1, 128, 16, 128; N 4096; K 512) or C4 (4, 4096, 128, 576; N 32768; K 2048; dv 512)."""

    def __init__(self, rank, world, device, tokens=None, cfg="c4"):
        super().__init__(rank, world, device, tokens)
        if cfg == "c2":
            self.B, M, self.H, self.D, self.N, self.K, self.dv = 1, 128, 16, 128, 4096, 512, 128
        else:
            self.B, M, self.H, self.D, self.N, self.K, self.dv = 4, 4096, 128, 576, 32768, 2048, 512
        self.S = tokens or M
        self.units = self.B * self.S
        self.desc = (f"SparseAttention bf16 q ({self.B}, {self.S}, {self.H}, {self.D}), kv ({self.B}, "
                     f"{self.N}, {self.D}) shared latent, top-{self.K} int32 indices "
                     f"({'randperm' if cfg == 'c2' else 'causal-valid'}), dv {self.dv}")
        self.l2 = ("inputs larger than L2" if cfg == "c4"
                   else "L2 flushed before every call (256 MB write); op time = CUDA-graph replays "
                        "of (flush + op) minus replays of the flush alone")
        self.flushes = cfg != "c4"
        self.launches = 1
        self.cfg = cfg
        if device is None:
            return
        import torch
        from kernelswift_b200 import shard

        m0, m1 = (shard.contiguous(self.S, world, rank) or [(0, 0)])[0]
        g = torch.Generator(device=device).manual_seed(11 + rank)
        n = m1 - m0
        self.q = torch.randn(self.B, n, self.H, self.D, device=device, generator=g).bfloat16()
        self.kv = torch.randn(self.B, self.N, self.D, device=device, generator=g).bfloat16()
        if cfg == "c2":
            self.idx = torch.stack([torch.stack([torch.randperm(self.N, device=device, generator=g)[:self.K]
                                                 for _ in range(n)]) for _ in range(self.B)]).int()
        else:  # query m at position N - M + m attends to positions <= its own
            pos = self.N - M + m0 + torch.arange(n, device=device)
            r = torch.rand(self.B, n, self.K, device=device, generator=g)
            self.idx = (r * (pos[None, :, None] + 1).float()).long().clamp_max(self.N - 1).int()
        self.sink = torch.zeros(self.H, device=device)
        self.out = torch.empty(self.B, n, self.H, self.dv, dtype=torch.bfloat16, device=device)
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        self.inputs, self.outputs = [self.q, self.idx], [self.out]
        self.rows = n

    def work(self):
        return {"sparse_attn": 2 * self.B * self.rows * self.H * self.K * (self.D + self.dv)}, "tensor"

    def traffic(self, kernel):
        if self.cfg != "c4" or kernel != "sparse_attn":
            return None
        return SA_DRAM_BYTES_PER_TOKEN_MLA * self.B * self.rows

    span_name = "sparse_attn"

    def op(self):
        from kernelswift_b200 import ops

        ops.sparse_attn(self.q, self.kv, self.sink, self.idx, self.D ** -0.5, self.dv, out=self.out)

    def run(self, timers=None):
        if timers is not None and self.cfg == "c2":
            self.flush.zero_()
        with _span(timers, "sparse_attn"):
            self.op()

    def cpu_sample(self, budget_rows=(8,)):
        import torch
        from oracle import ks_ref_torch as R

        torch.set_num_threads(os.cpu_count() or 1)
        g = torch.Generator().manual_seed(0)
        n = max(budget_rows[0], 128 if self.cfg == "c2" else 8)
        kv = torch.randn(1, self.N, self.D, generator=g).bfloat16()
        q = torch.randn(1, n, self.H, self.D, generator=g).bfloat16()
        idx = torch.stack([torch.randperm(self.N, generator=g)[: self.K] for _ in range(n)])[None].int()
        t0 = time.perf_counter()
        R.sparse_attn(q, kv, torch.zeros(self.H), idx, self.D ** -0.5)
        dt = time.perf_counter() - t0
        return n / dt, (f"the reference's torch forward (oracle/ks_ref_torch.py) on "
                        f"{torch.get_num_threads()} threads, {n} query rows, time per row")


class IndexerOp(SingleOp):
    """C3: q (1, 4096, 64, 128) before RoPE, keys (1, 4096, 128), rope 64, top-2048, causal.
    With `seq` set (C5's indexer stage: B=2, seq 32768), `tokens` selects the LAST
    `tokens` rows of the sequence (the longest causal rows) over all `seq` keys."""

    def __init__(self, rank, world, device, tokens=None, B=1, seq=None):
        super().__init__(rank, world, device, tokens)
        self.B, self.H, self.D, self.rd, self.k = B, 64, 128, 64, 2048
        self.T = seq or tokens or 4096
        self.S = tokens or self.T
        self.row0 = self.T - self.S  # position of the first row
        self.units = self.B * self.S
        self.desc = (f"Indexer bf16 q ({self.B}, {self.S}, {self.H}, {self.D}) before RoPE, keys "
                     f"({self.B}, {self.T}, {self.D}), RoPE on the last {self.rd} dims, causal, "
                     f"top-{self.k} int64" + (f", rows {self.row0}..{self.T - 1}" if self.row0 else ""))
        self.l2 = "inputs larger than L2"
        if device is None:
            return
        import torch
        from kernelswift_b200 import ops, shard

        self.ranges = [(a + self.row0, b + self.row0) for a, b in shard.zigzag(self.S, world, rank)]
        self.launches = 2 * len(self.ranges)
        g = torch.Generator(device=device).manual_seed(13 + rank)
        self.kx = torch.randn(self.B, self.T, self.D, device=device, generator=g).bfloat16()
        self.q, self.w, self.fr, self.out = [], [], [], []
        for a, b in self.ranges:
            self.q.append(torch.randn(self.B, b - a, self.H, self.D, device=device, generator=g).bfloat16())
            self.w.append((torch.rand(self.B, b - a, self.H, device=device, generator=g) *
                           (self.D ** -0.5 * self.H ** -0.5)).bfloat16())
            self.fr.append(_freqs(b - a, self.rd, a).to(device))
            self.out.append(torch.empty(self.B, b - a, min(self.k, self.T), dtype=torch.int64,
                                        device=device))
        self.ws = torch.empty(max(ops.indexer_workspace_size(self.B, b - a, self.T) for a, b in self.ranges),
                              dtype=torch.uint8, device=device)
        self.inputs, self.outputs = self.q + self.w, self.out

    def work(self):
        return {"indexer": sum(2 * self.H * self.D * self.B * ((a + 1 + b) * (b - a) // 2)
                               for a, b in self.ranges)}, "tensor"

    def run(self, timers=None):
        from kernelswift_b200 import ops

        for i, (a, b) in enumerate(self.ranges):
            with _span(timers, "indexer"):
                ops.indexer_topk(self.q[i], self.kx, self.w[i], self.fr[i], self.rd, self.T, self.k,
                                 1, True, 0, pos0=a, out=self.out[i], workspace=self.ws)

    def cpu_sample(self, budget_rows=(8,)):
        import torch
        from oracle import ks_ref_torch as R

        torch.set_num_threads(os.cpu_count() or 1)
        g = torch.Generator().manual_seed(0)
        n, rows_per_chunk = budget_rows[0], min(32, self.S)
        kx = torch.randn(1, self.T, self.D, generator=g).bfloat16()
        t_ix = 0.0
        for s0 in np.linspace(self.row0, self.T - rows_per_chunk, n).astype(int):
            q = torch.randn(1, rows_per_chunk, self.H, self.D, generator=g).bfloat16()
            w = (torch.rand(1, rows_per_chunk, self.H, generator=g) *
                 (self.D ** -0.5 * self.H ** -0.5)).bfloat16()
            t0 = time.perf_counter()
            R.indexer_after_projections(q, w, kx, _freqs_cis(rows_per_chunk, self.rd, int(s0)),
                                        self.rd, self.k, 1, 0, 0, s0=int(s0))
            t_ix += time.perf_counter() - t0
        return n * rows_per_chunk / t_ix, (
            f"the reference's torch forward (oracle/ks_ref_torch.py) on {torch.get_num_threads()} "
            f"threads, {n} chunks of {rows_per_chunk} rows spread over positions "
            f"{self.row0}..{self.T - 1}, time per row")


class CopyPipeline:
    """Host-buffer steps with the copies overlapped: piece j's host->device copy
    runs on one stream, its ops on the current stream, its device->host copy on a
    third.  Events keep each buffer's uses in order across steps (a piece's input
    is not overwritten before the previous step's ops read it, its output not
    before the previous step's copy-out read it), so every step still moves all
    of its inputs in and all of its results out."""

    def __init__(self, pieces):
        import torch

        self.pieces = pieces
        self.s_in, self.s_out = torch.cuda.Stream(), torch.cuda.Stream()
        n = len(pieces)
        self.ev_in = [torch.cuda.Event() for _ in range(n)]
        self.ev_done = [torch.cuda.Event() for _ in range(n)]
        self.ev_out = [torch.cuda.Event() for _ in range(n)]

    def begin(self):
        """Order the copy streams after all work already queued on the current
        stream (the timing event of the region that follows)."""
        import torch

        ev = torch.cuda.Event()
        ev.record()
        self.s_in.wait_event(ev)
        self.s_out.wait_event(ev)

    def step(self):
        import torch

        cs = torch.cuda.current_stream()
        for j, (ins, outs, launch) in enumerate(self.pieces):
            with torch.cuda.stream(self.s_in):
                self.s_in.wait_event(self.ev_done[j])
                for d, hsrc in ins:
                    d.copy_(hsrc, non_blocking=True)
                self.ev_in[j].record(self.s_in)
            cs.wait_event(self.ev_in[j])
            cs.wait_event(self.ev_out[j])
            launch()
            self.ev_done[j].record(cs)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(self.ev_done[j])
                for hdst, d in outs:
                    hdst.copy_(d, non_blocking=True)
                self.ev_out[j].record(self.s_out)

    def end(self):
        """Make the current stream wait for every copy queued so far."""
        import torch

        cs = torch.cuda.current_stream()
        cs.wait_stream(self.s_in)
        cs.wait_stream(self.s_out)


def _span(timers, name):
    return timers.span(name) if timers is not None else _null()


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class Timers:
    """CUDA-event spans per kernel family on the current stream."""

    def __init__(self):
        self.spans = {}

    def span(self, name):
        import torch

        t = self

        class _S:
            def __enter__(s):
                s.a = torch.cuda.Event(enable_timing=True)
                s.b = torch.cuda.Event(enable_timing=True)
                s.a.record()
                return s

            def __exit__(s, *exc):
                s.b.record()
                t.spans.setdefault(name, []).append((s.a, s.b))
                return False

        return _S()

    def per_step_ms(self, steps):
        """Total device time of each kernel family per step."""
        return {k: sum(a.elapsed_time(b) for a, b in v) / steps for k, v in self.spans.items()}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of the GPU that `index` names in this process.  The GPU is
    named to nvidia-smi by its UUID: a CUDA index can differ from nvidia-smi's when
    CUDA_VISIBLE_DEVICES remaps the devices."""

    def __init__(self, index):
        import torch

        self.index = index
        try:
            self.gpu_id = "GPU-" + str(torch.cuda.get_device_properties(index).uuid)
        except (AttributeError, RuntimeError):
            self.gpu_id = str(index)
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


WORKLOADS = {
    "dsa_e2e": DsaE2E,
    "c1": lambda r, w, d, tokens=None: SinkhornOp(r, w, d, tokens, (8, 4096, 4, 4)),
    "c2": lambda r, w, d, tokens=None: SparseAttnOp(r, w, d, tokens, "c2"),
    "c3": lambda r, w, d, tokens=None: IndexerOp(r, w, d, tokens),
    "c4": lambda r, w, d, tokens=None: SparseAttnOp(r, w, d, tokens, "c4"),
    "c5_indexer": lambda r, w, d, tokens=None: IndexerOp(r, w, d, tokens, B=2, seq=32768),
    "c5_sinkhorn": lambda r, w, d, tokens=None: SinkhornOp(r, w, d, tokens, (2, 32768, 8, 8)),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="dsa_e2e", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-rows", type=int, default=None,
                    help="query rows per piece of the host-buffer (e2e) pipeline")
    ap.add_argument("--no-per-op", action="store_true",
                    help="skip the per-operator block of the default workload's line")
    ap.add_argument("--tokens", type=int, default=None,
                    help="query rows per batch (small cases for profiling; not a bench line)")
    return ap.parse_args()


def timed_region(wl, steps, world, local, device, barrier):
    """Time `steps` device-resident steps of `wl` (already warmed up): CUDA events on
    the current stream around the whole loop, bracketed by a barrier and a device
    synchronize on both sides, max over ranks; per-kernel spans; the SM clocks
    sampled meanwhile.  Returns (ms per step, spans, clocks, ms with the flush):
    for workloads that flush L2 between steps the step time is the sum of the op
    spans and the whole-loop time (flush included) is returned beside it."""
    import torch
    import torch.distributed as dist
    from kernelswift_b200 import ops

    if wl.flushes and hasattr(wl, "op"):
        return timed_region_graphs(wl, steps, world, local, device, barrier)
    clocks = ClockSampler(local)
    clocks.start()
    timers = Timers()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        wl.run(timers)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / steps
    clk = clocks.stop()
    ops.device_status()
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    spans = timers.per_step_ms(steps)
    ms_with_flush = None
    if wl.flushes:
        ms_with_flush = ms
        t = torch.tensor([sum(spans.values())], device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, spans, clk, ms_with_flush


def timed_region_graphs(wl, steps, world, local, device, barrier):
    """Device time of a single-op workload whose input fits in L2: two CUDA graphs,
    (L2 flush + op) and (L2 flush alone), each replayed `steps` times under CUDA
    events; the op's time per call is the difference of the two per-replay times.
    The graphs take the host's launch work out of the measurement (for a kernel of
    tens of microseconds an event span around a Python call would time the call),
    and every timed call starts from a flushed L2."""
    import torch
    import torch.distributed as dist
    from kernelswift_b200 import ops

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g_op, g_fl = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g_op, stream=side):
            wl.flush.zero_()
            wl.op()
        with torch.cuda.graph(g_fl, stream=side):
            wl.flush.zero_()
    torch.cuda.current_stream().wait_stream(side)
    for g in (g_op, g_fl):
        for _ in range(3):
            g.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ev[0].record()
    for _ in range(steps):
        g_op.replay()
    ev[1].record()
    ev[2].record()
    for _ in range(steps):
        g_fl.replay()
    ev[3].record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ops.device_status()
    t = torch.tensor([ev[0].elapsed_time(ev[1]) / steps, ev[2].elapsed_time(ev[3]) / steps],
                     device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    with_flush, flush_only = float(t[0].item()), float(t[1].item())
    ms = max(with_flush - flush_only, 1e-6)
    del g_op, g_fl
    return ms, {wl.span_name: ms}, clk, with_flush


def roofline_of(wl, spans, peaks):
    """Roofline record of the workload's dominant kernel: algorithmic work per step
    over its CUDA-event time per step, against the measured peak."""
    work, bound = wl.work()
    dom = max(work, key=lambda k: spans.get(k, 0.0))
    if bound == "tensor":
        ach = work[dom] / (spans[dom] / 1e3) / 1e12
        peak, unit, src = peaks["bf16_tflops_sustained"], "TFLOP/s", "sustained bf16"
    else:
        ach = work[dom] / (spans[dom] / 1e3) / 1e9
        peak, unit, src = peaks["hbm_gbs"], "GB/s", "HBM copy"
    return {"bound": bound, "kernel": dom, "achieved": round(ach, 1), "peak": peak,
            "unit": unit, "frac": round(ach / peak, 4), "traffic": wl.traffic(dom),
            "algorithmic_per_step": work[dom],
            "peak_source": f"{peaks['source']} ({src})",
            "per_kernel_ms": {k: round(v, 4) for k, v in spans.items()}}


# BASELINE.json's per-operator configurations, timed after the headline workload
PER_OP = ["c1", "c2", "c3", "c4", "c5_sinkhorn"]


def per_op_block(rank, world, local, device, barrier, peaks, target_s=0.4):
    """µs per call, throughput and roofline of each operator at its own
    configuration (rows split over the ranks like the headline workload).  Each is
    warmed up, then timed over enough calls to fill ~`target_s` seconds (so the
    clock sampler sees the region), the same number on every rank."""
    import torch
    import torch.distributed as dist

    res = {}
    for name in PER_OP:
        wl = WORKLOADS[name](rank, world, device)
        for _ in range(3):
            wl.run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            wl.run()
        e1.record()
        torch.cuda.synchronize()
        est = max(e0.elapsed_time(e1) / 3, 1e-3)
        t = torch.tensor([min(2000, max(10, int(target_s * 1e3 / est)))], device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        steps = int(t.item())
        ms, spans, clk, ms_flush = timed_region(wl, steps, world, local, device, barrier)
        rf = roofline_of(wl, spans, peaks)
        res[name] = {"workload": wl.config()["workload"], "us_per_call": round(ms * 1e3, 2),
                     "value": wl.units / (ms / 1e3), "unit": wl.metric, "calls": steps,
                     "launches_per_call": wl.launches_per_step(), "l2": wl.config()["l2"],
                     "roofline": {k: rf[k] for k in ("bound", "kernel", "achieved", "peak", "unit",
                                                      "frac", "traffic")},
                     "clocks": clk}
        if ms_flush is not None:
            res[name]["us_per_call_with_l2_flush"] = round(ms_flush * 1e3, 2)
        del wl
        torch.cuda.empty_cache()
    return res


# v1 latency the reference publishes for its own default inputs (Ascend 910B3; other
# hardware, context only): optimized/sinkhorn_project/design.md:120-122,
# optimized/sparse_attention/README.md:58-59, optimized/indexer_project/design.md:173-174
REF_910B3_V1_MS = {"sinkhorn": 0.14, "sparse_attention": 0.92, "indexer": 1.741}


def dropin_block(device, calls=200, warmup=20):
    """The three drop-in ModelNew forwards at the reference's own default inputs
    (each module's get_init_inputs / get_inputs, what the reference's harness
    times), as its protocol measures them: warm-up, then the median of calls each
    followed by a device synchronize (wall clock; the device span of each call,
    CUDA events, beside it).  Each rank runs the whole inputs on its own GPU."""
    import importlib
    import torch

    res = {}
    for name in ("sinkhorn", "sparse_attention", "indexer"):
        mod = importlib.import_module(f"kernelswift_b200.{name}")
        torch.manual_seed(42)
        model = mod.ModelNew(*mod.get_init_inputs()).to(device)
        inputs = [x.to(device) if torch.is_tensor(x) else x for x in mod.get_inputs()]
        wall, dev = [], []
        with torch.no_grad():
            for _ in range(warmup):
                model(*inputs)
            torch.cuda.synchronize()
            for _ in range(calls):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0 = time.perf_counter()
                e0.record()
                model(*inputs)
                e1.record()
                torch.cuda.synchronize()
                wall.append((time.perf_counter() - t0) * 1e6)
                dev.append(e0.elapsed_time(e1) * 1e3)
        res[name] = {"inputs": [list(x.shape) if torch.is_tensor(x) else x for x in inputs],
                     "us_per_call": round(statistics.median(wall), 1),
                     "device_us_per_call": round(statistics.median(dev), 1),
                     "reference_910B3_v1_us": REF_910B3_V1_MS[name] * 1e3}
        del model, inputs
        torch.cuda.empty_cache()
    return res


def main():
    a = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if a.impl == "reference":
        return reference_arm(a, rank, world)
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    wl = WORKLOADS[a.workload](rank, world, device, tokens=a.tokens) if a.tokens else WORKLOADS[a.workload](rank, world, device)
    if a.e2e_rows:
        wl.e2e_rows = a.e2e_rows
    from kernelswift_b200 import ops

    for _ in range(a.warmup):
        wl.run()
    torch.cuda.synchronize()
    ops.device_status()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timed region
    ms, spans, clk, ms_with_flush = timed_region(wl, a.steps, world, local, device, barrier)

    # ---- end to end through the public ops, host buffers
    e2e = None
    if not a.no_e2e:
        wl.host_buffers()
        wl.e2e_begin()
        wl.run_e2e()
        wl.e2e_end()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        wl.e2e_begin()
        for _ in range(a.steps):
            wl.run_e2e()
        wl.e2e_end()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        t = torch.tensor([e0.elapsed_time(e1) / a.steps], device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        h2d, d2h = wl.e2e_bytes()  # this rank's copies; the line reports the whole job's
        if world > 1:
            nb = torch.tensor([h2d, d2h], dtype=torch.int64, device=device)
            dist.all_reduce(nb, op=dist.ReduceOp.SUM)
            h2d, d2h = int(nb[0].item()), int(nb[1].item())
        e2e = {"value": wl.units / (float(t.item()) / 1e3), "unit": wl.metric,
               "ms_per_step": float(t.item()), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "copies": wl.e2e_note()}

    peaks = measured_peaks()
    roofline = roofline_of(wl, spans, peaks)
    line = {"metric": wl.metric, "value": wl.units / (ms / 1e3), "unit": wl.metric, "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": wl.dtype,
            "data": "synthetic (seeded, shapes and distributions of the configuration)",
            "config": wl.config(), "roofline": roofline, "e2e": e2e,
            "gpu_launches": wl.launches_per_step() * a.steps, "clocks": clk}
    if ms_with_flush is not None:
        line["ms_per_step_with_l2_flush"] = ms_with_flush
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        wl.cpu_sample()  # first call pays the BLAS / allocator warm-up
        v, sample = wl.cpu_sample()
        line["cpu_baseline"] = {"value": v, "unit": wl.metric, "cores": os.cpu_count(),
                                "kind": "port", "sample": sample}
    if a.workload == "dsa_e2e" and a.tokens is None and not a.no_per_op:
        del wl
        torch.cuda.empty_cache()
        line["per_op"] = per_op_block(rank, world, local, device, barrier, peaks)
        line["dropin"] = dropin_block(device)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def reference_arm(a, rank, world):
    """The reference algorithm (its torch forwards restated in oracle/, on the host
    cores) on a bounded row sample of the workload per step, throughput
    extrapolated per row."""
    if rank != 0:
        return
    wl = WORKLOADS[a.workload](0, world, None)
    vals = []
    sample = ""
    for i in range(a.warmup + a.steps):
        v, sample = wl.cpu_sample()
        if i >= a.warmup:
            vals.append(v)
    v = statistics.median(vals)
    cfg = wl.config()
    cfg["parallelism"] = "host cores"
    line = {"impl": "reference", "metric": wl.metric, "value": v, "unit": wl.metric,
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": wl.units / v * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded)", "config": cfg,
            "cpu_baseline": {"value": v, "unit": wl.metric, "cores": os.cpu_count(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": v, "unit": wl.metric, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
