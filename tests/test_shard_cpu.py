"""Row sharding on CPU ranks (gloo, world size 2): the sharded-and-gathered result
equals the single-rank result, zigzag ranges balance causal work, and a rank that
never joins a collective makes the others fail within a short timeout instead of
hanging.  The per-rank compute is the oracle (no GPU)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kernelswift_b200 import shard
from oracle import ks_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_ranges_partition_and_balance():
    for n in (1, 7, 64, 4096, 32768):
        for world in (1, 2, 4, 8):
            for fn in (shard.contiguous, shard.zigzag):
                rows = sorted(r for rank in range(world) for a, b in fn(n, world, rank)
                              for r in range(a, b))
                assert rows == list(range(n))
    costs = [shard.causal_cost(shard.zigzag(32768, 8, r)) for r in range(8)]
    assert max(costs) / min(costs) < 1.001
    costs_c = [shard.causal_cost(shard.contiguous(32768, 8, r)) for r in range(8)]
    assert max(costs_c) / min(costs_c) > 10  # why zigzag is used for the indexer


def _indexer_worker(rank, world, port, q, kv, w, freqs, rd, k, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    S = q.shape[1]
    ranges = shard.zigzag(S, world, rank)
    parts = []
    for a, b in ranges:
        idx, _ = O.indexer_forward(q[:, a:b], kv, w[:, a:b], freqs[a:b], rd, k, 1, 0, 0, s0=a)
        parts.append(torch.from_numpy(idx))
    local = torch.cat(parts, dim=1)
    all_ranges = [shard.zigzag(S, world, r) for r in range(world)]
    full = shard.gather_rows(local, all_ranges, dim=1)
    if rank == 0:
        out_q.put(full.numpy())
    dist.destroy_process_group()


def test_zigzag_indexer_shards_equal_whole_call():
    rng = np.random.default_rng(0)
    B, S, H, D, rd, k = 1, 96, 16, 64, 32, 32
    q = O.f32_to_bf16(rng.standard_normal((B, S, H, D)).astype(np.float32))
    kv = O.f32_to_bf16(rng.standard_normal((B, S, D)).astype(np.float32))
    w = O.f32_to_bf16(rng.uniform(0, 0.02, (B, S, H)).astype(np.float32))
    ang = np.outer(np.arange(S), 1.0 / 10000.0 ** (np.arange(0, rd, 2) / rd)).astype(np.float32)
    freqs = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
    whole, _ = O.indexer_forward(q, kv, w, freqs, rd, k, 1, 0, 0)
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_indexer_worker, args=(r, 2, port, q, kv, w, freqs, rd, k, out_q))
             for r in range(2)]
    for p in procs:
        p.start()
    got = out_q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.array_equal(got, whole)


def _dropout_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        # leaves between steps without joining the next collective
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()  # flush before leaving
        os._exit(0)
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        result_q.put((rank, "completed"))
    except Exception as e:  # the surviving rank gets an error, not a hang
        result_q.put((rank, "error:" + type(e).__name__))
    result_q.close()
    result_q.join_thread()
    os._exit(0)


def test_rank_dropout_fails_fast():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=90) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0].startswith("error:")
