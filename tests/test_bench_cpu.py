"""Host logic of bench.py's end-to-end (host-buffer) step, on CPU: the pieces the
copy pipeline moves and launches tile every input and output of the step exactly
once, for every rank of 1, 2 and 4 (zigzag row ranges, ragged piece sizes)."""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


@pytest.fixture
def no_pinning(monkeypatch):
    """Pinned host memory needs a CUDA driver; plain host memory stands in."""
    real = torch.empty

    def empty(*a, **k):
        k.pop("pin_memory", None)
        return real(*a, **k)

    monkeypatch.setattr(torch, "empty", empty)


def _segments(pieces):
    seg = {}
    for ins, outs, _ in pieces:
        for dev, host in ins + [(d, h) for h, d in outs]:
            assert dev.shape == host.shape and dev.is_contiguous() and host.is_contiguous()
            base = dev.untyped_storage().data_ptr()
            seg.setdefault(base, []).append((dev.data_ptr() - base, dev.numel() * dev.element_size()))
    return seg


@pytest.mark.parametrize("world", [1, 2, 4])
def test_e2e_pieces_tile_the_step(built_lib, no_pinning, world):
    import bench

    for rank in range(world):
        wl = bench.DsaE2E(rank, world, torch.device("cpu"), tokens=3000, H_sa=8, D_sa=64, dv=64,
                          H_ix=16, D_ix=64, rd=16, k=64)
        pieces = wl.e2e_pieces(rows=700)
        seg = _segments(pieces)
        tensors = wl.q_ix + wl.w + wl.q_sa + wl.idx + wl.out + [wl.sk_x, wl.sk_out]
        for t in tensors:
            spans = sorted(seg[t.untyped_storage().data_ptr()])
            pos = 0
            for off, n in spans:
                assert off == pos, "gap or overlap between pieces"
                pos += n
            assert pos == t.numel() * t.element_size()
        h2d, d2h = wl.e2e_bytes()
        moved_in = sum(d.numel() * d.element_size() for ins, _, _ in pieces for d, _ in ins)
        moved_out = sum(d.numel() * d.element_size() for _, outs, _ in pieces for _, d in outs)
        assert (moved_in, moved_out) == (h2d, d2h)
