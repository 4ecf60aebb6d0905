"""ks_indexer_noalloc, the indexer entry point that allocates nothing, returns the
same indices as ks_indexer with a caller-provided workspace.

Some callers cannot allocate device memory: a process whose device memory is
owned by another allocator (a framework's caching allocator or a fixed pool that
must not be bypassed), a latency-critical path that must not call cudaMalloc
because it can synchronise the device, or a host such as an FFI binding or plugin
with no device allocator to call.  For them the indexer keeps its score rows in a
fixed 32 MiB device array inside the library instead of a workspace.

The file name makes pytest collect it last, so a run that stops at the first
failure has run every other test before this one.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(B, S, T, H, D, rd, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, S, H, D, device="cuda", generator=g).bfloat16()
    kv = torch.randn(B, T, D, device="cuda", generator=g).bfloat16()
    w = (torch.rand(B, S, H, device="cuda", generator=g) * (D ** -0.5 * H ** -0.5)).bfloat16()
    inv = 1.0 / (10000.0 ** (torch.arange(0, rd, 2, device="cuda").float() / max(rd, 1)))
    ang = torch.outer(torch.arange(S, device="cuda").float(), inv)
    freqs = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    return q, kv, w, freqs


def test_noalloc_matches_workspace_entry_point(cuda_ok):
    """Calls in a row with different shapes: none may see an earlier call's
    leftovers in the shared scratch (the last fills it exactly, after a call with
    longer rows)."""
    from kernelswift_b200 import _lib, ops

    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [  # B, S, T, H, D, rd, k, ratio, causal, offset
        (1, 512, 512, 64, 128, 64, 256, 1, 1, 0),
        (2, 300, 77, 16, 64, 32, 128, 4, 1, 0),
        (1, 130, 300, 32, 128, 64, 64, 1, 0, 9),       # not causal (decode-style), + offset
        (1, 256, 16384, 64, 128, 64, 512, 1, 1, 0),    # longer rows than the next call
        (1, 2048, 8192, 64, 128, 64, 2048, 1, 1, 0),   # score rows fill the 32 MiB exactly
    ]
    for seed, (B, S, T, H, D, rd, k, ratio, causal, offset) in enumerate(cases):
        q, kv, w, fr = _inputs(B, S, T, H, D, rd, seed)
        kk = min(k, T)
        ref = torch.empty(B, S, kk, dtype=torch.int64, device="cuda")
        ws = torch.empty(lib.ks_indexer_workspace_size(B, S, T), dtype=torch.uint8, device="cuda")
        _lib.check(lib.ks_indexer(q.data_ptr(), kv.data_ptr(), T, w.data_ptr(), fr.data_ptr(),
                                  B, S, H, D, T, rd, 0, causal, ratio, k, offset, ref.data_ptr(),
                                  _lib.KS_INT64, ws.data_ptr(), ws.numel(), stream), "ks_indexer")
        got = torch.full_like(ref, -7)
        _lib.check(lib.ks_indexer_noalloc(q.data_ptr(), kv.data_ptr(), T, w.data_ptr(),
                                          fr.data_ptr(), B, S, H, D, T, rd, 0, causal, ratio, k,
                                          offset, got.data_ptr(), _lib.KS_INT64, stream),
                   "ks_indexer_noalloc")
        ops.device_status()
        assert torch.equal(got, ref), f"case {seed}: {(got != ref).sum().item()} indices differ"


def test_noalloc_rejects_calls_beyond_its_scratch(cuda_ok):
    """Score rows that would not fit the fixed scratch are refused before any launch."""
    from kernelswift_b200 import _lib

    lib = _lib.lib()
    B, S, T, H, D = 1, 8192, 8192, 64, 128  # 128 MiB of scores > 32 MiB
    small = torch.zeros(1024, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(16, dtype=torch.int64, device="cuda")
    rc = lib.ks_indexer_noalloc(small.data_ptr(), small.data_ptr(), T, small.data_ptr(),
                                small.float().data_ptr(), B, S, H, D, T, 64, 0, 1, 1, 2048, 0,
                                out.data_ptr(), _lib.KS_INT64, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.KS_ERR_WORKSPACE
    assert b"scratch" in lib.ks_last_error()
