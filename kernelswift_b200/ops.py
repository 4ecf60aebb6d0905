"""torch-facing operators over the C ABI of libks_b200.so.

These are the B200 counterparts of the reference's torch extension ops
(KernelSwift ``optimized/*/op_extension``):

* ``sinkhorn``        <- ``sinkhorn_ext.sinkhorn`` (sinkhorn_torch.cpp:18-66)
* ``sparse_attn``     <- ``torch.ops.npu.sparse_attn_megakernel_basic`` (sparse_attn_torch.cpp:96-160)
* ``indexer_topk``    <- ``indexer_ops.rope_inplace`` + ``fused_qk_reduce`` + ``topk_mask``
  (indexer_torch.cpp:100-268), fused behind one call
* ``indexer_scores`` / ``topk_rows`` expose the two indexer stages separately.
* ``dsa`` runs the indexer's int32 top-k straight into ``sparse_attn`` in one call.
* ``proj_rope``: the indexer's projections (``wq_b`` + RoPE, ``weights_proj`` x scale)
  on the tensor cores, the producer of ``indexer_topk``'s inputs.
* ``quant_fp8_rows`` / ``indexer_topk_fp8`` / ``indexer_scores_fp8``: the FP8 indexer
  (``ModelArgs.dtype = "fp8"``), which the reference declares but does not implement.

Every op runs on the current CUDA stream of its input's device, validates its
arguments like the reference (a ``RuntimeError`` on a bad dtype, device, shape
or layout) and has no CPU fallback.
"""
from __future__ import annotations

import torch

from ._lib import KS_INT32, KS_INT64, check, lib

_DV_MAX = 512


def _require_cuda(name: str, *tensors: torch.Tensor) -> None:
    for t in tensors:
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise RuntimeError(f"{name}: inputs must be CUDA tensors")
        if not t.is_contiguous():
            raise RuntimeError(f"{name}: inputs must be contiguous")
    dev = tensors[0].device
    if any(t.device != dev for t in tensors):
        raise RuntimeError(f"{name}: inputs must be on one device")


def _check_out(name: str, out: torch.Tensor, shape, dtype, device) -> None:
    """A caller-supplied output must be exactly what the kernel writes: the kernels
    take a raw pointer and would write past a smaller or differently typed buffer."""
    if not isinstance(out, torch.Tensor):
        raise RuntimeError(f"{name}: out must be a tensor")
    if out.dtype != dtype:
        raise RuntimeError(f"{name}: out must be {dtype}, got {out.dtype}")
    if tuple(out.shape) != tuple(shape):
        raise RuntimeError(f"{name}: out must have shape {tuple(shape)}, got {tuple(out.shape)}")
    if out.device != device:
        raise RuntimeError(f"{name}: out must be on {device}, got {out.device}")
    if not out.is_contiguous():
        raise RuntimeError(f"{name}: out must be contiguous")


def _check_workspace(name: str, ws: torch.Tensor, need: int, device) -> None:
    if not isinstance(ws, torch.Tensor):
        raise RuntimeError(f"{name}: workspace must be a tensor")
    if ws.device != device:
        raise RuntimeError(f"{name}: workspace must be on {device}, got {ws.device}")
    if not ws.is_contiguous():
        raise RuntimeError(f"{name}: workspace must be contiguous")
    if ws.numel() * ws.element_size() < need:
        raise RuntimeError(f"{name}: workspace of {need} bytes needed, got "
                           f"{ws.numel() * ws.element_size()}")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def sinkhorn(x: torch.Tensor, repeat: int = 10, eps: float = 1e-6,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Sinkhorn normalisation over the last two dims of ``x`` ([..., n, n] fp32)."""
    if x.dtype != torch.float32:
        raise RuntimeError("sinkhorn: x must be float32")
    if x.dim() < 2 or x.shape[-1] != x.shape[-2]:
        raise RuntimeError("sinkhorn: x must be [..., n, n]")
    _require_cuda("sinkhorn", x)
    if out is None:
        out = torch.empty_like(x)
    else:
        _check_out("sinkhorn", out, x.shape, torch.float32, x.device)
    n = x.shape[-1]
    n_mats = x.numel() // (n * n) if n else 0
    with torch.cuda.device(x.device):
        check(lib().ks_sinkhorn(_ptr(x), _ptr(out), n_mats, n, int(repeat), float(eps),
                                _stream(x)), "ks_sinkhorn")
    return out


def sparse_attn(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor,
                topk_idxs: torch.Tensor, softmax_scale: float, dv: int | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Top-k gathered MQA attention with a per-head sink (baseline/sparse_attention.py:5-42).

    q bf16 [B,M,H,D], kv bf16 [B,N,D], attn_sink fp32 [H], topk_idxs int32 [B,M,K].
    Returns bf16 [B,M,H,dv] = the first ``dv`` (default D) output columns."""
    if q.dtype != torch.bfloat16 or kv.dtype != torch.bfloat16:
        raise RuntimeError("sparse_attn: q and kv must be bfloat16")
    if attn_sink.dtype != torch.float32:
        raise RuntimeError("sparse_attn: attn_sink must be float32")
    if topk_idxs.dtype != torch.int32:
        raise RuntimeError("sparse_attn: topk_idxs must be int32")
    if q.dim() != 4 or kv.dim() != 3 or attn_sink.dim() != 1 or topk_idxs.dim() != 3:
        raise RuntimeError("sparse_attn: expected q [b,m,h,d], kv [b,n,d], sink [h], idx [b,m,k]")
    B, M, H, D = q.shape
    N, K = kv.shape[1], topk_idxs.shape[2]
    if kv.shape[0] != B or kv.shape[2] != D:
        raise RuntimeError("sparse_attn: kv shape mismatch")
    if attn_sink.shape[0] != H:
        raise RuntimeError("sparse_attn: attn_sink shape mismatch")
    if topk_idxs.shape[0] != B or topk_idxs.shape[1] != M:
        raise RuntimeError("sparse_attn: topk_idxs shape mismatch")
    _require_cuda("sparse_attn", q, kv, attn_sink, topk_idxs)
    dv = D if dv is None else int(dv)
    if out is None:
        out = torch.empty((B, M, H, dv), dtype=torch.bfloat16, device=q.device)
    else:
        _check_out("sparse_attn", out, (B, M, H, dv), torch.bfloat16, q.device)
    with torch.cuda.device(q.device):
        if dv <= _DV_MAX:
            check(lib().ks_sparse_attn(_ptr(q), _ptr(kv), _ptr(attn_sink), _ptr(topk_idxs),
                                       _ptr(out), B, M, H, D, N, K, 0, dv, float(softmax_scale),
                                       _stream(q)), "ks_sparse_attn")
        else:  # output wider than one pass: column slices, each a full kernel call
            for c0 in range(0, dv, _DV_MAX):
                c1 = min(dv, c0 + _DV_MAX)
                part = torch.empty((B, M, H, c1 - c0), dtype=torch.bfloat16, device=q.device)
                check(lib().ks_sparse_attn(_ptr(q), _ptr(kv), _ptr(attn_sink), _ptr(topk_idxs),
                                           _ptr(part), B, M, H, D, N, K, c0, c1 - c0,
                                           float(softmax_scale), _stream(q)), "ks_sparse_attn")
                out[..., c0:c1].copy_(part)
    return out


def _indexer_args(q, k, w, freqs, T):
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise RuntimeError("indexer: q, k and w must be bfloat16")
    if freqs is not None and freqs.dtype != torch.float32:
        raise RuntimeError("indexer: freqs must be float32 [s, rope_dim/2, 2]")
    if q.dim() != 4 or k.dim() != 3 or w.dim() != 3:
        raise RuntimeError("indexer: expected q [b,s,h,d], k [b,t,d], w [b,s,h]")
    B, S, H, D = q.shape
    if k.shape[0] < B or k.shape[2] != D or k.shape[1] < T:
        raise RuntimeError("indexer: k shape mismatch")
    if tuple(w.shape) != (B, S, H):
        raise RuntimeError("indexer: w shape mismatch")
    ts = [q, k[:B], w] + ([freqs] if freqs is not None else [])
    _require_cuda("indexer", *ts)
    return B, S, H, D


def indexer_workspace_size(B: int, S: int, T: int) -> int:
    return int(lib().ks_indexer_workspace_size(B, S, T))


def indexer_topk(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, freqs: torch.Tensor | None,
                 rope_dim: int, T: int, topk: int, ratio: int = 1, causal: bool = True,
                 offset: int = 0, pos0: int = 0, out_dtype: torch.dtype = torch.int64,
                 out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Indexer top-k after the projections (baseline/indexer.py:170-205).

    q bf16 [B,S,H,D] before RoPE, k bf16 [B,Tk>=T,D] (rows t < T used), w bf16
    [B,S,H], freqs fp32 [S, rope_dim/2, 2].  Returns [B,S,min(topk,T)]."""
    B, S, H, D = _indexer_args(q, k, w, freqs, T)
    kk = min(int(topk), int(T))
    if out is None:
        out = torch.empty((B, S, kk), dtype=out_dtype, device=q.device)
    elif out.dtype not in (torch.int32, torch.int64):
        raise RuntimeError("indexer: out must be int32 or int64")
    else:
        _check_out("indexer", out, (B, S, kk), out.dtype, q.device)
    if T == 0:
        return out
    need = indexer_workspace_size(B, S, T)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    else:
        _check_workspace("indexer", workspace, need, q.device)
    with torch.cuda.device(q.device):
        check(lib().ks_indexer(_ptr(q), _ptr(k), k.shape[1], _ptr(w), _ptr(freqs), B, S, H, D,
                               int(T), int(rope_dim), int(pos0), int(bool(causal)), int(ratio),
                               int(topk), int(offset), _ptr(out),
                               KS_INT64 if out.dtype == torch.int64 else KS_INT32,
                               _ptr(workspace), workspace.numel() * workspace.element_size(),
                               _stream(q)), "ks_indexer")
    return out


def dsa(q_ix: torch.Tensor, k_ix: torch.Tensor, w: torch.Tensor, freqs: torch.Tensor | None,
        rope_dim: int, T: int, topk: int, q_sa: torch.Tensor, kv: torch.Tensor,
        attn_sink: torch.Tensor, softmax_scale: float, dv: int | None = None, ratio: int = 1,
        causal: bool = True, offset: int = 0, pos0: int = 0, out: torch.Tensor | None = None,
        idx_out: torch.Tensor | None = None, workspace: torch.Tensor | None = None
        ) -> tuple[torch.Tensor, torch.Tensor]:
    """One DeepSeek-sparse-attention step in a single library call: the indexer's
    top-k (``indexer_topk`` with int32 output) feeding ``sparse_attn`` on the same
    query rows (baseline/indexer.py:195-205 -> baseline/sparse_attention.py:16-17).

    q_ix bf16 [B,S,H_ix,D_ix] before RoPE, k_ix bf16 [B,Tk>=T,D_ix], w bf16
    [B,S,H_ix], freqs fp32 [S, rope_dim/2, 2]; q_sa bf16 [B,S,H_sa,D_sa], kv bf16
    [B,N,D_sa], attn_sink fp32 [H_sa].  Returns (out bf16 [B,S,H_sa,dv], indices
    int32 [B,S,min(topk,T)])."""
    B, S, H, D = _indexer_args(q_ix, k_ix, w, freqs, T)
    if q_sa.dtype != torch.bfloat16 or kv.dtype != torch.bfloat16:
        raise RuntimeError("dsa: q_sa and kv must be bfloat16")
    if attn_sink.dtype != torch.float32:
        raise RuntimeError("dsa: attn_sink must be float32")
    if q_sa.dim() != 4 or kv.dim() != 3 or attn_sink.dim() != 1:
        raise RuntimeError("dsa: expected q_sa [b,s,h,d], kv [b,n,d], attn_sink [h]")
    if q_sa.shape[0] != B or q_sa.shape[1] != S:
        raise RuntimeError("dsa: q_sa must have the indexer's [b, s] rows")
    H_sa, D_sa = q_sa.shape[2], q_sa.shape[3]
    if kv.shape[0] != B or kv.shape[2] != D_sa or attn_sink.shape[0] != H_sa:
        raise RuntimeError("dsa: kv / attn_sink shape mismatch")
    _require_cuda("dsa", q_ix, q_sa, kv, attn_sink)
    if int(T) < 1:
        raise RuntimeError("dsa: T must be >= 1")
    dv = D_sa if dv is None else int(dv)
    if dv > _DV_MAX:
        raise RuntimeError(f"dsa: dv={dv} > {_DV_MAX} (use indexer_topk + sparse_attn)")
    kk = min(int(topk), int(T))
    if idx_out is None:
        idx_out = torch.empty((B, S, kk), dtype=torch.int32, device=q_ix.device)
    else:
        _check_out("dsa", idx_out, (B, S, kk), torch.int32, q_ix.device)
    if out is None:
        out = torch.empty((B, S, H_sa, dv), dtype=torch.bfloat16, device=q_ix.device)
    else:
        _check_out("dsa", out, (B, S, H_sa, dv), torch.bfloat16, q_ix.device)
    need = indexer_workspace_size(B, S, T)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q_ix.device)
    else:
        _check_workspace("dsa", workspace, need, q_ix.device)
    with torch.cuda.device(q_ix.device):
        check(lib().ks_dsa(_ptr(q_ix), _ptr(k_ix), k_ix.shape[1], _ptr(w), _ptr(freqs), B, S, H, D,
                           int(T), int(rope_dim), int(pos0), int(bool(causal)), int(ratio),
                           int(topk), int(offset), _ptr(q_sa), _ptr(kv), kv.shape[1],
                           _ptr(attn_sink), H_sa, D_sa, dv, float(softmax_scale), _ptr(idx_out),
                           _ptr(out), _ptr(workspace), workspace.numel() * workspace.element_size(),
                           _stream(q_ix)), "ks_dsa")
    return out, idx_out


def proj_rope(a: torch.Tensor, w: torch.Tensor, head_dim: int = 0, rope_dim: int = 0,
              freqs: torch.Tensor | None = None, scale: float | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear(a, w)`` (bf16, fp32 accumulation) on the tensor cores with the
    indexer's follow-up arithmetic fused into the epilogue: with ``rope_dim`` the
    last ``rope_dim`` of every ``head_dim`` output columns are rotated by
    ``freqs[s]`` ([S, rope_dim/2, 2] fp32, row s of the sequence dim, i.e. dim -2
    of ``a``), as baseline/indexer.py:114-129,172; with ``scale`` the bf16
    result is multiplied by it and rounded again (baseline/indexer.py:173-175).
    a bf16 [..., K], w bf16 [N, K] -> bf16 [..., N]."""
    if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise RuntimeError("proj_rope: a and w must be bfloat16")
    if a.dim() < 1 or w.dim() != 2 or a.shape[-1] != w.shape[1]:
        raise RuntimeError("proj_rope: expected a [..., K] and w [N, K]")
    if freqs is not None and freqs.dtype != torch.float32:
        raise RuntimeError("proj_rope: freqs must be float32 [S, rope_dim/2, 2]")
    if rope_dim and freqs is None:
        raise RuntimeError("proj_rope: rope_dim needs freqs")
    ts = [a, w] + ([freqs] if freqs is not None else [])
    _require_cuda("proj_rope", *ts)
    N, K = w.shape
    M = a.numel() // K
    S = a.shape[-2] if a.dim() >= 2 else 1
    if rope_dim and freqs.shape[0] < S:
        raise RuntimeError("proj_rope: freqs has fewer rows than the sequence")
    shape = tuple(a.shape[:-1]) + (N,)
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=a.device)
    else:
        _check_out("proj_rope", out, shape, torch.bfloat16, a.device)
    with torch.cuda.device(a.device):
        check(lib().ks_proj_rope(_ptr(a), _ptr(w), _ptr(out), M, N, K, int(head_dim),
                                 int(rope_dim), _ptr(freqs), S,
                                 float(scale) if scale is not None else 1.0,
                                 int(scale is not None), _stream(a)), "ks_proj_rope")
    return out


_FP8 = (torch.float8_e4m3fn, torch.uint8)


def quant_fp8_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """e4m3 quantisation of bf16 rows [..., D] with one power-of-two ("ue8m0")
    scale per row: returns (x8 float8_e4m3fn [..., D], scale fp32 [...]), with
    x ~= x8 * scale.  The input side of ``indexer_topk_fp8``."""
    if x.dtype != torch.bfloat16 or x.dim() < 1:
        raise RuntimeError("quant_fp8_rows: x must be bfloat16 [..., D]")
    _require_cuda("quant_fp8_rows", x)
    D = x.shape[-1]
    x8 = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    scale = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        check(lib().ks_quant_fp8_rows(_ptr(x), _ptr(x8), _ptr(scale), x.numel() // max(D, 1), D,
                                      _stream(x)), "ks_quant_fp8_rows")
    return x8, scale


def _indexer_fp8_args(q8, k8, w, k_scale, T):
    if q8.dtype not in _FP8 or k8.dtype not in _FP8:
        raise RuntimeError("indexer_fp8: q8 and k8 must be float8_e4m3fn (or their uint8 bytes)")
    if w.dtype != torch.float32 or k_scale.dtype != torch.float32:
        raise RuntimeError("indexer_fp8: w and k_scale must be float32")
    if q8.dim() != 4 or k8.dim() != 3 or w.dim() != 3 or k_scale.dim() != 2:
        raise RuntimeError("indexer_fp8: expected q8 [b,s,h,d], k8 [b,t,d], w [b,s,h], k_scale [b,t]")
    B, S, H, D = q8.shape
    if k8.shape[0] < B or k8.shape[2] != D or k8.shape[1] < T:
        raise RuntimeError("indexer_fp8: k8 shape mismatch")
    if tuple(w.shape) != (B, S, H) or tuple(k_scale.shape) != tuple(k8.shape[:2]):
        raise RuntimeError("indexer_fp8: w / k_scale shape mismatch")
    _require_cuda("indexer_fp8", q8, k8[:B], w, k_scale)
    return B, S, H, D


def indexer_topk_fp8(q8: torch.Tensor, k8: torch.Tensor, w: torch.Tensor, k_scale: torch.Tensor,
                     T: int, topk: int, ratio: int = 1, causal: bool = True, offset: int = 0,
                     pos0: int = 0, out_dtype: torch.dtype = torch.int64,
                     out: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None) -> torch.Tensor:
    """FP8 indexer top-k (ModelArgs.dtype = "fp8", baseline/indexer.py:14-17):
    e4m3 queries q8 [B,S,H,128] (rotated, then quantised per (token, head)) and
    keys k8 [B,Tk>=T,128] with per-key scales k_scale [B,Tk]; w fp32 [B,S,H] =
    head weight x query scale.  Scores bf16(k_scale * sum_h relu(q8.k8) * w), then
    the mask, top-k and post-processing of ``indexer_topk``."""
    B, S, H, D = _indexer_fp8_args(q8, k8, w, k_scale, T)
    kk = min(int(topk), int(T))
    if out is None:
        out = torch.empty((B, S, kk), dtype=out_dtype, device=q8.device)
    elif out.dtype not in (torch.int32, torch.int64):
        raise RuntimeError("indexer_fp8: out must be int32 or int64")
    else:
        _check_out("indexer_fp8", out, (B, S, kk), out.dtype, q8.device)
    if T == 0:
        return out
    need = indexer_workspace_size(B, S, T)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q8.device)
    else:
        _check_workspace("indexer_fp8", workspace, need, q8.device)
    with torch.cuda.device(q8.device):
        check(lib().ks_indexer_fp8(_ptr(q8), _ptr(k8), k8.shape[1], _ptr(w), _ptr(k_scale), B, S,
                                   H, D, int(T), int(pos0), int(bool(causal)), int(ratio),
                                   int(topk), int(offset), _ptr(out),
                                   KS_INT64 if out.dtype == torch.int64 else KS_INT32,
                                   _ptr(workspace), workspace.numel() * workspace.element_size(),
                                   _stream(q8)), "ks_indexer_fp8")
    return out


def indexer_scores_fp8(q8: torch.Tensor, k8: torch.Tensor, w: torch.Tensor,
                       k_scale: torch.Tensor, T: int, ratio: int = 1, causal: bool = True,
                       pos0: int = 0) -> torch.Tensor:
    """Score stage of ``indexer_topk_fp8`` alone: bf16 [B, S, ld] laid out as
    ``indexer_scores``."""
    B, S, H, D = _indexer_fp8_args(q8, k8, w, k_scale, T)
    ld = (int(T) + 7) // 8 * 8
    scores = torch.full((B, S, ld), float("-inf"), dtype=torch.bfloat16, device=q8.device)
    with torch.cuda.device(q8.device):
        check(lib().ks_indexer_fp8_scores(_ptr(q8), _ptr(k8), k8.shape[1], _ptr(w), _ptr(k_scale),
                                          B, S, H, D, int(T), int(pos0), int(bool(causal)),
                                          int(ratio), _ptr(scores), ld, _stream(q8)),
              "ks_indexer_fp8_scores")
    return scores


def indexer_scores(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, freqs: torch.Tensor | None,
                   rope_dim: int, T: int, ratio: int = 1, causal: bool = True,
                   pos0: int = 0) -> torch.Tensor:
    """Score stage alone: bf16 [B, S, ld] (ld = T rounded up to 8); columns at or
    beyond a row's causal limit are -inf inside the last 128-key tile and
    unwritten after it."""
    B, S, H, D = _indexer_args(q, k, w, freqs, T)
    ld = (int(T) + 7) // 8 * 8
    scores = torch.full((B, S, ld), float("-inf"), dtype=torch.bfloat16, device=q.device)
    with torch.cuda.device(q.device):
        check(lib().ks_indexer_scores(_ptr(q), _ptr(k), k.shape[1], _ptr(w), _ptr(freqs), B, S,
                                      H, D, int(T), int(rope_dim), int(pos0), int(bool(causal)),
                                      int(ratio), _ptr(scores), ld, _stream(q)),
              "ks_indexer_scores")
    return scores


def topk_rows(scores: torch.Tensor, T: int, topk: int, ratio: int = 1, causal: bool = True,
              offset: int = 0, pos0: int = 0, out_dtype: torch.dtype = torch.int64
              ) -> torch.Tensor:
    """Top-k stage alone over bf16 scores [B, S, ld>=T] (ld % 8 == 0)."""
    if scores.dtype != torch.bfloat16 or scores.dim() != 3:
        raise RuntimeError("topk_rows: scores must be bf16 [b, s, ld]")
    _require_cuda("topk_rows", scores)
    B, S, ld = scores.shape
    kk = min(int(topk), int(T))
    out = torch.empty((B, S, kk), dtype=out_dtype, device=scores.device)
    with torch.cuda.device(scores.device):
        check(lib().ks_topk_rows(_ptr(scores), ld, B, S, int(T), int(pos0), int(bool(causal)),
                                 int(ratio), int(topk), int(offset), _ptr(out),
                                 KS_INT64 if out_dtype == torch.int64 else KS_INT32,
                                 _stream(scores)), "ks_topk_rows")
    return out


def device_status(device: torch.device | int | None = None) -> None:
    """Synchronise the current stream and raise if a kernel reported a timed-out
    wait or a bounds error since the last check."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    with torch.cuda.device(dev):
        check(lib().ks_device_status(torch.cuda.current_stream(dev).cuda_stream),
              "ks_device_status")
