"""The reference harness's compare procedure, restated for the tests — TEST
INFRASTRUCTURE ONLY.

The reference checks a v1 file against its v0 file with
benchmarks/ks/auto_bench.py: it loads each file through an AST filter, seeds and
builds both models, copies the v0 state into v1, moves models and inputs to the
accelerator, runs both forwards on clones of the same inputs and compares the
outputs (floats: allclose, anything else: torch.equal).  The reference checkout
does not travel to the GPU box, so this module restates those steps, and the v0
forwards of baseline/*.py in torch, so the same comparison runs on the B200:

* ``filter_load``      <- auto_bench.py:59-98,143-178 (the AST filter and loader)
* ``set_seed``         <- auto_bench.py:224-230
* ``harness_run``      <- auto_bench.py:358-409 (build order) and :513-539 (compare_case)
* ``compare``          <- auto_bench.py:270-312 (compare_values, for tensors)
* ``v0_class``         the reference Model of each op: constructor, parameter
  names and random draws come from the drop-in ``ModelNew`` (which keeps them
  identical to the reference's), forward from oracle/ks_ref_torch.py (the
  reference's baseline/sinkhorn.py:13-19, baseline/sparse_attention.py:5-42 and
  baseline/indexer.py:114-129,161-206 restated with the same torch operations).

``tests/test_harness_cpu.py`` pins the v0 restatements on the CPU against
fixtures that the reference's own modules produced (tests/golden/hx_*.npz).
"""
from __future__ import annotations

import ast
import os
import sys
import types

import torch

from oracle import ks_ref_torch as R

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "kernelswift_b200")


# ---------------------------------------------------------------- loading
def _safe_literal(node) -> bool:
    if isinstance(node, ast.Constant):
        return True
    if isinstance(node, (ast.Tuple, ast.List, ast.Set)):
        return all(_safe_literal(e) for e in node.elts)
    if isinstance(node, ast.Dict):
        return all((k is None or _safe_literal(k)) and _safe_literal(v)
                   for k, v in zip(node.keys, node.values))
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, (ast.UAdd, ast.USub)):
        return _safe_literal(node.operand)
    return False


def filter_load(path: str) -> types.ModuleType:
    """Load a v0/v1 file keeping only imports, defs, classes and literal
    assignments, as the harness does before executing it."""
    tree = ast.parse(open(path).read())
    keep = []
    for node in tree.body:
        if isinstance(node, (ast.Import, ast.ImportFrom, ast.ClassDef, ast.FunctionDef,
                             ast.AsyncFunctionDef)):
            keep.append(node)
        elif isinstance(node, ast.Assign) and _safe_literal(node.value):
            keep.append(node)
        elif isinstance(node, ast.AnnAssign) and node.value is not None and _safe_literal(node.value):
            keep.append(node)
    tree.body = keep
    ast.fix_missing_locations(tree)
    name = "ks_v1_" + os.path.basename(path)[:-3]
    mod = types.ModuleType(name)
    mod.__file__ = path
    mod.__package__ = ""
    # registered while it executes (dataclasses look their module up), then removed
    sys.modules[name] = mod
    try:
        exec(compile(tree, path, "exec"), mod.__dict__)
    finally:
        sys.modules.pop(name, None)
    return mod


def dropin(name: str) -> types.ModuleType:
    return filter_load(os.path.join(PKG, name + ".py"))


def set_seed(seed: int) -> None:
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def clone_value(v):
    if isinstance(v, torch.Tensor):
        return v.clone()
    if isinstance(v, (list, tuple)):
        return type(v)(clone_value(x) for x in v)
    return v


def to_device(v, device):
    if isinstance(v, torch.Tensor):
        return v.to(device)
    if isinstance(v, (list, tuple)):
        return type(v)(to_device(x, device) for x in v)
    return v


# ---------------------------------------------------------------- v0 forwards
# (the arithmetic lives in oracle/ks_ref_torch.py; these bind it to the modules)
def _sinkhorn_v0(self, x):
    return R.sinkhorn(x, self.repeat, self.eps)


def _sparse_attention_v0(self, q, kv, topk_idxs):
    return R.sparse_attn(q, kv, self.attn_sink, topk_idxs, self.softmax_scale)


def _indexer_v0(self, x, qr, start_pos, offset):
    """baseline/indexer.py:161-206.  Also keeps the masked bf16 scores in
    ``self.last_scores`` for classifying index differences."""
    S = x.size(1)
    q = self.wq_b(qr).unflatten(-1, (self.n_local_heads, self.head_dim))
    w = self.weights_proj(x) * (self.softmax_scale * self.n_heads ** -0.5)
    idx, self.last_scores = R.indexer_after_projections(
        q, w, self.kv_cache, self.freqs_cis[start_pos:start_pos + S], self.rope_head_dim,
        self.index_topk, self.compress_ratio, start_pos, offset)
    return idx


_V0_FORWARD = {"sinkhorn": _sinkhorn_v0, "sparse_attention": _sparse_attention_v0,
               "indexer": _indexer_v0}


def v0_class(name: str, mod: types.ModuleType):
    """The reference's Model for op `name`: the drop-in's constructor (identical
    parameters, buffers and random draws) with the reference forward."""
    return type("Model", (mod.ModelNew,), {"forward": _V0_FORWARD[name]})


# ---------------------------------------------------------------- the compare
def harness_run(name: str, device, seed: int = 42, v1: bool = True):
    """Build v0 (and v1) in the harness's order, move them and the inputs to
    `device`, run both forwards under no_grad on clones of v0's inputs.
    Returns (v0 model, v0 output, v1 model or None, v1 output or None, the inputs
    on `device`)."""
    mod = dropin(name)
    V0 = v0_class(name, mod)
    set_seed(seed)
    v0_init = mod.get_init_inputs()
    set_seed(seed)
    v1_init = mod.get_init_inputs()
    model = V0(*v0_init)
    model_new = mod.ModelNew(*v1_init) if v1 else None
    model.eval()
    if model_new is not None:
        model_new.eval()
        model_new.load_state_dict(model.state_dict())
    set_seed(seed)
    inputs = mod.get_inputs()
    model = model.to(device)
    inputs = to_device(inputs, device)
    set_seed(seed)
    with torch.no_grad():
        out0 = model(*clone_value(inputs))
    out1 = None
    if model_new is not None:
        model_new = model_new.to(device)
        set_seed(seed)
        with torch.no_grad():
            out1 = model_new(*clone_value(inputs))
    return model, out0, model_new, out1, inputs


def compare(v0: torch.Tensor, v1: torch.Tensor, atol: float = 1e-2, rtol: float = 1e-2):
    """compare_values for a tensor output: None when the harness would pass, else
    its reason."""
    if v0.shape != v1.shape:
        return f"shape {tuple(v0.shape)} vs {tuple(v1.shape)}"
    if v0.dtype.is_floating_point or v1.dtype.is_floating_point:
        if not torch.allclose(v0, v1.to(v0.device), atol=atol, rtol=rtol, equal_nan=True):
            d = (v0.float() - v1.float().to(v0.device)).abs()
            return f"values differ: max {d.max().item():.3e}, mean {d.mean().item():.3e}"
        return None
    if not torch.equal(v0, v1.to(v0.device)):
        return f"{(v0 != v1.to(v0.device)).sum().item()} elements differ"
    return None
