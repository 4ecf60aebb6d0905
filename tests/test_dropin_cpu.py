"""The drop-in modules keep the reference's interface and survive the harness's
AST filter (benchmarks/ks/auto_bench.py:59-98 keeps only imports, defs, classes
and literal assignments).  CPU only: no kernel is called."""
import ast
import os
import types

import pytest
import torch

from conftest import ROOT

PKG = os.path.join(ROOT, "kernelswift_b200")


def _safe_literal(node):
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


def harness_load(path):
    """Load a v1 file the way the reference's harness does."""
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
    mod = types.ModuleType("v1")
    mod.__file__ = path
    exec(compile(tree, path, "exec"), mod.__dict__)
    return mod


@pytest.mark.parametrize("name,params", [
    ("sinkhorn", []),
    ("sparse_attention", ["attn_sink"]),
    ("indexer", ["wq_b.weight", "weights_proj.weight", "kv_cache", "freqs_cis"]),
])
def test_dropin_interface(name, params):
    mod = harness_load(os.path.join(PKG, name + ".py"))
    for attr in ("ModelNew", "get_inputs", "get_init_inputs"):
        assert callable(getattr(mod, attr)), attr
    torch.manual_seed(0)
    init = mod.get_init_inputs()
    m = mod.ModelNew(*init)
    assert sorted(m.state_dict().keys()) == sorted(params)


def test_sinkhorn_inputs_match_reference_shapes():
    mod = harness_load(os.path.join(PKG, "sinkhorn.py"))
    (x,) = mod.get_inputs()
    assert x.shape == (1, 1024, 4, 4) and x.dtype == torch.float32


def test_no_cpu_fallback():
    """The product path refuses CPU tensors instead of computing on the host."""
    mod = harness_load(os.path.join(PKG, "sinkhorn.py"))
    m = mod.ModelNew(*mod.get_init_inputs())
    with pytest.raises(RuntimeError):
        m(torch.randn(1, 8, 4, 4))
    sa = harness_load(os.path.join(PKG, "sparse_attention.py"))
    m = sa.ModelNew(16, 64)
    with pytest.raises(RuntimeError):
        m(torch.randn(1, 2, 16, 64).bfloat16(), torch.randn(1, 8, 64).bfloat16(),
          torch.zeros(1, 2, 4, dtype=torch.int32))


def test_indexer_init_inputs_match_reference_rng_order():
    """get_init_inputs draws the same random stream as the reference's: the
    kv_cache after seeding equals a direct re-draw with the same calls."""
    mod = harness_load(os.path.join(PKG, "indexer.py"))
    torch.manual_seed(42)
    args, freqs_cis, kv_cache, ratio = mod.get_init_inputs()
    torch.manual_seed(42)
    ref = torch.randn(args.max_batch_size, args.max_seq_len // 4, args.index_head_dim,
                      dtype=torch.bfloat16)
    assert torch.equal(kv_cache, ref) and ratio == 4
    assert freqs_cis.dtype == torch.complex64 and freqs_cis.shape == (2600, 16)
