"""Pin the harness restatement (tests/harness.py) on the CPU: built and run in the
reference harness's order at its default seed 42, each v0 model reproduces what
the reference's own baseline/*.py Model produced in that order
(tests/golden/hx_*.npz, written by tests/golden/make_golden.py).  This also pins
the drop-ins' get_init_inputs / get_inputs / constructors, whose random draws the
v0 models reuse."""
import numpy as np
import pytest
import torch

import harness as Hn
from conftest import load_golden

CPU = torch.device("cpu")


def test_sinkhorn_v0_matches_reference():
    _, out, _, _, _ = Hn.harness_run("sinkhorn", CPU, v1=False)
    np.testing.assert_allclose(out.numpy(), load_golden("hx_sinkhorn")["out"], rtol=1e-6, atol=1e-7)


def test_sparse_attention_v0_matches_reference():
    _, out, _, _, _ = Hn.harness_run("sparse_attention", CPU, v1=False)
    d = load_golden("hx_sparse_attention")
    rows = out[:, d["rows"]].contiguous().view(torch.int16).numpy().view(np.uint16)
    assert (rows == d["out_rows"]).mean() > 0.999
    np.testing.assert_allclose(out.double().sum(dim=(2, 3)).numpy(), d["row_sums"], rtol=1e-5, atol=1e-2)


def test_indexer_v0_matches_reference():
    _, out, _, _, _ = Hn.harness_run("indexer", CPU, v1=False)
    ref = load_golden("hx_indexer")["out"].astype(np.int64)
    assert out.dtype == torch.int64 and out.shape == ref.shape
    assert np.array_equal(out.numpy(), ref)


@pytest.mark.parametrize("name", ["sinkhorn", "sparse_attention", "indexer"])
def test_state_dict_copies_into_dropin(name):
    """The harness copies v0's state into v1 by name (auto_bench.py:518-521); a
    silent name mismatch would leave v1 with its own random weights."""
    mod = Hn.dropin(name)
    Hn.set_seed(42)
    init = mod.get_init_inputs()
    v0 = Hn.v0_class(name, mod)(*init)
    v1 = mod.ModelNew(*init)
    missing, unexpected = v1.load_state_dict(v0.state_dict(), strict=True)
    assert not missing and not unexpected
    for k, v in v0.state_dict().items():
        assert torch.equal(v1.state_dict()[k], v)
