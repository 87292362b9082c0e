"""Pin the CPU oracle (oracle/sol_oracle.py) against the reference's own oracle outputs.

The golden fixtures were produced by ``sol_attn_amd.reference.sol_reference``
(``src/sol_attn_amd/reference.py:19-66``) with tests/golden/make_golden.py on seeded inputs;
here the inputs are regenerated from the same seeds (checked by SHA-256) and the oracle must
reproduce the reference's outputs to FP32 summation-order tolerance and its exact-block
counts exactly.
"""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F



from helpers import digest, golden  # noqa: E402
from make_golden import bthd_cases, indexed_cases  # noqa: E402
from oracle.sol_oracle import dense_oracle, sol_oracle  # noqa: E402
from sol_attn_b200 import workloads  # noqa: E402

CASES = {name: (make, kw, every) for name, make, kw, every in bthd_cases()}


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name):
    make, kw, every = CASES[name]
    ref = golden(name)
    q, k, v = make()
    assert digest(q, k, v) == str(ref["sha256"]), "input generator drifted from the fixture"
    out, counts = sol_oracle(q, k, v, **kw)
    np.testing.assert_array_equal(counts.numpy(), ref["counts"])
    got = out.numpy() if every is None else out[:, ref["rows"]].numpy()
    want = ref["out"] if every is None else ref["out_rows"]
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=2e-6)


def test_oracle_query_subset_matches_reference():
    make, kw, _ = CASES["beta0_subsetq"]
    ref = golden("beta0_subsetq")
    q, k, v = make()
    part, counts = sol_oracle(q, k, v, query_blocks=[0, 2], **kw)
    np.testing.assert_array_equal(counts.numpy(), ref["subset_counts"])
    np.testing.assert_allclose(part.numpy(), ref["subset_out"], rtol=1e-4, atol=2e-6)
    assert torch.isnan(part[:, 64:128]).all()


@pytest.mark.parametrize("tag", ["minf", "pinf", "b1"])
def test_indexed_oracle_matches_reference(tag):
    from oracle.sol_oracle import indexed_oracle
    ref = golden(f"indexed_{tag}")
    cpu, rows, keys = indexed_cases()
    assert digest(*cpu) == str(ref["sha256"])
    beta = {"minf": -math.inf, "pinf": math.inf, "b1": 1.0}[tag]
    out, counts = indexed_oracle(*cpu, rows, keys, torch.from_numpy(ref["protected"]), beta=beta)
    np.testing.assert_array_equal(counts.numpy(), ref["counts"])
    np.testing.assert_allclose(out.numpy(), ref["out"], rtol=1e-4, atol=2e-6)


@pytest.mark.parametrize("d", [64, 128])
def test_oracle_dense_limit(d):
    """``tests/test_attention.py:27-34``: beta=-inf equals dense attention, every block exact."""
    q, k, v = workloads.reference_fixture(d=d)
    out, counts = sol_oracle(q, k, v, beta=-math.inf)
    expected = F.scaled_dot_product_attention(q.float().transpose(1, 2), k.float().transpose(1, 2),
                                              v.float().transpose(1, 2)).transpose(1, 2)
    torch.testing.assert_close(out, expected, atol=1e-6, rtol=2e-5)
    torch.testing.assert_close(dense_oracle(q, k, v), expected, atol=1e-6, rtol=2e-5)
    assert (counts == 5).all()


def test_oracle_constant_keys_correction():
    """``tests/test_attention.py:37-43``."""
    q, k, v = workloads.reference_fixture()
    k[:] = k[:, :1].clone()
    sparse, _ = sol_oracle(q, k, v, beta=math.inf)
    dense, _ = sol_oracle(q, k, v, beta=-math.inf)
    torch.testing.assert_close(sparse, dense, atol=0.001, rtol=0.04)


def test_oracle_prefix_protection_rounds_outward():
    """``tests/test_attention.py:46-52``."""
    q, k, v = workloads.reference_fixture()
    _, counts = sol_oracle(q, k, v, beta=math.inf, kv_sink_tokens=65, query_sink_tokens=1,
                           local_blocks=0)
    assert (counts[:, 0] == 5).all()
    assert (counts[:, 1] == 2).all()
    assert (counts[:, 2:] == 3).all()
