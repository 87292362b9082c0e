"""GPU parity of sol_attention / dense_attention against the reference's golden outputs and
the CPU oracle (reference tests: ``tests/test_attention.py:55-146``)."""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import CAbi, assert_close, assert_north_star, golden, to_device
from make_golden import bthd_cases
from oracle import kernel_order
from oracle.sol_oracle import sol_oracle
from sol_attn_b200 import dense_attention, sol_attention, workloads

pytestmark = pytest.mark.gpu
CASES = {name: (make, kw, every) for name, make, kw, every in bthd_cases()}
SMALL = sorted(n for n, (_, _, every) in CASES.items() if every is None and n != "beta0_subsetq")


@pytest.mark.parametrize("name", SMALL)
def test_sol_matches_reference_golden(name):
    make, kw, _ = CASES[name]
    ref = golden(name)
    q, k, v = (to_device(x) for x in make())
    actual, stats = sol_attention(q, k, v, return_stats=True, **kw)
    assert actual.is_contiguous() and actual.dtype == torch.bfloat16
    assert_close(actual.cpu(), torch.from_numpy(ref["out"]))
    assert_north_star(actual.cpu(), torch.from_numpy(ref["out"]))
    np.testing.assert_array_equal(stats.exact_blocks.cpu().numpy(), ref["counts"])
    repeated = sol_attention(q, k, v, **kw)
    assert torch.equal(actual, repeated)


@pytest.mark.parametrize("name", ["c2_block_smooth_b1", "c2_block_smooth_minf",
                                  "c2_block_smooth_pinf", "c4_ragged_cross"])
def test_sol_matches_reference_golden_configs(name):
    make, kw, _ = CASES[name]
    ref = golden(name)
    q, k, v = (to_device(x) for x in make())
    actual, stats = sol_attention(q, k, v, return_stats=True, **kw)
    rows = torch.from_numpy(ref["rows"])
    assert_close(actual[:, rows.cuda()].cpu(), torch.from_numpy(ref["out_rows"]))
    assert_north_star(actual[:, rows.cuda()].cpu(), torch.from_numpy(ref["out_rows"]))
    np.testing.assert_array_equal(stats.exact_blocks.cpu().numpy(), ref["counts"])


@pytest.mark.parametrize("case", ["ragged_d64_strided_b1", "ragged_d128_dense_b1", "groups_tail_b1",
                                  "c1_plumbing", "c2_beta0", "c2_beta05", "c4_ragged_cross"])
def test_routing_bit_identical_given_pooled_statistics(case):
    """Pool / threshold / routing of the kernels equal their CPU restatement bit for bit."""
    if case == "c2_beta0":
        make, kw = CASES["c2_block_smooth_b1"][0], dict(beta=0.0, kv_sink_tokens=128,
                                                       query_sink_tokens=128, local_blocks=1)
    elif case == "c2_beta05":
        make, kw = CASES["c2_block_smooth_b1"][0], dict(beta=0.5, kv_sink_tokens=128,
                                                       query_sink_tokens=128, local_blocks=1)
    else:
        make, kw, _ = CASES[case]
    qh, kh, vh = make()
    q, k, v = (to_device(x) for x in (qh, kh, vh))
    beta = kw.get("beta", 1.0)
    kvs = (kw.get("kv_sink_tokens", 0) + 63) // 64
    qs = (kw.get("query_sink_tokens", 0) + 63) // 64
    local = kw.get("local_blocks", 1)
    r = CAbi().stages(q, k, v, beta=beta, local=local, kv_sink_blocks=kvs, q_sink_blocks=qs)
    # (1) pooling, bit for bit
    np.testing.assert_array_equal(r["qc"].cpu().numpy(), kernel_order.pool(qh, False))
    np.testing.assert_array_equal(r["kc"].float().cpu().numpy(), kernel_order.pool(kh, True))
    np.testing.assert_array_equal(r["vc"].float().cpu().numpy(), kernel_order.pool(vh, True))
    qc, kc = r["qc"].cpu().numpy(), r["kc"].float().cpu().numpy()
    # (2) moments and cutoffs from the GPU's pooled statistics
    mean, var = kernel_order.moments(kc)
    np.testing.assert_array_equal(r["mean"].cpu().numpy(), mean)
    np.testing.assert_array_equal(r["var"].cpu().numpy(), var)
    cut = kernel_order.cutoffs(qc, mean, var, beta, r["scale"])
    np.testing.assert_array_equal(r["cut"].cpu().numpy(), cut)
    # (3) routing decisions from the GPU's pooled statistics, bit for bit
    sel = kernel_order.route(qc, kc, r["cut"].cpu().numpy(), r["scale"], r["force"], local, kvs, qs)
    np.testing.assert_array_equal(r["mask"].cpu().numpy().view(np.uint32), kernel_order.pack_mask(sel))
    np.testing.assert_array_equal(r["counts"].cpu().numpy(), sel.sum(-1).transpose(0, 2, 1))
    # (4) and against the reference-style oracle: output within the north-star gate
    ref, counts, internals = sol_oracle(qh, kh, vh, return_internals=True, **kw)
    assert_north_star(r["out"].cpu(), ref)
    disagree = (torch.from_numpy(sel.transpose(0, 2, 1, 3)) != internals["selection"]).sum()
    assert int(disagree) <= max(2, sel.size // 1000), int(disagree)


@pytest.mark.parametrize("nq,nk", [(1, 1), (63, 65), (64, 64), (65, 63), (1025, 1089)])
def test_dense_tail(nq, nk):
    q, k, v = (to_device(x) for x in workloads.reference_fixture(nq=nq, nk=nk, d=128))
    actual = dense_attention(q, k, v)
    expected = F.scaled_dot_product_attention(q.float().transpose(1, 2), k.float().transpose(1, 2),
                                              v.float().transpose(1, 2)).transpose(1, 2)
    assert_close(actual, expected)


def test_sol_zero_inputs_and_exact_sinks():
    q, k, v = (to_device(x) for x in workloads.reference_fixture())
    q.zero_(); k.zero_()
    actual, stats = sol_attention(q, k, v, beta=math.inf, local_blocks=0, kv_sink_tokens=65,
                                  query_sink_tokens=1, return_stats=True)
    ref, counts = sol_oracle(q.cpu(), k.cpu(), v.cpu(), beta=math.inf, local_blocks=0,
                             kv_sink_tokens=65, query_sink_tokens=1)
    assert_close(actual.cpu(), ref)
    torch.testing.assert_close(stats.exact_blocks.cpu(), counts, atol=0, rtol=0)


def test_sol_single_token_no_empty_mass_nan():
    q, k, v = (to_device(x) for x in workloads.reference_fixture(nq=1, nk=1))
    for beta in (-math.inf, math.inf, 1.0):
        assert torch.equal(sol_attention(q, k, v, beta=beta), v)


def test_sol_rows_with_no_exact_blocks():
    q, k, v = (to_device(x) for x in workloads.reference_fixture(nq=321, nk=65, h=1))
    actual, stats = sol_attention(q, k, v, beta=math.inf, local_blocks=0, return_stats=True)
    ref, counts = sol_oracle(q.cpu(), k.cpu(), v.cpu(), beta=math.inf, local_blocks=0)
    assert (stats.exact_blocks[:, 2:] == 0).all()
    assert_close(actual.cpu(), ref)
    torch.testing.assert_close(stats.exact_blocks.cpu(), counts, atol=0, rtol=0)


def test_sol_preserves_inputs_and_rejects_masks():
    q, k, v = (to_device(x) for x in workloads.reference_fixture())
    copies = tuple(x.clone() for x in (q, k, v))
    sol_attention(q, k, v)
    for x, copy in zip((q, k, v), copies):
        assert torch.equal(x, copy)
    with pytest.raises(TypeError):
        sol_attention(q, k, v, attn_mask=torch.ones((193, 317), device="cuda"))


def test_sol_rejects_invalid_controls():
    q, k, v = (to_device(x) for x in workloads.reference_fixture())
    for controls in ({"beta": math.nan}, {"local_blocks": -1}, {"kv_sink_tokens": 318},
                     {"query_sink_tokens": 194}, {"scale": 0}, {"scale": math.inf}):
        with pytest.raises(ValueError):
            sol_attention(q, k, v, **controls)


def test_unaligned_strides_are_handled():
    """Positive strides that are not 16-byte multiples go through a contiguous copy."""
    g = torch.Generator().manual_seed(5)
    base = torch.randn((1, 200, 2 * 64 + 8), generator=g, dtype=torch.bfloat16)
    kv = torch.randn((1, 200, 2, 64), generator=g, dtype=torch.bfloat16)
    q = base[:, :, 1:129].unflatten(-1, (2, 64))       # row starts 2 bytes off 16-byte alignment
    gq = to_device(base)[:, :, 1:129].unflatten(-1, (2, 64))
    out = sol_attention(gq, to_device(kv), to_device(kv))
    ref, _ = sol_oracle(q, kv, kv)
    assert_close(out.cpu(), ref)


def test_sol_matches_oracle_on_random_shapes():
    g = torch.Generator().manual_seed(11)
    for nq, nk, h, d, beta in [(300, 700, 3, 64, 0.3), (129, 2000, 2, 128, 1.5), (2048, 64, 1, 128, -0.5)]:
        q = torch.randn((1, nq, h, d), generator=g, dtype=torch.bfloat16)
        k = torch.randn((1, nk, h, d), generator=g, dtype=torch.bfloat16)
        v = torch.randn((1, nk, h, d), generator=g, dtype=torch.bfloat16)
        sink = min(100, nk)
        actual, stats = sol_attention(*(to_device(x) for x in (q, k, v)), beta=beta,
                                      kv_sink_tokens=sink, return_stats=True)
        ref, counts = sol_oracle(q, k, v, beta=beta, kv_sink_tokens=sink)
        assert_close(actual.cpu(), ref)
        assert_north_star(actual.cpu(), ref)
        assert (stats.exact_blocks.cpu() - counts).abs().sum() <= 2


def test_claim_modes_give_identical_results():
    """The fused kernel claims work items early (item after next, at 16 or more items per CTA)
    or late (while the current item's last tiles load).  Results do not depend on which CTA ran
    an item: a 40-head call (2560 items, early) and a 4-head call on the same tensors (256
    items, late) must agree bit for bit on those heads, counts included."""
    q, k, v = (to_device(x) for x in workloads.video_dit(t=8192, h=40, d=128, sigma=0.3, seed=3))
    kw = dict(beta=1.0, kv_sink_tokens=128, query_sink_tokens=128, local_blocks=1)
    full, full_stats = sol_attention(q, k, v, return_stats=True, **kw)
    part, part_stats = sol_attention(q[:, :, 4:8], k[:, :, 4:8], v[:, :, 4:8], return_stats=True, **kw)
    assert torch.equal(part, full[:, :, 4:8])
    assert torch.equal(part_stats.exact_blocks, full_stats.exact_blocks[:, :, 4:8])
