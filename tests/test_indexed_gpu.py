"""GPU parity of sol_attention_indexed (``tests/test_indexed.py:59-88``)."""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import CAbi, assert_north_star, golden, to_device
from make_golden import indexed_cases
from oracle import kernel_order
from sol_attn_b200 import IndexedPlan, sol_attention_indexed

pytestmark = pytest.mark.gpu
BETAS = {"minf": -math.inf, "pinf": math.inf, "b1": 1.0}


@pytest.mark.parametrize("tag", ["minf", "pinf", "b1"])
def test_indexed_mask_pooling_oracle_and_unchanged_inputs(tag):
    beta = BETAS[tag]
    ref = golden(f"indexed_{tag}")
    cpu, rows, keys = indexed_cases()
    p = IndexedPlan.create(rows, keys, 1200, protected_ranges=((0, 7), (1180, 1193)), local_tokens=64)
    gpu = [to_device(x) for x in cpu]
    assert gpu[0].stride() == cpu[0].stride()
    before = [x.clone() for x in gpu]
    actual, stats = sol_attention_indexed(*gpu, p.to("cuda"), beta=beta, return_stats=True)
    want = torch.from_numpy(ref["out"])
    torch.testing.assert_close(actual.cpu().float(), want, atol=0.012, rtol=0.025)
    assert (actual.cpu().float() - want).norm() / want.norm() < 0.008
    assert_north_star(actual.cpu(), want)
    np.testing.assert_array_equal(stats.exact_blocks.cpu().numpy(), ref["counts"])
    if beta == -math.inf:
        dense = F.scaled_dot_product_attention(cpu[0][rows].float().transpose(1, 2),
                                               cpu[1][keys].float().transpose(1, 2),
                                               cpu[2][keys].float().transpose(1, 2)).transpose(1, 2)
        torch.testing.assert_close(actual.cpu().float(), dense, atol=0.012, rtol=0.025)
    # Keys not in the declared mask must not affect exact OR approximate output.
    seen = torch.unique(keys)
    excluded = torch.ones(1200, dtype=torch.bool, device="cuda")
    excluded[seen.to("cuda")] = False
    gpu[1][excluded] = 80
    gpu[2][excluded] = 80
    assert torch.equal(actual, sol_attention_indexed(*gpu, p.to("cuda"), beta=beta))
    assert torch.equal(gpu[0], before[0])
    assert torch.equal(gpu[1][seen], before[1][seen])
    assert torch.equal(gpu[2][seen], before[2][seen])


def test_indexed_routing_and_pooling_bit_identical():
    cpu, rows, keys = indexed_cases()
    p = IndexedPlan.create(rows, keys, 1200, protected_ranges=((0, 7), (1180, 1193)), local_tokens=64)
    gpu = [to_device(x) for x in cpu]
    r = CAbi().stages(*gpu, beta=1.0, local=-1, protect=p.protected_blocks.cuda(),
                      rows=rows.cuda(), keys=keys.cuda())
    qg, kg, vg = cpu[0][rows], cpu[1][keys], cpu[2][keys]
    np.testing.assert_array_equal(r["qc"].cpu().numpy(), kernel_order.pool(qg, False))
    np.testing.assert_array_equal(r["kc"].float().cpu().numpy(), kernel_order.pool(kg, True))
    np.testing.assert_array_equal(r["vc"].float().cpu().numpy(), kernel_order.pool(vg, True))
    qc, kc = r["qc"].cpu().numpy(), r["kc"].float().cpu().numpy()
    sel = kernel_order.route(qc, kc, r["cut"].cpu().numpy(), r["scale"], 0, -1, 0, 0,
                             p.protected_blocks.numpy())
    np.testing.assert_array_equal(r["mask"].cpu().numpy().view(np.uint32), kernel_order.pack_mask(sel))


def test_indexed_scatter_writes_rows_in_place():
    """``out=`` writes each window's rows at their original positions (the VDN adapter's
    ``out[plan.rows] = result``, ``integrations/vdn.py:64-70``), bit-identical to the gathered
    result, and leaves every other row untouched."""
    cpu, rows, keys = indexed_cases()
    p = IndexedPlan.create(rows, keys, 1200, protected_ranges=((0, 7), (1180, 1193)), local_tokens=64)
    gpu = [to_device(x) for x in cpu]
    pd = p.to("cuda")
    want, stats = sol_attention_indexed(*gpu, pd, beta=1.0, return_stats=True)
    out = torch.full(gpu[0].shape, 7.0, dtype=torch.bfloat16, device="cuda")
    got, stats2 = sol_attention_indexed(*gpu, pd, beta=1.0, return_stats=True, out=out)
    assert got is out
    r = rows.to("cuda")
    assert torch.equal(out[r], want)
    untouched = torch.ones(1200, dtype=torch.bool, device="cuda")
    untouched[r.flatten()] = False
    assert bool((out[untouched] == 7.0).all())
    assert torch.equal(stats.exact_blocks, stats2.exact_blocks)


def test_dense_attention_rows_matches_sdpa_and_gathered_dense():
    """``dense_attention_rows`` (the adapter's dense step for global query rows) against FP32
    SDPA of the gathered rows over all keys, and bit-identical to ``dense_attention`` of the
    gathered rows; rows it does not name stay untouched."""
    from sol_attn_b200 import dense_attention, dense_attention_rows
    g = torch.Generator().manual_seed(5)
    N, H, D = 1000, 3, 128
    q, k, v = (torch.randn((N, H, D), generator=g, dtype=torch.bfloat16).cuda() for _ in range(3))
    rows = torch.cat((torch.arange(0, 40), torch.arange(517, 600, 3), torch.tensor([999]))).cuda()
    out = torch.full((N, H, D), -5.0, dtype=torch.bfloat16, device="cuda")
    assert dense_attention_rows(q, k, v, rows, out=out) is out
    ref = F.scaled_dot_product_attention(q[rows].float().transpose(0, 1)[None],
                                         k.float().transpose(0, 1)[None],
                                         v.float().transpose(0, 1)[None])[0].transpose(0, 1)
    torch.testing.assert_close(out[rows].float(), ref, atol=0.012, rtol=0.025)
    gathered = dense_attention(q[rows][None].contiguous(), k[None], v[None])[0]
    assert torch.equal(out[rows], gathered)
    untouched = torch.ones(N, dtype=torch.bool, device="cuda")
    untouched[rows] = False
    assert bool((out[untouched] == -5.0).all())
    fresh = dense_attention_rows(q, k, v, rows)
    assert torch.equal(fresh[rows], out[rows])


def test_ragged_plan_equals_separate_window_plans():
    """One launch over windows with different key counts gives, bit for bit, what one
    rectangular plan per window gives (outputs, exact-block counts), also with scatter."""
    from test_plan import ragged_fixture
    rows, keys = ragged_fixture()
    ranges = ((0, 7), (1180, 1193))
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn((1200, 2, 128), generator=g, dtype=torch.bfloat16).cuda()
               for _ in range(3))
    p = IndexedPlan.create(rows, keys, 1200, protected_ranges=ranges, local_tokens=64).to("cuda")
    for beta in (1.0, 0.0, -math.inf, math.inf):
        out, stats = sol_attention_indexed(q, k, v, p, beta=beta, return_stats=True)
        scat = torch.zeros_like(q)
        sol_attention_indexed(q, k, v, p, beta=beta, out=scat)
        for w, x in enumerate(keys):
            own = IndexedPlan.create(rows[w:w + 1], x[None], 1200, protected_ranges=ranges,
                                     local_tokens=64).to("cuda")
            o1, s1 = sol_attention_indexed(q, k, v, own, beta=beta, return_stats=True)
            assert torch.equal(out[w], o1[0]), (beta, w)
            assert torch.equal(stats.exact_blocks[w], s1.exact_blocks[0]), (beta, w)
            assert torch.equal(scat[rows[w].cuda()], o1[0]), (beta, w)
    d = stats.density()
    assert 0.0 < d <= 1.0


def test_window_sharded_plan_equals_full_plan_windows():
    """Window sharding across ranks (one process per GPU): the sub-plan of windows [2, 5) of a
    ragged plan gives, bit for bit, the outputs and exact-block counts of those windows in a
    call on the whole plan."""
    from sol_attn_b200 import workloads
    from sol_attn_b200.sharding import plan_windows
    t = 8192
    q, k, v = (to_device(x[0]) for x in workloads.video_dit(t=t, h=4, d=128, sigma=0.3, seed=7))
    wins = workloads.indexed_windows(t, window=512, halo=1024, anchor=256, stride=8)
    plan = IndexedPlan.create(torch.stack([r for r, _ in wins]), [kk for _, kk in wins], t,
                              protected_ranges=((0, 256),))
    full, full_stats = sol_attention_indexed(q, k, v, plan.to("cuda"), beta=1.0, return_stats=True)
    part, part_stats = sol_attention_indexed(q, k, v, plan_windows(plan, 2, 5).to("cuda"), beta=1.0,
                                             return_stats=True)
    assert torch.equal(part, full[2:5])
    assert torch.equal(part_stats.exact_blocks, full_stats.exact_blocks[2:5])
