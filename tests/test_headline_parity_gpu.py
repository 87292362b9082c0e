"""Parity at the measured configurations themselves: the video-DiT self-attention workload
(B=1, T=32768, H=24, D=128, beta in {0, 0.5, 1}, sinks 128/128, local 1) and the indexed-window
workload (64 windows of 512 queries, six key counts from 5440 to 6560, one ragged plan).

The reference pins every shape it ships against its oracle with exact counts
(``tests/test_attention.py:55-69``, ``tests/test_indexed.py:62-88``).  Here, on heads spread
over the 24 (the query-sink q-blocks included) and on one window of each key count:

* outputs against the CPU oracle on every q-block, under the reference's ``assert_close`` and
  the north-star gate (max-abs 2e-2, mean-rel 5e-3);
* pooling, moments, cutoffs and routing bitmasks of the full 512 x 512-block heads bit-identical
  to their CPU restatement given the GPU's pooled statistics (the north-star routing criterion);
* exact-block counts against the oracle's: the number of disagreements is reported, and every
  routing decision that differs lies within FP32 rounding of the cutoff.
"""


import numpy as np
import pytest
import torch

from helpers import CAbi, assert_close, assert_north_star, to_device
from oracle import kernel_order
from oracle.sol_oracle import indexed_oracle, sol_oracle
from sol_attn_b200 import IndexedPlan, sol_attention, sol_attention_indexed, workloads

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
T, H, D = 32768, 24, 128
HEADS = (0, 11, 23)
KW = dict(kv_sink_tokens=128, query_sink_tokens=128, local_blocks=1)
# A routing decision may differ from the oracle's only where |proxy - cut| is within rounding of
# the FP32 dot products: bounded relative to the magnitude sum(|qbar_d| |kbar_d|) * scale.
NEAR = 1e-4


@pytest.fixture(scope="module")
def video_dit():
    cpu = workloads.video_dit(b=1, t=T, h=H, d=D, sigma=0.3, seed=0)
    return cpu, tuple(x.cuda() for x in cpu)


def near_cut_ok(internals, sel_gpu, scale):
    """Disagreements between the GPU's selection [B, nqb, H, nkb] and the oracle's, and whether
    each lies within NEAR of its cutoff (float64 proxy from the oracle's pooled statistics)."""
    sel_ref = internals["selection"].numpy()
    diff = np.argwhere(sel_gpu != sel_ref)
    qm = internals["qm"].double().numpy()      # [B, nqb, H, D]
    km = internals["km"].double().numpy()      # [B, nkb, H, D]
    cut = internals["cut"].double().numpy()    # [B, nqb, H]
    worst = 0.0
    for b, qb, h, kb in diff:
        proxy = float(qm[b, qb, h] @ km[b, kb, h]) * scale
        mag = float(np.abs(qm[b, qb, h]) @ np.abs(km[b, kb, h])) * scale + abs(cut[b, qb, h])
        worst = max(worst, abs(proxy - cut[b, qb, h]) / mag)
    return len(diff), worst


@pytest.mark.parametrize("beta", [1.0, 0.5, 0.0])
def test_video_dit_outputs_and_counts_against_oracle(video_dit, beta):
    (qh, kh, vh), (q, k, v) = video_dit
    out, stats = sol_attention(q, k, v, beta=beta, return_stats=True, **KW)
    counts = stats.exact_blocks.cpu()
    scale = D ** -0.5
    total_diff, worst = 0, 0.0
    for h in HEADS:
        q1, k1, v1 = (x[:, :, h:h + 1].contiguous() for x in (qh, kh, vh))
        ref, ref_counts, internals = sol_oracle(q1, k1, v1, beta=beta, return_internals=True, **KW)
        got = out[:, :, h:h + 1].cpu()
        assert_close(got, ref)
        assert_north_star(got, ref)
        # the GPU's routing of this head (its own bitmask) against the oracle's selection
        gpu_counts = counts[:, :, h:h + 1]
        r = CAbi().stages(q[:, :, h:h + 1], k[:, :, h:h + 1], v[:, :, h:h + 1], beta=beta,
                          local=1, kv_sink_blocks=2, q_sink_blocks=2)
        mask = r["mask"].cpu().numpy().view(np.uint32)                     # [1, 1, nqb, nw]
        bits = np.unpackbits(mask.view(np.uint8), bitorder="little").reshape(1, 1, 512, -1)
        sel_gpu = bits[..., :512].astype(bool).transpose(0, 2, 1, 3)       # [1, nqb, 1, nkb]
        assert torch.equal(torch.from_numpy(sel_gpu.sum(-1).astype(np.int32)), gpu_counts)
        n, w = near_cut_ok(internals, sel_gpu, scale)
        # per-q-block counts equal the oracle's except where a decision differs
        assert int((gpu_counts - ref_counts).abs().sum()) <= n, (h, beta)
        total_diff += n
        worst = max(worst, w)
    print(f"beta {beta}: {total_diff} of {len(HEADS) * 512 * 512} routing decisions differ from "
          f"the oracle's, worst |proxy - cut| / magnitude {worst:.2e}")
    assert worst <= NEAR, (beta, total_diff, worst)
    assert total_diff <= len(HEADS) * 512 * 512 // 10000, (beta, total_diff)


@pytest.mark.parametrize("beta", [1.0, 0.0])
def test_video_dit_routing_bit_identical_on_full_heads(video_dit, beta):
    """North-star criterion 1 on whole 512 x 512-block heads: pooled statistics, moments,
    cutoffs and the routing bitmask equal the CPU restatement bit for bit."""
    (qh, kh, vh), _ = video_dit
    idx = list(HEADS)
    qs, ks, vs = (x[:, :, idx].contiguous() for x in (qh, kh, vh))
    r = CAbi().stages(*(to_device(x) for x in (qs, ks, vs)), beta=beta, local=1,
                      kv_sink_blocks=2, q_sink_blocks=2)
    np.testing.assert_array_equal(r["qc"].cpu().numpy(), kernel_order.pool(qs, False))
    np.testing.assert_array_equal(r["kc"].float().cpu().numpy(), kernel_order.pool(ks, True))
    np.testing.assert_array_equal(r["vc"].float().cpu().numpy(), kernel_order.pool(vs, True))
    qc, kc = r["qc"].cpu().numpy(), r["kc"].float().cpu().numpy()
    mean, var = kernel_order.moments(kc)
    np.testing.assert_array_equal(r["mean"].cpu().numpy(), mean)
    np.testing.assert_array_equal(r["var"].cpu().numpy(), var)
    cut = kernel_order.cutoffs(qc, mean, var, beta, r["scale"])
    np.testing.assert_array_equal(r["cut"].cpu().numpy(), cut)
    sel = kernel_order.route(qc, kc, r["cut"].cpu().numpy(), r["scale"], 0, 1, 2, 2)
    np.testing.assert_array_equal(r["mask"].cpu().numpy().view(np.uint32),
                                  kernel_order.pack_mask(sel))
    np.testing.assert_array_equal(r["counts"].cpu().numpy(), sel.sum(-1).transpose(0, 2, 1))


def test_indexed_windows_one_per_key_count_against_oracle(video_dit):
    """The indexed-window workload in one ragged plan: the first window of each of the six key
    counts against the oracle on that window (all 24 heads), counts included."""
    (qh, kh, vh), (q, k, v) = video_dit
    qn, kn, vn = (x[0] for x in (qh, kh, vh))
    wins = workloads.indexed_windows(T, window=512, halo=1024, anchor=256, stride=8)
    rows = torch.stack([r for r, _ in wins])
    keys = [kk for _, kk in wins]
    plan = IndexedPlan.create(rows, keys, T, protected_ranges=((0, 256),))
    out, stats = sol_attention_indexed(q[0], k[0], v[0], plan.to("cuda"), beta=1.0,
                                       return_stats=True)
    counts = stats.exact_blocks.cpu()
    firsts = {}
    for w, kk in enumerate(keys):
        firsts.setdefault(kk.numel(), w)
    assert sorted(firsts) == [5440, 5664, 5888, 6112, 6336, 6560]
    scale = D ** -0.5
    for nk, w in sorted(firsts.items()):
        own = IndexedPlan.create(rows[w:w + 1], keys[w][None], T, protected_ranges=((0, 256),))
        ref, ref_counts, internals = indexed_oracle(qn, kn, vn, own.rows, own.keys,
                                                    own.protected_blocks, beta=1.0,
                                                    return_internals=True)
        got = out[w:w + 1].cpu()
        assert_close(got, ref)
        assert_north_star(got, ref)
        nkb = (nk + 63) // 64
        got_counts = counts[w:w + 1]
        # the GPU's decisions for this window from its own plan (equal to the ragged plan's)
        r = CAbi().stages(q[0], k[0], v[0], beta=1.0, local=-1,
                          protect=own.protected_blocks.cuda(), rows=own.rows.cuda(),
                          keys=own.keys.cuda())
        mask = r["mask"].cpu().numpy().view(np.uint32)
        bits = np.unpackbits(mask.view(np.uint8), bitorder="little")
        sel_gpu = bits.reshape(1, H, 8, -1)[..., :nkb].astype(bool).transpose(0, 2, 1, 3)
        assert torch.equal(torch.from_numpy(sel_gpu.sum(-1).astype(np.int32)), got_counts)
        n, worst = near_cut_ok(internals, sel_gpu, scale)
        print(f"window {w} ({nk} keys): {n} routing decisions differ from the oracle's, "
              f"worst |proxy - cut| / magnitude {worst:.2e}")
        assert worst <= NEAR, (nk, n, worst)
        assert int((got_counts - ref_counts).abs().sum()) <= n, nk
