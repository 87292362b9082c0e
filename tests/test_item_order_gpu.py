"""The routing pass's per-head item order (``csrc/route.cu: order_head_items``), read back from
the mask buffer after real calls: for every head it is a permutation of the q-block pairs after
the sink pairs, sorted by tile count (most tiles first), stamped with the call's epoch, and the
head's arrival counter is left at zero for the next call.  The order only decides which CTA
runs an item when; the outputs must not change with it (a repeated call, whose epoch differs,
gives the same bits)."""

import numpy as np
import pytest
import torch

from sol_attn_b200 import workloads
from sol_attn_b200.stages import Stages

pytestmark = pytest.mark.gpu


def _layout(st):
    """Byte offsets of the mask buffer's sections (mirrors csrc/capi.cu: masks_bytes)."""
    bh = st.B * st.H
    npairs = (st.nqb + 1) // 2
    nw = (st.nkb + 31) // 32
    words = (bh * st.nqb * nw + 1 + 3) & ~3
    capacity = ((st.nkb + 63) // 64 + st.nkb + 1 + 7) & ~7
    stride = 16 + 2 * capacity
    lists = 4 * words
    sec = lists + bh * npairs * stride
    pad = (bh + 3) & ~3
    return bh, npairs, lists, stride, sec, pad


def _read(st):
    bh, npairs, lists, stride, sec, pad = _layout(st)
    raw = st._mask_words.view(torch.uint8).cpu().numpy()
    w = raw[sec:sec + 4 * (2 * pad + bh * npairs)].view(np.int32)
    arrive, stamp = w[:bh], w[pad:pad + bh].view(np.uint32)
    order = w[2 * pad:2 * pad + bh * npairs].reshape(bh, npairs)
    tiles = np.array([[raw[lists + (h * npairs + j) * stride:][:4].view(np.int32)[0]
                       for j in range(npairs)] for h in range(bh)])
    return arrive, stamp, order, tiles


# At least two items per CTA of the persistent grid (148 SMs): smaller launches skip the sort.
CASES = {
    "video_dit_t16k_h8": (lambda: workloads.video_dit(b=1, t=16384, h=8, d=128, seed=3),
                          dict(beta=1.0, local=1, kv_sink_blocks=2, q_sink_blocks=2)),
    "ragged_cross_b2": (lambda: workloads.ragged_cross(b=2, tq=8192, tk=5000, h=8, d=64, seed=4),
                        dict(beta=0.5, local=1, kv_sink_blocks=1, q_sink_blocks=3)),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_head_order_is_sorted_permutation(name):
    make, kw = CASES[name]
    q, k, v = (x.cuda() for x in make())
    st = Stages(q, k, v, **kw)
    first = st.run().clone()
    arrive, stamp1, order, tiles = _read(st)
    npairs = (st.nqb + 1) // 2
    sink = min(npairs, (st.qs + 1) // 2)
    assert not arrive.any(), "arrival counters must be left at zero"
    assert (stamp1 != 0).all() and len(set(stamp1.tolist())) == 1
    for h in range(st.B * st.H):
        got = order[h, :npairs - sink]
        assert sorted(got.tolist()) == list(range(sink, npairs))
        counts = tiles[h, got]
        assert (np.diff(counts) <= 0).all(), (h, counts)
    second = st.run()
    arrive2, stamp2, order2, _ = _read(st)
    assert not arrive2.any()
    assert (stamp2 != stamp1).all()  # a fresh epoch per call
    assert torch.equal(first, second)


def test_small_launches_keep_the_natural_order():
    """Fewer than two items per CTA (4 heads x 64 q-block pairs = 256 items): the routing pass
    skips the sort, the stamps of a zero-filled buffer stay zero, and the outputs are the same."""
    q, k, v = (x.cuda() for x in workloads.video_dit(b=1, t=8192, h=4, d=128, seed=3))
    st = Stages(q, k, v, beta=1.0, local=1, kv_sink_blocks=2, q_sink_blocks=2)
    first = st.run().clone()
    arrive, stamp, _, _ = _read(st)
    assert not arrive.any() and not stamp.any()
    assert torch.equal(first, st.run())
