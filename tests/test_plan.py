"""IndexedPlan: validation and protection parity (``src/sol_attn_amd/indexed.py:11-66``,
``tests/test_indexed.py:12-56``)."""

import random

import numpy as np
import pytest
import torch

from helpers import golden
from oracle.sol_oracle import protection_loops
from sol_attn_b200 import IndexedPlan, workloads


def fixture():
    rows = torch.stack((torch.arange(87, 152), torch.arange(300, 365)))
    keys = torch.stack((torch.cat((torch.arange(0, 23), torch.arange(70, 198), torch.arange(500, 509))),
                        torch.cat((torch.arange(0, 23), torch.arange(283, 411), torch.arange(500, 509)))))
    return IndexedPlan.create(rows, keys, 509, protected_ranges=((0, 23), (500, 509)), local_tokens=0)


def test_indexed_protection_uses_original_indices():
    p = fixture()
    assert p.protected_blocks.shape == (2, 2, 3)
    assert p.protected_blocks.all()
    rows = torch.tensor([[400]], dtype=torch.int64)
    keys = torch.arange(128).reshape(1, -1)
    p = IndexedPlan.create(rows, keys, 509, local_tokens=0)
    assert not p.protected_blocks.any()


@pytest.mark.parametrize("kind", ["unsorted", "duplicate", "negative", "outside", "dtype", "batch"])
def test_indexed_rejects_invalid_metadata(kind):
    rows = torch.tensor([[1, 2]], dtype=torch.int64)
    keys = torch.arange(8).reshape(1, -1)
    if kind == "unsorted": keys = keys.flip(1)
    if kind == "duplicate": keys[0, 1] = 0
    if kind == "negative": rows[0, 0] = -1
    if kind == "outside": keys[0, -1] = 20
    if kind == "dtype": keys = keys.int()
    if kind == "batch": rows = rows.repeat(2, 1)
    with pytest.raises(ValueError):
        IndexedPlan.create(rows, keys, 20)


@pytest.mark.parametrize("bad", [dict(protected_ranges=((5, 5),)), dict(protected_ranges=((0, 21),)),
                                 dict(local_tokens=-1), dict(local_tokens=True)])
def test_indexed_rejects_invalid_controls(bad):
    rows = torch.tensor([[1, 2]], dtype=torch.int64)
    keys = torch.arange(8).reshape(1, -1)
    with pytest.raises(ValueError):
        IndexedPlan.create(rows, keys, 20, **bad)


def test_protection_matches_reference_fixture():
    ref = golden("indexed_b1")
    rows = torch.stack((torch.arange(231, 361), torch.arange(901, 1031)))
    keys = torch.stack((torch.cat((torch.arange(7), torch.arange(191, 703), torch.arange(1180, 1193))),
                        torch.cat((torch.arange(7), torch.arange(661, 1173), torch.arange(1180, 1193)))))
    p = IndexedPlan.create(rows, keys, 1200, protected_ranges=((0, 7), (1180, 1193)), local_tokens=64)
    np.testing.assert_array_equal(p.protected_blocks.numpy(), ref["protected"])


def test_protection_matches_reference_on_indexed_config():
    ref = golden("c5_protection")
    for ids, r, k in workloads.group_windows(workloads.indexed_windows()):
        p = IndexedPlan.create(r, k, 32768, protected_ranges=((0, 256),), local_tokens=64)
        np.testing.assert_array_equal(p.protected_blocks[:4].numpy(), ref[f"w{ids[0]}_n{k.shape[1]}"])


def test_protection_fuzz_against_loop_restatement():
    rnd = random.Random(3)
    g = torch.Generator().manual_seed(3)
    for _ in range(150):
        W, S = rnd.randint(1, 3), rnd.randint(5, 400)
        nq, nk = rnd.randint(1, min(S, 150)), rnd.randint(1, min(S, 200))
        rows = torch.stack([torch.sort(torch.randperm(S, generator=g)[:nq]).values for _ in range(W)])
        keys = torch.stack([torch.sort(torch.randperm(S, generator=g)[:nk]).values for _ in range(W)])
        ranges = []
        for _ in range(rnd.randint(0, 2)):
            a = rnd.randint(0, S - 1)
            ranges.append((a, rnd.randint(a + 1, S)))
        loc = rnd.choice([0, 1, 5, 64, 100])
        p = IndexedPlan.create(rows, keys, S, protected_ranges=tuple(ranges), local_tokens=loc)
        assert torch.equal(p.protected_blocks, protection_loops(rows, keys, ranges, loc))


def test_plan_to_keeps_fields():
    p = fixture().to("cpu")
    assert p.sequence_length == 509 and p.rows.is_contiguous() and p.keys.dtype == torch.int64


def ragged_fixture():
    """Three windows of 96 queries whose key sets have 200, 70 and 131 keys."""
    g = torch.Generator().manual_seed(3)
    rows = torch.stack([torch.arange(s, s + 96) for s in (10, 400, 900)])
    keys = [torch.sort(torch.randperm(1200, generator=g)[:n]).values for n in (200, 70, 131)]
    return rows, keys


def test_ragged_plan_matches_per_window_plans():
    """A ragged plan (per-window key counts, an extension) pads keys with each window's last
    key and protection with False, and each window's protection equals its own plan's."""
    rows, keys = ragged_fixture()
    ranges = ((0, 7), (1180, 1193))
    p = IndexedPlan.create(rows, keys, 1200, protected_ranges=ranges, local_tokens=64)
    assert p.key_counts.tolist() == [200, 70, 131]
    assert p.key_counts.dtype == torch.int32
    assert p.keys.shape == (3, 200) and p.protected_blocks.shape == (3, 2, 4)
    for w, x in enumerate(keys):
        own = IndexedPlan.create(rows[w:w + 1], x[None], 1200, protected_ranges=ranges,
                                 local_tokens=64)
        n, nb = x.numel(), (x.numel() + 63) // 64
        assert torch.equal(p.keys[w, :n], x) and bool((p.keys[w, n:] == x[-1]).all())
        assert torch.equal(p.protected_blocks[w, :, :nb], own.protected_blocks[0])
        assert not p.protected_blocks[w, :, nb:].any()
    rect = IndexedPlan.create(rows, torch.stack([k[:70] for k in keys]), 1200)
    assert rect.key_counts is None


def test_ragged_plan_rejects_invalid_windows():
    rows, keys = ragged_fixture()
    with pytest.raises(ValueError, match="strictly increasing"):
        IndexedPlan.create(rows, [keys[0], keys[1].flip(0), keys[2]], 1200)
    with pytest.raises(ValueError, match="same batch size"):
        IndexedPlan.create(rows, keys[:2], 1200)
    with pytest.raises(ValueError, match="nonempty"):
        IndexedPlan.create(rows, [keys[0], keys[1][:0], keys[2]], 1200)
    with pytest.raises(ValueError, match="nonempty"):
        IndexedPlan.create(rows, [], 1200)
