"""Multi-rank head sharding (the N>1 path of bench.py) and window sharding of indexed plans, on
CPU with gloo, world size 2.

Each rank computes its head shard with the CPU oracle as the compute stand-in (the GPU kernels
are per-(b, h) independent, so the harness logic is what is under test): shard bounds, MAX
reduction of per-rank timings and the all-gather of outputs and exact-block counts must
reproduce the single-process result exactly.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "solattn-amd_b200")]
    from oracle.sol_oracle import sol_oracle
    from sol_attn_b200 import workloads
    from sol_attn_b200.sharding import gather_heads, head_shard, max_over_ranks
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = workloads.block_smooth(b=1, t=256, h=4, d=64, sigma=0.1, seed=3)
        h0, h1 = head_shard(q.shape[2], rank, world)
        out, counts = sol_oracle(q[:, :, h0:h1], k[:, :, h0:h1], v[:, :, h0:h1], beta=1.0,
                                 kv_sink_tokens=64, query_sink_tokens=64)
        t = max_over_ranks([float(rank + 1), 10.0 * (world - rank)])
        full_out = gather_heads(out)
        full_counts = gather_heads(counts)
        if rank == 0:
            torch.save(dict(out=full_out, counts=full_counts, t=t), result_path)
    finally:
        dist.destroy_process_group()


def test_head_sharding_matches_single_process(tmp_path):
    from oracle.sol_oracle import sol_oracle
    from sol_attn_b200 import workloads
    world = 2
    path = str(tmp_path / "r.pt")
    mp.start_processes(_worker, args=(world, _free_port(), path), nprocs=world,
                       start_method="spawn", join=True)
    r = torch.load(path)
    q, k, v = workloads.block_smooth(b=1, t=256, h=4, d=64, sigma=0.1, seed=3)
    out, counts = sol_oracle(q, k, v, beta=1.0, kv_sink_tokens=64, query_sink_tokens=64)
    assert torch.equal(r["counts"], counts)
    torch.testing.assert_close(r["out"], out, rtol=0, atol=0)
    assert r["t"] == [2.0, 20.0]


def test_head_shard_bounds():
    from sol_attn_b200.sharding import head_shard
    assert [head_shard(24, r, 8) for r in range(8)][-1] == (21, 24)
    assert head_shard(24, 1, 2) == (12, 24)
    with pytest.raises(ValueError):
        head_shard(24, 0, 5)


def _plan_inputs():
    from sol_attn_b200 import IndexedPlan, workloads
    t, window = 1024, 128
    q, k, v = (x[0] for x in workloads.block_smooth(b=1, t=t, h=2, d=64, sigma=0.1, seed=5))
    wins = workloads.indexed_windows(t, window=window, halo=128, anchor=64, stride=4)
    # rectangular (equal key counts) so that the CPU oracle takes the plan as it is
    sizes = {kk.numel() for _, kk in wins}
    n = min(sizes)
    rows = torch.stack([r for r, _ in wins])
    keys = torch.stack([kk[:n] for _, kk in wins])
    plan = IndexedPlan.create(rows, keys, t, protected_ranges=((0, 64),))
    return q, k, v, plan


def _window_worker(rank, world, port, result_path):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "solattn-amd_b200")]
    from oracle.sol_oracle import indexed_oracle
    from sol_attn_b200.sharding import gather_windows, plan_windows, window_shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, plan = _plan_inputs()
        windows = plan.rows.shape[0]
        w0, w1 = window_shard(windows, rank, world)
        sub = plan_windows(plan, w0, w1)
        out, counts = indexed_oracle(q, k, v, sub.rows, sub.keys, sub.protected_blocks, beta=1.0)
        full_out = gather_windows(out, windows)
        full_counts = gather_windows(counts, windows)
        if rank == 0:
            torch.save(dict(out=full_out, counts=full_counts), result_path)
    finally:
        dist.destroy_process_group()


def test_window_sharding_matches_single_process(tmp_path):
    from oracle.sol_oracle import indexed_oracle
    world = 2
    path = str(tmp_path / "w.pt")
    mp.start_processes(_window_worker, args=(world, _free_port(), path), nprocs=world,
                       start_method="spawn", join=True)
    r = torch.load(path)
    q, k, v, plan = _plan_inputs()
    out, counts = indexed_oracle(q, k, v, plan.rows, plan.keys, plan.protected_blocks, beta=1.0)
    assert r["out"].shape == out.shape
    assert torch.equal(r["counts"], counts)
    torch.testing.assert_close(r["out"], out, rtol=0, atol=0)


def test_window_shard_bounds_and_plan_slices():
    import torch as th
    from sol_attn_b200.sharding import plan_windows, window_shard
    assert [window_shard(64, r, 8) for r in range(8)][-1] == (56, 64)
    assert [window_shard(10, r, 4) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    with pytest.raises(ValueError):
        window_shard(3, 0, 4)
    _, _, _, plan = _plan_inputs()
    sub = plan_windows(plan, 2, 5)
    assert th.equal(sub.rows, plan.rows[2:5]) and th.equal(sub.keys, plan.keys[2:5])
    assert th.equal(sub.protected_blocks, plan.protected_blocks[2:5])
    assert sub.sequence_length == plan.sequence_length and sub.key_counts is None
    with pytest.raises(ValueError):
        plan_windows(plan, 3, 3)
