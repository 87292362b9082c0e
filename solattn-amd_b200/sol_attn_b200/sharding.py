"""Sharding across ranks (one process per GPU): heads for the BTHD path, windows for indexed
plans.

Units of the path are independent: (b, h) pairs for BTHD inputs, and the windows of an
``IndexedPlan`` (each window is pooled, thresholded and routed on its own).  Each rank takes a
contiguous range of heads (strided views of its heads) or of windows (a plan of its own) and runs
pool -> threshold -> attention on it; no data crosses ranks on the hot path.  After the timed
region the harness reduces timings (MAX over ranks) and gathers per-rank results along the head
or window axis.  Works with any torch.distributed backend (NCCL on GPUs, gloo in the CPU tests).
"""

from __future__ import annotations

import torch


def head_shard(heads: int, rank: int, world: int):
    """Contiguous head range [h0, h1) of ``rank``; heads must divide evenly."""
    if world <= 0 or heads % world:
        raise ValueError(f"{heads} heads do not shard evenly over {world} ranks")
    per = heads // world
    return rank * per, (rank + 1) * per


def max_over_ranks(values, device=None):
    """MAX all-reduce of a list of floats (per-rank timings) -> list of floats."""
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def gather_heads(local: torch.Tensor, head_dim: int = 2) -> torch.Tensor:
    """All-gather per-rank head shards and concatenate them along ``head_dim``."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return local
    local = local.contiguous()
    parts = [torch.empty_like(local) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, local)
    return torch.cat(parts, dim=head_dim)


def window_shard(windows: int, rank: int, world: int):
    """Contiguous window range [w0, w1) of ``rank``: the first ``windows % world`` ranks take one
    window more than the others, so any window count of at least ``world`` shards."""
    if world <= 0 or windows < world:
        raise ValueError(f"{windows} windows do not shard over {world} ranks")
    base, extra = divmod(windows, world)
    w0 = rank * base + min(rank, extra)
    return w0, w0 + base + (1 if rank < extra else 0)


def plan_windows(plan, w0: int, w1: int):
    """Windows [w0, w1) of an ``IndexedPlan`` as a plan of their own (rows, keys, protection and,
    for a ragged plan, key counts sliced).  Its results are bitwise those of the same windows in
    a call on the whole plan."""
    from .indexed import IndexedPlan
    if not 0 <= w0 < w1 <= plan.rows.shape[0]:
        raise ValueError(f"window range [{w0}, {w1}) outside the plan's {plan.rows.shape[0]}")
    counts = plan.key_counts
    return IndexedPlan(plan.rows[w0:w1].contiguous(), plan.keys[w0:w1].contiguous(),
                       plan.protected_blocks[w0:w1].contiguous(), plan.sequence_length,
                       None if counts is None else counts[w0:w1].contiguous())


def gather_windows(local: torch.Tensor, windows: int) -> torch.Tensor:
    """All-gather per-rank window shards (dim 0, as ``window_shard`` splits ``windows``) into
    one tensor in window order; uneven shards are padded for the collective and trimmed."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return local
    world = dist.get_world_size()
    bounds = [window_shard(windows, r, world) for r in range(world)]
    most = max(b - a for a, b in bounds)
    padded = torch.zeros((most,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    padded[:local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded)
    return torch.cat([part[:b - a] for part, (a, b) in zip(parts, bounds)], dim=0)
