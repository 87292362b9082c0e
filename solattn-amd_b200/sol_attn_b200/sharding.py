"""Head sharding across ranks (one process per GPU) for the BTHD path.

Units of the path are independent (b, h) pairs: each rank takes a contiguous range of heads
and runs pool -> threshold -> attention on strided views of its heads only; no data crosses
ranks on the hot path.  After the timed region the harness reduces timings (MAX over ranks) and
gathers per-rank results along the head axis.  Works with any torch.distributed backend (NCCL
on GPUs, gloo in the CPU tests).
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
