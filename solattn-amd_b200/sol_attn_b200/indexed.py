"""Explicit indexed windows (mirrors ``src/sol_attn_amd/indexed.py``).

``IndexedPlan`` keeps the reference's fields, validation and messages; its protection matrix
is built with sorted-index searches instead of the reference's Python double loop over
(key block, query block) (``indexed.py:52-61``), with identical results.  As an extension the
windows may have different key counts (``keys`` given as one 1-D tensor per window): one plan
and one launch then cover windows that the reference needs a separate plan each for.
``sol_attention_indexed`` does not materialise gathered Q/K/V copies: the plan's row and key
indices are handed to the kernels, which gather rows while pooling and while loading tiles.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from .attention import SolStats, _check_out, _nonnegative_integer, _validate, launch_sol

BLOCK = 64


def build_protection(rows, keys, sequence_length, ranges, local_tokens):
    """Protected packed blocks [W, ceil(nq/64), ceil(nk/64)] (bool), ``indexed.py:50-61``.

    Key block kb of window w is protected for query block qb when one of its keys lies in a
    protected range [a, b), or within [first_row - local, last_row + local] of the q-block
    (original token indices).  ``keys`` rows are strictly increasing, so each condition is an
    interval of packed key positions found with ``searchsorted``.
    """
    W, nq = rows.shape
    nk = keys.shape[1]
    nqb, nkb = (nq + BLOCK - 1) // BLOCK, (nk + BLOCK - 1) // BLOCK
    kb_lo = torch.arange(nkb) * BLOCK          # first packed position of each key block
    kb_hi = (kb_lo + BLOCK).clamp(max=nk)      # one past its last position
    keys = keys.contiguous()

    def blocks_hit(lo, hi):
        # packed positions [lo, hi) -> which key blocks they intersect; lo/hi [W, m]
        return (lo[..., None] < kb_hi) & (hi[..., None] > kb_lo) & (lo < hi)[..., None]

    sink = torch.zeros((W, 1, nkb), dtype=torch.bool)
    for a, b in ranges:
        lo = torch.searchsorted(keys, torch.full((W, 1), a, dtype=torch.int64))
        hi = torch.searchsorted(keys, torch.full((W, 1), b, dtype=torch.int64))
        sink |= blocks_hit(lo, hi)
    first = rows[:, ::BLOCK]
    last = rows[:, (torch.arange(nqb) * BLOCK + BLOCK - 1).clamp(max=nq - 1)]
    lo = torch.searchsorted(keys, (first - local_tokens).contiguous())
    hi = torch.searchsorted(keys, (last + local_tokens).contiguous(), right=True)
    return blocks_hit(lo, hi) | sink


@dataclass(frozen=True)
class IndexedPlan:
    """Each batch has independent, sorted Q rows and an identical allowed KV set.

    Construct on CPU and transfer once, outside repeated operator timing
    (``indexed.py:11-66``). Blocks touching protected keys or the original-index local
    neighbourhood are exact; protection rounds outward to whole packed blocks.
    """

    rows: torch.Tensor
    keys: torch.Tensor
    protected_blocks: torch.Tensor
    sequence_length: int
    # Ragged plans only: int32 [W] key count of each window; ``keys`` is then padded to the
    # longest window (with the window's last key, never read) and ``protected_blocks`` to its
    # block count (False).  None for the reference's rectangular plans.
    key_counts: Optional[torch.Tensor] = None

    @classmethod
    def create(cls, rows, keys, sequence_length, *, protected_ranges=(), local_tokens=64):
        """``keys`` is a [W, nk] matrix (the reference's form) or, as an extension, a list of
        W 1-D tensors with per-window lengths (a ragged plan)."""
        _nonnegative_integer("local_tokens", local_tokens)
        _nonnegative_integer("sequence_length", sequence_length)
        if sequence_length == 0:
            raise ValueError("sequence_length must be positive")
        ragged = isinstance(keys, (list, tuple))
        key_rows = list(keys) if ragged else None
        if ragged:
            if not key_rows or any(not isinstance(x, torch.Tensor) or x.ndim != 1
                                   for x in key_rows):
                raise ValueError("keys must be a nonempty CPU int64 matrix")
            checks = [("rows", rows)] + [("keys", x[None]) for x in key_rows]
        else:
            checks = [("rows", rows), ("keys", keys)]
        for name, x in checks:
            if (x.device.type != "cpu" or x.dtype != torch.int64 or x.ndim != 2
                    or any(n == 0 for n in x.shape)):
                raise ValueError(f"{name} must be a nonempty CPU int64 matrix")
            if bool((x < 0).any() or (x >= sequence_length).any()):
                raise ValueError(f"{name} index outside sequence")
            if bool((x[:, 1:] <= x[:, :-1]).any()):
                raise ValueError(f"{name} must be strictly increasing within each batch")
        if rows.shape[0] != (len(key_rows) if ragged else keys.shape[0]):
            raise ValueError("rows and keys must have the same batch size")
        ranges = tuple(protected_ranges)
        for a, b in ranges:
            if not (isinstance(a, int) and isinstance(b, int)
                    and 0 <= a < b <= sequence_length):
                raise ValueError("Invalid protected key range")
        if not ragged:
            protection = build_protection(rows, keys, sequence_length, ranges, local_tokens)
            return cls(rows.clone().contiguous(), keys.clone().contiguous(), protection,
                       sequence_length)
        # Ragged: each window's protection exactly as its own rectangular plan, padded.
        counts = torch.tensor([x.numel() for x in key_rows], dtype=torch.int32)
        nk = int(counts.max())
        nqb, nkb = (rows.shape[1] + BLOCK - 1) // BLOCK, (nk + BLOCK - 1) // BLOCK
        padded = torch.empty((len(key_rows), nk), dtype=torch.int64)
        protection = torch.zeros((len(key_rows), nqb, nkb), dtype=torch.bool)
        for w, x in enumerate(key_rows):
            padded[w, :x.numel()] = x
            padded[w, x.numel():] = x[-1]
            own = build_protection(rows[w:w + 1], x[None], sequence_length, ranges, local_tokens)
            protection[w, :, :own.shape[2]] = own[0]
        return cls(rows.clone().contiguous(), padded, protection, sequence_length, counts)

    def to(self, device):
        return IndexedPlan(self.rows.to(device), self.keys.to(device),
                           self.protected_blocks.to(device), self.sequence_length,
                           None if self.key_counts is None else self.key_counts.to(device))


def sol_attention_indexed(q, k, v, plan, *, beta=1.0, scale=None, return_stats=False,
                          out=None):
    """BF16 NHD inputs -> [windows, query_rows, heads, D] output (``indexed.py:69-104``).

    Includes pooling, thresholds and attention over the plan's gathered rows. Plan creation
    and transfer are explicit one-time setup costs. Does not scatter output, unless ``out``
    is given (an extension: a contiguous BF16 NHD tensor shaped like ``q``): then each query
    row's output goes straight to ``out[plan.rows[w, i]]`` - the caller-side
    ``out[plan.rows] = result`` of the reference's VDN adapter - and ``out`` is returned; rows
    no window names keep their contents, and windows naming the same row race on it.
    """
    if any(t.ndim != 3 for t in (q, k, v)) or q.shape != k.shape or k.shape != v.shape:
        raise ValueError("Indexed Q/K/V must have matching NHD shapes")
    scale = _validate(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), scale)
    if not isinstance(plan, IndexedPlan):
        raise ValueError("An explicit IndexedPlan is required")
    if plan.sequence_length != q.shape[0]:
        raise ValueError("Plan sequence length does not match Q/K/V")
    if any(x.device != q.device for x in (plan.rows, plan.keys, plan.protected_blocks)):
        raise ValueError("Transfer the plan to the Q/K/V device first")
    b, nq = plan.rows.shape
    if (plan.rows.ndim != 2 or plan.keys.ndim != 2 or plan.keys.shape[0] != b
            or b <= 0 or nq <= 0 or plan.keys.shape[1] <= 0
            or plan.rows.dtype != torch.int64 or plan.keys.dtype != torch.int64
            or plan.protected_blocks.dtype != torch.bool
            or plan.protected_blocks.shape != (b, (nq + 63) // 64, (plan.keys.shape[1] + 63) // 64)
            or any(not x.is_contiguous() for x in (plan.rows, plan.keys, plan.protected_blocks))):
        raise ValueError("Invalid indexed descriptor; use IndexedPlan.create")
    kc = plan.key_counts
    if kc is not None and (kc.dtype != torch.int32 or tuple(kc.shape) != (b,)
                           or kc.device != q.device or not kc.is_contiguous()):
        raise ValueError("Invalid indexed descriptor; use IndexedPlan.create")
    beta = float(beta)
    if math.isnan(beta):
        raise ValueError("beta must not be NaN")
    out = _check_out(out, q)
    with torch.no_grad(), torch.cuda.device(q.device):
        out, counts = launch_sol(q, k, v, scale, beta, -1, 0, 0, return_stats,
                                 plan.protected_blocks, rows=plan.rows, keys=plan.keys, out=out,
                                 key_counts=kc)
    if return_stats:
        key_blocks = ((plan.keys.shape[1] + 63) // 64 if kc is None
                      else ((kc + 63) // 64).view(b, 1, 1))
        return out, SolStats(counts, key_blocks)
    return out
