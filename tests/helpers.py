"""Shared helpers of the test suite: golden fixtures, tolerances, input regeneration."""

from __future__ import annotations

import hashlib
import math
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
INF = math.inf


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


def digest(*xs) -> str:
    h = hashlib.sha256()
    for x in xs:
        h.update(x.detach().cpu().contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def assert_close(actual, expected):
    """The reference's tolerance (``tests/test_attention.py:20-24``)."""
    actual, expected = torch.as_tensor(actual).float().cpu(), torch.as_tensor(expected).float().cpu()
    assert torch.isfinite(actual).all()
    torch.testing.assert_close(actual, expected, atol=0.012, rtol=0.025)
    rel_l2 = (actual - expected).norm() / expected.norm().clamp_min(1e-8)
    assert rel_l2 < 0.008, float(rel_l2)


def assert_north_star(actual, expected):
    """North-star output gate: max-abs <= 2e-2 and mean-rel sum|d|/sum|ref| <= 5e-3."""
    actual, expected = torch.as_tensor(actual).float().cpu(), torch.as_tensor(expected).float().cpu()
    assert torch.isfinite(actual).all()
    delta = (actual - expected).abs()
    max_abs = float(delta.max())
    mean_rel = float(delta.sum() / expected.abs().sum().clamp_min(1e-30))
    assert max_abs <= 2e-2, max_abs
    assert mean_rel <= 5e-3, mean_rel
    return max_abs, mean_rel


def to_device(x: torch.Tensor, device="cuda") -> torch.Tensor:
    """Copy to the device keeping the exact element strides (strided views stay strided)."""
    y = torch.empty_strided(x.size(), x.stride(), dtype=x.dtype, device=device)
    y.copy_(x)
    return y


class CAbi:
    """Direct stage-by-stage calls of the C ABI (include/solattn.h), routing masks included."""

    def stages(self, q, k, v, *, beta, scale=None, local=1, kv_sink_blocks=0, q_sink_blocks=0,
               protect=None, rows=None, keys=None):
        from sol_attn_b200.stages import Stages
        st = Stages(q, k, v, beta=beta, scale=scale, local=local, kv_sink_blocks=kv_sink_blocks,
                    q_sink_blocks=q_sink_blocks, protect=protect, rows=rows, keys=keys)
        st.run()
        torch.cuda.synchronize()
        assert int(st.status[0]) == 0, f"device status {int(st.status[0])}"
        return dict(qc=st.qc, kc=st.kc, vc=st.vc, mean=st.mean, var=st.var, cut=st.cut,
                    out=st.out, counts=st.counts, mask=st.mask, force=st.force, scale=st.scale)
