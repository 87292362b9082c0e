"""The allocation-free entry point ``solattn_sol_forward_noalloc``.

It exists for callers that cannot obtain device memory when they call the operator (a plugin
inside a host program that owns all device memory through its own pool, or a loop that cannot
afford cudaMalloc's implicit synchronisation): its scratch is a fixed 32 MiB device array
inside libsolattn.so rather than a caller-provided workspace.  These tests call it through the
C ABI and check it against the workspace entry point ``solattn_sol_forward`` on the same
inputs, on two calls in a row with different problems (the shared array keeps the previous
call's contents, so the second call must not see stale data).  This file is named so that
pytest collects it last.
"""

import ctypes
import math

import pytest
import torch

from helpers import assert_close, to_device
from sol_attn_b200 import _lib, workloads


def _args(q, k, v, scale, beta, local, kvs, qs):
    B, Tq, H, D = q.shape
    st = [*q.stride()[:3], *k.stride()[:3], *v.stride()[:3]]
    return [q.data_ptr(), k.data_ptr(), v.data_ptr(), B, Tq, k.shape[1], H, D, *st,
            None, None, 0, None, scale, beta, local, kvs, qs]


def _run_both(q, k, v, *, beta, local=1, kv_sink=0, q_sink=0):
    L = _lib.load()
    B, Tq, H, D = q.shape
    nqb = (Tq + 63) // 64
    scale = D ** -0.5
    common = _args(q, k, v, scale, beta, local, (kv_sink + 63) // 64, (q_sink + 63) // 64)
    stream = torch.cuda.current_stream().cuda_stream
    out_na = torch.empty((B, Tq, H, D), dtype=torch.bfloat16, device=q.device)
    cnt_na = torch.full((B, nqb, H), -1, dtype=torch.int32, device=q.device)
    rc = L.solattn_sol_forward_noalloc(*common, out_na.data_ptr(), cnt_na.data_ptr(), stream)
    _lib.check(rc, "solattn_sol_forward_noalloc")
    total, _ = _lib.workspace_layout(B, Tq, k.shape[1], H, D)
    ws = torch.empty(total + 256, dtype=torch.uint8, device=q.device)
    ws_ptr = (ws.data_ptr() + 255) // 256 * 256
    out_ws = torch.empty_like(out_na)
    cnt_ws = torch.full_like(cnt_na, -1)
    rc = L.solattn_sol_forward(*common, ws_ptr, total, out_ws.data_ptr(), cnt_ws.data_ptr(), stream)
    _lib.check(rc, "solattn_sol_forward")
    torch.cuda.synchronize()
    return out_na, cnt_na, out_ws, cnt_ws


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_two_calls_in_a_row():
    # Call 1: the reference's ragged, strided fixture with a finite beta.
    q, k, v = (to_device(x) for x in workloads.reference_fixture(d=128, b=2, strided=True))
    out_na, cnt_na, out_ws, cnt_ws = _run_both(q, k, v, beta=1.0)
    assert_close(out_na, out_ws)
    assert torch.equal(cnt_na, cnt_ws)
    first = out_na.clone()
    # Call 2: a different, larger problem (different pooled statistics, sinks, D=64).
    q2, k2, v2 = (to_device(x) for x in workloads.iid((1, 1024, 4, 64), seed=0))
    out_na, cnt_na, out_ws, cnt_ws = _run_both(q2, k2, v2, beta=1.0, kv_sink=128, q_sink=128)
    assert_close(out_na, out_ws)
    assert torch.equal(cnt_na, cnt_ws)
    # and the first problem again: the shared scratch keeps no state that changes results
    out_na, cnt_na, out_ws, _ = _run_both(q, k, v, beta=1.0)
    assert_close(out_na, first)
    assert_close(out_na, out_ws)


@pytest.mark.gpu
def test_noalloc_force_modes():
    q, k, v = (to_device(x) for x in workloads.reference_fixture(nq=1025, nk=1089, h=1))
    for beta in (-math.inf, math.inf):
        out_na, cnt_na, out_ws, cnt_ws = _run_both(q, k, v, beta=beta)
        assert_close(out_na, out_ws)
        assert torch.equal(cnt_na, cnt_ws)


def test_noalloc_rejects_problems_beyond_its_scratch():
    """Rejected on the host, before any GPU work: no device is needed for this check."""
    L = _lib.load()
    limit = L.solattn_noalloc_scratch_bytes()
    assert limit == 32 << 20
    B, T, H, D = 1, 65536, 64, 128
    assert _lib.workspace_layout(B, T, T, H, D)[0] > limit
    fake = 1 << 12  # never dereferenced: the size check fails first
    rc = L.solattn_sol_forward_noalloc(fake, fake, fake, B, T, T, H, D, T * H * D, H * D, D,
                                       T * H * D, H * D, D, T * H * D, H * D, D, None, None, 0,
                                       None, D ** -0.5, 1.0, 1, 0, 0, fake, None, None)
    assert rc == -6
    assert b"no-allocation" in L.solattn_strerror(rc)
