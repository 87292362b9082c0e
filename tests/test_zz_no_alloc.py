"""The allocation-free entry point ``solattn_sol_forward_noalloc``.

It exists for callers that cannot obtain device memory when they call the operator (a plugin
inside a host program that owns all device memory through its own pool, or a loop that cannot
afford cudaMalloc's implicit synchronisation): its scratch is a fixed 32 MiB device array
inside libsolattn.so rather than a caller-provided workspace.  These tests call it through the
C ABI and check it against the workspace entry point ``solattn_sol_forward`` on the same
inputs, on calls in a row with different problems.  The shared array keeps the previous call's
contents, so before the later calls it is filled with NaN bytes: a call that read anything it
had not written first would not reproduce the workspace entry point bit for bit.  This file is
named so that pytest collects it last.
"""

import ctypes
import math

import pytest
import torch

from helpers import to_device
from sol_attn_b200 import _lib, workloads


def _args(q, k, v, scale, beta, local, kvs, qs):
    B, Tq, H, D = q.shape
    st = [*q.stride()[:3], *k.stride()[:3], *v.stride()[:3]]
    return [q.data_ptr(), k.data_ptr(), v.data_ptr(), B, Tq, k.shape[1], H, D, *st,
            None, None, 0, None, scale, beta, local, kvs, qs]


class _DeviceBytes:
    """A raw device address seen as a uint8 tensor (no allocation, no copy)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}


def _scratch():
    L = _lib.load()
    addr = ctypes.c_void_p(0)
    _lib.check(L.solattn_noalloc_scratch_address(ctypes.byref(addr)),
               "solattn_noalloc_scratch_address")
    return torch.as_tensor(_DeviceBytes(addr.value, L.solattn_noalloc_scratch_bytes()),
                           device="cuda")


def _poison():
    """Fill the whole shared array with 0xFF bytes (NaN as BF16 and FP32)."""
    _scratch().fill_(0xFF)


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
    status = ctypes.c_int32(-1)
    _lib.check(L.solattn_noalloc_read_status(ctypes.byref(status), stream),
               "solattn_noalloc_read_status")
    assert status.value == 0
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
    assert torch.equal(out_na, out_ws)
    assert torch.equal(cnt_na, cnt_ws)
    first = out_na.clone()
    # Call 2: a different, larger problem (different pooled statistics, sinks, D=64), on a
    # poisoned array.
    _poison()
    q2, k2, v2 = (to_device(x) for x in workloads.iid((1, 1024, 4, 64), seed=0))
    out_na, cnt_na, out_ws, cnt_ws = _run_both(q2, k2, v2, beta=1.0, kv_sink=128, q_sink=128)
    assert torch.equal(out_na, out_ws)
    assert torch.equal(cnt_na, cnt_ws)
    # and the first problem again, poisoned again: the shared scratch keeps no state that
    # changes results
    _poison()
    out_na, cnt_na, out_ws, cnt_ws = _run_both(q, k, v, beta=1.0)
    assert torch.equal(out_na, first)
    assert torch.equal(out_na, out_ws)
    assert torch.equal(cnt_na, cnt_ws)


@pytest.mark.gpu
def test_noalloc_force_modes():
    q, k, v = (to_device(x) for x in workloads.reference_fixture(nq=1025, nk=1089, h=1))
    for beta in (-math.inf, math.inf):
        _poison()
        out_na, cnt_na, out_ws, cnt_ws = _run_both(q, k, v, beta=beta)
        assert torch.equal(out_na, out_ws)
        assert torch.equal(cnt_na, cnt_ws)


@pytest.mark.gpu
def test_noalloc_status_word_is_readable():
    """The status word at offset 0 of the array is what solattn_noalloc_read_status reads and
    clears (written here by the host; no kernel is made to fail)."""
    L = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    word = _scratch()[:4].view(torch.int32)
    word.fill_(2)
    status = ctypes.c_int32(0)
    assert L.solattn_noalloc_read_status(ctypes.byref(status), stream) == -4
    assert status.value == 2
    assert L.solattn_noalloc_read_status(ctypes.byref(status), stream) == 0
    assert status.value == 0


@pytest.mark.gpu
def test_noalloc_reports_a_gather_index_outside_its_tensor():
    """A query row index equal to the NHD tensor's row count (the Python layer rejects such
    plans; the C entry point does not look at the indices): the kernels' own bounds checks read
    row 0 in its place and record kStatusBadIndex (2) in the array's status word, which
    solattn_noalloc_read_status returns as SOLATTN_ERR_DEVICE and clears."""
    L = _lib.load()
    N, H, D, W, n = 1024, 2, 64, 2, 256
    gen = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn((N, H, D), generator=gen).to(torch.bfloat16).cuda() for _ in range(3))
    rows = torch.arange(W * n, dtype=torch.int64).view(W, n)
    rows[1, 7] = N  # outside [0, N)
    keys = torch.arange(W * n, dtype=torch.int64).view(W, n)
    rows, keys = rows.cuda(), keys.cuda()
    out = torch.empty((W, n, H, D), dtype=torch.bfloat16, device="cuda")
    counts = torch.empty((W, (n + 63) // 64, H), dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    st = (0, H * D, D)
    rc = L.solattn_sol_forward_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), W, n, n, H, D,
                                       *st, *st, *st, rows.data_ptr(), keys.data_ptr(), N, None,
                                       D ** -0.5, 1.0, -1, 0, 0, out.data_ptr(),
                                       counts.data_ptr(), stream)
    assert rc == 0
    status = ctypes.c_int32(0)
    assert L.solattn_noalloc_read_status(ctypes.byref(status), stream) == -4
    assert status.value == 2
    assert L.solattn_noalloc_read_status(ctypes.byref(status), stream) == 0
    assert status.value == 0


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


@pytest.mark.parametrize("shape,code", [
    ((1, 64, 64, 1, 96), -2),            # head dimension
    ((1, 64, 64 * 16385, 1, 64), -2),    # more key blocks than the routing bitmask holds
    ((1, 64, 64, 65536, 64), -2),        # more (batch x head) units than the grid takes
    ((0, 64, 64, 1, 64), -1),            # empty batch
])
def test_noalloc_rejects_shapes_like_the_workspace_entry_point(shape, code):
    """A shape the workspace entry point rejects gets the same code here (host-side checks)."""
    L = _lib.load()
    B, Tq, Tk, H, D = shape
    fake = 1 << 12
    st = [Tq * H * D, H * D, D]
    common = [fake, fake, fake, B, Tq, Tk, H, D, *st, *st, *st, None, None, 0, None, 0.125, 1.0,
              1, 0, 0]
    rc_na = L.solattn_sol_forward_noalloc(*common, fake, None, None)
    rc_ws = L.solattn_sol_forward(*common, fake * 256, 1 << 40, fake, None, None)
    assert rc_na == rc_ws == code
