"""The C-ABI library loads, exports every symbol of include/solattn.h and rejects bad
arguments on the host (no GPU needed: every rejected call returns before any CUDA call)."""

import ctypes
import re
from pathlib import Path

import pytest

from sol_attn_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "solattn.h"


def declared():
    return re.findall(r"SOLATTN_API\s+[\w\s\*]+?\b(solattn_\w+)\s*\(", HEADER.read_text())


def test_header_declares_the_boundary():
    names = set(declared())
    assert {"solattn_pool_qkv", "solattn_threshold", "solattn_attention", "solattn_sol_forward",
            "solattn_dense", "solattn_workspace_layout", "solattn_strerror"} <= names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared():
        assert hasattr(lib, name), name
    # and the Python binding declares a signature for each of them
    assert set(declared()) == set(_lib.SIGNATURES)


def test_version_and_messages():
    L = _lib.load()
    assert b"sm_100a" in L.solattn_version()
    for code in (0, -1, -2, -3, -4, -5):
        assert L.solattn_strerror(code)


def test_workspace_layout():
    total, offs = _lib.workspace_layout(1, 32768, 32768, 24, 128)
    nkb = nqb = 512
    assert offs["status"] == 0
    assert all(v % 256 == 0 for v in offs.values())
    assert offs["vc"] - offs["kc"] >= 24 * nkb * 128 * 2
    assert offs["mean"] - offs["qc"] >= 24 * nqb * 128 * 4
    assert offs["masks"] >= offs["cutoff"] + 24 * nqb * 4
    assert total >= offs["masks"] + 24 * nqb * (nkb // 32) * 4
    assert _lib.workspace_layout(1, 100, 100, 2, 96)[0] == 0      # unsupported head dim
    assert _lib.workspace_layout(0, 100, 100, 2, 64)[0] == 0      # empty batch
    # the status section holds the status word and two int32 [B * H] counter arrays
    assert offs["kc"] >= 16 + 8 * 24
    # cached per shape: the same values, and a dict the caller may change freely
    again = _lib.workspace_layout(1, 32768, 32768, 24, 128)
    assert again == (total, offs) and again[1] is not offs
    offs["kc"] = -1
    assert _lib.workspace_layout(1, 32768, 32768, 24, 128)[1]["kc"] >= 0


@pytest.mark.parametrize("B,Tq,Tk,H", [(1, 32768, 32768, 24), (2, 8192, 5000, 8), (3, 100, 65, 5)])
def test_mask_buffer_sections(B, Tq, Tk, H):
    """solattn_masks_bytes = bitmask words and the work counter (padded to 16 bytes), one tile
    list per q-block pair, then the item-order section (arrive and stamp words padded to 16
    bytes, one order word per pair); the GPU tests read the sections with this arithmetic."""
    nqb, nkb = -(-Tq // 64), -(-Tk // 64)
    bh, npairs = B * H, -(-nqb // 2)
    words = (bh * nqb * -(-nkb // 32) + 1 + 3) & ~3
    stride = 16 + 2 * (((nkb + 63) // 64 + nkb + 1 + 7) & ~7)
    pad = (bh + 3) & ~3
    want = 4 * words + bh * npairs * stride + 4 * (2 * pad + bh * npairs)
    assert _lib.load().solattn_masks_bytes(B, Tq, Tk, H) == want
    assert stride % 16 == 0 and (4 * words) % 16 == 0  # lists and the order section 16-aligned


def _forward(**over):
    args = dict(q=16, k=16, v=16, B=1, Tq=64, Tk=64, H=1, D=64, strides=(4096, 64, 64),
                q_idx=None, kv_idx=None, idx_rows=0, protect=None, scale=0.125, beta=1.0,
                local=1, kvs=0, qs=0, ws=256, ws_bytes=1 << 20, out=16, counts=None)
    args.update(over)
    a = args
    return _lib.load().solattn_sol_forward(
        a["q"], a["k"], a["v"], a["B"], a["Tq"], a["Tk"], a["H"], a["D"], *a["strides"],
        *a["strides"], *a["strides"], a["q_idx"], a["kv_idx"], a["idx_rows"], a["protect"],
        a["scale"], a["beta"], a["local"], a["kvs"], a["qs"], a["ws"], a["ws_bytes"], a["out"],
        a["counts"], None)


@pytest.mark.parametrize("bad,code", [
    (dict(D=96), -2), (dict(Tq=0), -1), (dict(H=0), -1), (dict(beta=float("nan")), -1),
    (dict(ws=None), -1), (dict(ws_bytes=16), -1), (dict(ws=128), -1), (dict(q=8), -1),
    (dict(strides=(4096, 63, 64)), -1), (dict(q=None), -1), (dict(scale=0.0), -1),
    (dict(scale=float("inf")), -1), (dict(kvs=-1), -1), (dict(kv_idx=16, idx_rows=0), -1),
])
def test_forward_rejects_bad_arguments(bad, code):
    assert _forward(**bad) == code


def test_threshold_rejects_nonfinite_beta():
    L = _lib.load()
    assert L.solattn_threshold(16, 16, 1, 1, 1, 1, 64, 0.125, float("inf"), 16, 16, 16, None) == -1


def test_scatter_and_dense_rows_reject_bad_arguments():
    """The scatter forward needs the query index and a positive row count; the dense-rows form
    needs a row index, at least one row and a nonempty sequence (all rejected before any CUDA
    call)."""
    L = _lib.load()
    st = (4096, 64, 64)
    common = [16, 16, 16, 1, 64, 64, 1, 64, *st, *st, *st]
    tail = [None, 0.125, 1.0, 1, 0, 0, 256, 1 << 20, 16]
    assert L.solattn_sol_forward_scatter(*common, None, None, 0, *tail, 64, None, None) == -1
    assert L.solattn_sol_forward_scatter(*common, 16, None, 64, *tail, 0, None, None) == -1
    assert L.solattn_dense_rows(16, 16, 16, None, 4, 64, 1, 64, 64, 64, 64, 64, 64, 64, 0.125,
                                16, None, None) == -1
    assert L.solattn_dense_rows(16, 16, 16, 16, 0, 64, 1, 64, 64, 64, 64, 64, 64, 64, 0.125,
                                16, None, None) == -1
    assert L.solattn_dense_rows(16, 16, 16, 16, 4, 64, 1, 96, 64, 64, 64, 64, 64, 64, 0.125,
                                16, None, None) == -2


def test_status_entry_points_reject_null_pointers():
    """The status copy and the no-allocation status accessors check their pointers first."""
    L = _lib.load()
    assert L.solattn_status_to_host(None, 16, None) == -1
    assert L.solattn_status_to_host(16, None, None) == -1
    assert L.solattn_noalloc_read_status(None, None) == -1
    assert L.solattn_noalloc_scratch_address(None) == -1
