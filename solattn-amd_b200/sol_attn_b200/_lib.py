"""ctypes binding of libsolattn.so (the C ABI declared in include/solattn.h).

The library is loaded lazily on first use so that the package imports on machines without a
GPU (plan construction and validation are host-only).  There is no fallback: if the library
is missing or fails to load, every operator raises.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_void_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libsolattn.so")

_I64 = c_int64
_P = c_void_p

# name -> (restype, argtypes); mirrors include/solattn.h exactly.
SIGNATURES = {
    "solattn_version": (ctypes.c_char_p, []),
    "solattn_strerror": (ctypes.c_char_p, [c_int]),
    "solattn_workspace_layout": (_I64, [_I64] * 5 + [POINTER(_I64)] * 8),
    "solattn_pool_qkv": (c_int, [_P, _P, _P] + [_I64] * 5 + [_I64] * 9 + [_P, _P, _I64, c_int]
                         + [_P, _P, _P, _P, _P]),
    "solattn_threshold": (c_int, [_P, _P] + [_I64] * 5 + [c_float, c_float] + [_P] * 3 + [_P]),
    "solattn_attention": (c_int, [_P, _P, _P] + [_I64] * 5 + [_I64] * 9 + [_P, _P, _I64]
                          + [_P, _P, _P, _P, _P, c_float, c_int, c_int, c_int, c_int]
                          + [_P, _P, _P, _P, _P]),
    "solattn_sol_forward": (c_int, [_P, _P, _P] + [_I64] * 5 + [_I64] * 9 + [_P, _P, _I64, _P]
                            + [c_float, c_float, c_int, c_int, c_int, _P, _I64, _P, _P, _P]),
    "solattn_sol_forward_scatter": (c_int, [_P, _P, _P] + [_I64] * 5 + [_I64] * 9
                                    + [_P, _P, _I64, _P]
                                    + [c_float, c_float, c_int, c_int, c_int, _P, _I64, _P, _I64,
                                       _P, _P]),
    "solattn_sol_forward_ex": (c_int, [_P, _P, _P] + [_I64] * 5 + [_I64] * 9
                               + [_P, _P, _I64, _P]
                               + [c_float, c_float, c_int, c_int, c_int, _P, _I64, _P, _P, _I64,
                                  _P, _P]),
    "solattn_dense": (c_int, [_P, _P, _P] + [_I64] * 5 + [_I64] * 9 + [c_float, _P, _P, _P]),
    "solattn_dense_rows": (c_int, [_P, _P, _P, _P] + [_I64] * 4 + [_I64] * 6
                           + [c_float, _P, _P, _P]),
    "solattn_read_status": (c_int, [_P, _P, _P]),
    "solattn_status_to_host": (c_int, [_P, _P, _P]),
    "solattn_noalloc_scratch_address": (c_int, [POINTER(c_void_p)]),
    "solattn_noalloc_read_status": (c_int, [_P, _P]),
    "solattn_sol_forward_noalloc": (c_int, [_P, _P, _P] + [_I64] * 5 + [_I64] * 9
                                    + [_P, _P, _I64, _P]
                                    + [c_float, c_float, c_int, c_int, c_int, _P, _P, _P]),
    "solattn_noalloc_scratch_bytes": (_I64, []),
    "solattn_masks_bytes": (_I64, [_I64] * 4),
    "solattn_copy_2d": (c_int, [_P, _I64, _P, _I64, _I64, _I64, c_int, _P]),
}

_lib = None


class SolAttnError(RuntimeError):
    """A nonzero status returned by libsolattn."""


def load():
    """Load (once) and return the ctypes library handle; raise if it is absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built (expected at {LIB_PATH}); run "
                "`python -m sol_attn_b200.build` or __graft_entry__.build(). There is no "
                "fallback implementation.")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().solattn_strerror(rc).decode()
        raise SolAttnError(f"{what} failed: {msg} (code {rc})")


_LAYOUTS: dict = {}


def workspace_layout(B, Tq, Tk, H, D):
    """Byte offsets and total size of the scratch of one forward call (cached per shape and
    library handle: the call sits on every forward's host path)."""
    lib = load()
    key = (id(lib), B, Tq, Tk, H, D)
    hit = _LAYOUTS.get(key)
    if hit is None:
        offs = [c_int64(0) for _ in range(8)]
        total = lib.solattn_workspace_layout(B, Tq, Tk, H, D, *[ctypes.byref(o) for o in offs])
        names = ("kc", "vc", "qc", "mean", "var", "cutoff", "status", "masks")
        hit = (total, {n: o.value for n, o in zip(names, offs)})
        if len(_LAYOUTS) >= 4096:
            _LAYOUTS.clear()
        _LAYOUTS[key] = hit
    return hit[0], dict(hit[1])
