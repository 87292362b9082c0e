"""Public BTHD interface (mirrors ``src/sol_attn_amd/attention.py`` of zihaomu/SolAttn-AMD).

Same names, keyword-only arguments, defaults, return types and ValueError messages as the
reference; the device requirement is an NVIDIA B200 (sm_100a) instead of a ROCm GPU.  The
compute runs in libsolattn.so (hand-written sm_100a CUDA) through its C ABI on torch's
current stream; there is no fallback path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib
from .status import check_device_errors, monitor

BLOCK = 64
_DEVICE_OK = {}


@dataclass(frozen=True)
class SolStats:
    """Per-(batch, q-block, head) exact-block counts (``attention.py:10-16``)."""

    # Device tensor [batch, query_blocks, heads]; obtaining a Python density syncs.
    exact_blocks: torch.Tensor
    # Key blocks per query block; for a ragged indexed plan a per-window int tensor
    # [batch, 1, 1] on the same device (windows have different key counts).
    key_blocks: int

    def density(self) -> float:
        # Synchronises anyway: first raise if a call on this device reported a device error.
        if self.exact_blocks.is_cuda:
            check_device_errors(self.exact_blocks.device)
        if isinstance(self.key_blocks, torch.Tensor):
            return (self.exact_blocks.float() / self.key_blocks).mean().item()
        return self.exact_blocks.float().mean().item() / self.key_blocks


def _is_b200(device: torch.device) -> bool:
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _DEVICE_OK:
        _DEVICE_OK[key] = torch.cuda.get_device_capability(key) == (10, 0)
    return _DEVICE_OK[key]


def _validate(q, k, v, scale):
    """Input contract of ``attention.py:19-44`` (device check re-targeted to sm_100a)."""
    if any(t.ndim != 4 for t in (q, k, v)):
        raise ValueError("Q/K/V must have BTHD rank-4 layout")
    if (k.shape != v.shape or q.shape[0] != k.shape[0]
            or q.shape[2:] != k.shape[2:] or any(n <= 0 for n in q.shape + k.shape)):
        raise ValueError("Q/K/V batch, head and dimension shapes must agree and be nonempty")
    if any(t.dtype != torch.bfloat16 for t in (q, k, v)):
        raise ValueError("Only BF16 Q/K/V are implemented")
    if q.shape[-1] not in (64, 128):
        raise ValueError("Only head dimensions 64 and 128 are implemented")
    if any(t.requires_grad for t in (q, k, v)):
        raise ValueError("Inference only: Q/K/V must not require gradients")
    if any(t.stride(-1) != 1 or any(s <= 0 for s in t.stride()) for t in (q, k, v)):
        raise ValueError("Q/K/V need positive strides and contiguous head dimension")
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    if not math.isfinite(scale) or scale <= 0:
        raise ValueError("scale must be finite and positive")
    if (q.device.type != "cuda" or k.device != q.device or v.device != q.device
            or not _is_b200(q.device)):
        raise ValueError("The sm_100a backend requires Q/K/V on the same NVIDIA B200 CUDA GPU")
    return scale


def _nonnegative_integer(name, value):
    if not isinstance(value, int) or isinstance(value, bool) or value < 0:
        raise ValueError(f"{name} must be a nonnegative integer")


def _aligned(x: torch.Tensor) -> bool:
    """Rows must start on 16-byte boundaries for the 128-bit loads of the kernels."""
    return x.data_ptr() % 16 == 0 and all(s % 8 == 0 for s in x.stride()[:-1])


def _strides(x: torch.Tensor, indexed: bool):
    """(sB, sT, sH) element strides; NHD tensors of the indexed API have sB = 0."""
    if indexed:
        return 0, x.stride(0), x.stride(1)
    return x.stride(0), x.stride(1), x.stride(2)


def launch_sol(q, k, v, scale, beta, local, kv_sink, q_sink, stats, protection=None,
               rows=None, keys=None, out=None, key_counts=None):
    """Allocate outputs + workspace and run the all-in forward (``kernels.py:203-225``).

    BTHD inputs, or NHD inputs with gather indices ``rows`` [W, nq] / ``keys`` [W, nk]
    (then the logical shape is B=W, Tq=nq, Tk=nk).  With ``out`` (indexed only: an NHD tensor
    like ``q``) each query row's output is written to ``out[rows[w, i]]`` instead of a fresh
    [W, nq, H, D] tensor.  ``key_counts`` (int32 [W] on the device) gives each window its own
    key count in a ragged plan (``keys`` padded to the longest window).  Returns (out, counts).
    """
    indexed = rows is not None
    # The kernels need 16-byte-aligned rows; other positive strides are made contiguous first.
    q, k, v = (x if _aligned(x) else x.contiguous() for x in (q, k, v))
    if indexed:
        B, Tq = rows.shape
        Tk = keys.shape[1]
        H, D = q.shape[1], q.shape[2]
        out_shape = (B, Tq, H, D)
    else:
        B, Tq, H, D = q.shape
        Tk = k.shape[1]
        out_shape = tuple(q.shape)
    nqb = (Tq + BLOCK - 1) // BLOCK
    L = _lib.load()
    mon = monitor(q.device)
    mon.poll(wait=False)  # an earlier call's device-side error surfaces here
    total, offs = _lib.workspace_layout(B, Tq, Tk, H, D)
    if total <= 0:
        raise _lib.SolAttnError("unsupported shape for libsolattn")
    workspace = torch.empty(total + 256, dtype=torch.uint8, device=q.device)
    ws_ptr = (workspace.data_ptr() + 255) // 256 * 256
    scatter = out is not None
    if not scatter:
        out = torch.empty(out_shape, dtype=torch.bfloat16, device=q.device)
    counts = torch.empty((B, nqb, H), dtype=torch.int32, device=q.device)
    tstream = torch.cuda.current_stream(q.device)
    stream = tstream.cuda_stream
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), B, Tq, Tk, H, D,
            *_strides(q, indexed), *_strides(k, indexed), *_strides(v, indexed),
            rows.data_ptr() if indexed else None, keys.data_ptr() if indexed else None,
            q.shape[0] if indexed else 0,
            protection.data_ptr() if protection is not None else None,
            float(scale), float(beta), int(local), (kv_sink + BLOCK - 1) // BLOCK,
            (q_sink + BLOCK - 1) // BLOCK, ws_ptr, total, out.data_ptr())
    if key_counts is not None:
        rc = L.solattn_sol_forward_ex(*args[:-1], key_counts.data_ptr(), out.data_ptr(),
                                      out.shape[0] if scatter else 0,
                                      counts.data_ptr() if stats else None, stream)
        _lib.check(rc, "solattn_sol_forward_ex")
    elif scatter:
        rc = L.solattn_sol_forward_scatter(*args, out.shape[0],
                                           counts.data_ptr() if stats else None, stream)
        _lib.check(rc, "solattn_sol_forward_scatter")
    else:
        rc = L.solattn_sol_forward(*args, counts.data_ptr() if stats else None, stream)
        _lib.check(rc, "solattn_sol_forward")
    # The call's status word (cleared by the call itself) travels to pinned host memory
    # asynchronously; the next call or SolStats.density() looks at it.
    mon.record(ws_ptr + offs["status"], tstream)
    return out, counts


def _dense_status(device):
    """A zeroed device status word for the dense entry points, after polling earlier calls."""
    mon = monitor(device)
    mon.poll(wait=False)
    return mon, torch.zeros(4, dtype=torch.int32, device=device)


def dense_attention(q, k, v, *, scale=None):
    """Noncausal BF16 attention over all keys, FP32 softmax/accumulation (``attention.py:47-55``).

    Runs the all-exact route of the fused sm_100a kernel.
    """
    scale = _validate(q, k, v, scale)
    with torch.no_grad(), torch.cuda.device(q.device):
        q, k, v = (x if _aligned(x) else x.contiguous() for x in (q, k, v))
        B, Tq, H, D = q.shape
        mon, status = _dense_status(q.device)
        out = torch.empty(tuple(q.shape), dtype=torch.bfloat16, device=q.device)
        tstream = torch.cuda.current_stream(q.device)
        rc = _lib.load().solattn_dense(q.data_ptr(), k.data_ptr(), v.data_ptr(), B, Tq,
                                       k.shape[1], H, D, *_strides(q, False), *_strides(k, False),
                                       *_strides(v, False), float(scale), out.data_ptr(),
                                       status.data_ptr(), tstream.cuda_stream)
        _lib.check(rc, "solattn_dense")
        mon.record(status.data_ptr(), tstream)
        return out


def dense_attention_rows(q, k, v, rows, *, scale=None, out=None):
    """Dense attention of the query rows ``rows`` against all keys, written to ``out[rows]``.

    ``q``, ``k``, ``v`` are NHD [N, H, D] BF16 CUDA tensors of one sequence and ``rows`` a 1-D
    int64 tensor of row indices on their device.  This is the VDN adapter's dense step for
    global queries (``out[rows] = dense(q[rows], k, v, scale)``,
    ``integrations/vdn.py:58-63``) without the gathered copy of Q or the scatter; it has no
    counterpart in the reference package.  ``out`` (NHD like ``q``, contiguous) receives the
    rows and is returned; when omitted a new uninitialised tensor like ``q`` is used, as the
    adapter's ``torch.empty_like(q)``.  Rows outside [0, N) are reported by the kernel's status
    word and skipped.
    """
    if any(t.ndim != 3 for t in (q, k, v)) or q.shape != k.shape or k.shape != v.shape:
        raise ValueError("Q/K/V must have matching NHD shapes")
    scale = _validate(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), scale)
    if (not isinstance(rows, torch.Tensor) or rows.dtype != torch.int64 or rows.ndim != 1
            or rows.numel() == 0 or rows.device != q.device):
        raise ValueError("rows must be a nonempty 1-D int64 tensor on the Q/K/V device")
    out = _check_out(out, q)
    with torch.no_grad(), torch.cuda.device(q.device):
        q, k, v = (x if _aligned(x) else x.contiguous() for x in (q, k, v))
        rows = rows.contiguous()
        if out is None:
            out = torch.empty_like(q, memory_format=torch.contiguous_format)
        N, H, D = q.shape
        mon, status = _dense_status(q.device)
        tstream = torch.cuda.current_stream(q.device)
        rc = _lib.load().solattn_dense_rows(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), rows.data_ptr(), rows.numel(), N, H, D,
            q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
            float(scale), out.data_ptr(), status.data_ptr(), tstream.cuda_stream)
        _lib.check(rc, "solattn_dense_rows")
        mon.record(status.data_ptr(), tstream)
        return out


def _check_out(out, q):
    """Validate a caller-provided NHD output tensor shaped like ``q``."""
    if out is None:
        return None
    if (not isinstance(out, torch.Tensor) or out.dtype != torch.bfloat16
            or out.device != q.device or tuple(out.shape) != tuple(q.shape)
            or not out.is_contiguous()):
        raise ValueError("out must be a contiguous BF16 tensor shaped like Q on its device")
    return out


def sol_attention(q, k, v, *, beta=1.0, scale=None, local_blocks=1,
                  kv_sink_tokens=0, query_sink_tokens=0, return_stats=False):
    """SOL-style noncausal attention; no semantic mask support (``attention.py:58-85``).

    Physical blocks contain 64 tokens. Selected blocks use BF16 QK/PV with FP32
    softmax/accumulation; other blocks contribute pooled-key/value correction.
    Thresholds use the diagonal-covariance estimator (paper Eq. 15).
    Prefix protection rounds OUTWARD to whole blocks. beta=-inf forces dense;
    beta=+inf leaves only protected blocks exact.
    """
    scale = _validate(q, k, v, scale)
    beta = float(beta)
    if math.isnan(beta):
        raise ValueError("beta must not be NaN")
    for name, value in (("local_blocks", local_blocks),
                        ("kv_sink_tokens", kv_sink_tokens),
                        ("query_sink_tokens", query_sink_tokens)):
        _nonnegative_integer(name, value)
    if kv_sink_tokens > k.shape[1] or query_sink_tokens > q.shape[1]:
        raise ValueError("Sink token counts must not exceed their sequence lengths")
    with torch.no_grad(), torch.cuda.device(q.device):
        out, counts = launch_sol(q, k, v, scale, beta, local_blocks,
                                 kv_sink_tokens, query_sink_tokens, return_stats)
    if return_stats:
        return out, SolStats(counts, (k.shape[1] + 63) // 64)
    return out
