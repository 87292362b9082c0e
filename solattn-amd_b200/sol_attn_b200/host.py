"""Host-resident inputs: SOL attention on BTHD tensors that live in (pinned) host memory.

The reference's API (``attention.py:58-85``) takes device tensors only; a caller whose Q/K/V sit
in host memory must copy them to the GPU first, then copy the output back.  Heads are
independent, so ``sol_attention_host`` streams them through the GPU in groups instead: while
group g is pooled, routed and attended to, the inputs of group g + 1 are on their way in and the
output of group g - 1 on its way out (three CUDA streams, two device slots).  The copies are
strided 2-D transfers straight between the host BTHD layout and contiguous device slices
(``solattn_copy_2d``), so nothing is repacked on the host.  Results equal ``sol_attention`` on
the same inputs bit for bit: every head is computed by the same kernels with the same routing
(the key moments, thresholds and selections of a head never involve another head).
"""

from __future__ import annotations

import math

import torch

from . import _lib
from .attention import BLOCK, SolStats, _nonnegative_integer

_H2D, _D2H = 0, 1
# Per-device pipeline resources (three streams), kept across calls so that buffers allocated on
# them are recycled by torch's caching allocator instead of being allocated anew each call.
_STREAMS = {}


def _streams(dev: torch.device):
    if dev.index not in _STREAMS:
        _STREAMS[dev.index] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    return _STREAMS[dev.index]


def _copy_heads(dst_ptr: int, dst_pitch: int, src_ptr: int, src_pitch: int, width: int,
                x_host: torch.Tensor, rows_per_batch: int, batch_stride: int, uniform: bool,
                direction: int, stream: int) -> None:
    """2-D copy of one head group for every batch item (one call when the rows are evenly
    spaced across batch items)."""
    L = _lib.load()
    B = x_host.shape[0]
    if uniform:
        rc = L.solattn_copy_2d(dst_ptr, dst_pitch, src_ptr, src_pitch, width, B * rows_per_batch,
                               direction, stream)
        _lib.check(rc, "solattn_copy_2d")
        return
    for b in range(B):
        if direction == _H2D:
            rc = L.solattn_copy_2d(dst_ptr + b * rows_per_batch * dst_pitch, dst_pitch,
                                   src_ptr + b * batch_stride, src_pitch, width, rows_per_batch,
                                   direction, stream)
        else:
            rc = L.solattn_copy_2d(dst_ptr + b * batch_stride, dst_pitch,
                                   src_ptr + b * rows_per_batch * src_pitch, src_pitch, width,
                                   rows_per_batch, direction, stream)
        _lib.check(rc, "solattn_copy_2d")


def sol_attention_host(q, k, v, *, beta=1.0, scale=None, local_blocks=1, kv_sink_tokens=0,
                       query_sink_tokens=0, return_stats=False, out=None, device=None,
                       heads_per_group=None):
    """``sol_attention`` on host BTHD tensors, returning a host BTHD output.

    q, k, v: CPU BF16 tensors [B, T, H, D] (pinned memory makes the copies asynchronous and
    overlapped with the compute) whose H*D values of a token are contiguous (strides
    [sB, sT, D, 1]; rows may be spaced, as in a packed QKV buffer).  ``out``: an optional
    preallocated CPU BF16 tensor of q's shape with the same rule (pinned for overlap).  ``device``: the
    B200 to use (default: the current CUDA device).  ``heads_per_group``: heads per pipeline
    stage (default: one head in the first and the last stage, whose copy-in and copy-out
    nothing overlaps, and about eleven equal stages in between).  Blocks until the output is
    in host memory.
    """
    for name, x in (("q", q), ("k", k), ("v", v)):
        if x.device.type != "cpu":
            raise ValueError(f"{name} must be a host (CPU) tensor")
    if any(x.ndim != 4 for x in (q, k, v)):
        raise ValueError("Q/K/V must have BTHD rank-4 layout")
    if any(x.dtype != torch.bfloat16 for x in (q, k, v)):
        raise ValueError("Only BF16 Q/K/V are implemented")
    if (k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[2:] != k.shape[2:]
            or any(n <= 0 for n in q.shape + k.shape)):
        raise ValueError("Q/K/V batch, head and dimension shapes must agree and be nonempty")
    if any(x.stride(-1) != 1 or x.stride(2) != x.shape[3] for x in (q, k, v)):
        raise ValueError("Q/K/V need contiguous heads within each row (strides [..., D, 1])")
    beta = float(beta)
    if math.isnan(beta):
        raise ValueError("beta must not be NaN")
    for name, val in (("local_blocks", local_blocks), ("kv_sink_tokens", kv_sink_tokens),
                      ("query_sink_tokens", query_sink_tokens)):
        _nonnegative_integer(name, val)
    if kv_sink_tokens > k.shape[1] or query_sink_tokens > q.shape[1]:
        raise ValueError("Sink token counts must not exceed their sequence lengths")
    B, Tq, H, D = q.shape
    Tk = k.shape[1]
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if out is None:
        out = torch.empty((B, Tq, H, D), dtype=torch.bfloat16).pin_memory()
    elif (out.shape != q.shape or out.dtype != torch.bfloat16 or out.device.type != "cpu"
          or out.stride(-1) != 1 or out.stride(2) != D):
        raise ValueError("out must be a CPU BF16 tensor of q's shape with contiguous heads "
                         "within each row")
    if heads_per_group is None:
        # Tapered: the first copy-in and the last copy-out overlap nothing, so the first and
        # last groups hold one head; about eleven groups in between keep the per-group launch
        # costs small against the copies.
        mid = max(1, -(-(H - 2) // 11)) if H >= 4 else 1
        sizes = [1] + [mid] * ((H - 2) // mid) + ([(H - 2) % mid] if (H - 2) % mid else []) + [1] \
            if H >= 4 else [1] * H
    else:
        hgi = int(heads_per_group)
        if hgi <= 0:
            raise ValueError("heads_per_group must be positive")
        sizes = [min(hgi, H - h0) for h0 in range(0, H, hgi)]
    groups, h0 = [], 0
    for n in sizes:
        groups.append((h0, h0 + n))
        h0 += n
    hg = max(sizes)
    nqb = (Tq + BLOCK - 1) // BLOCK
    from .attention import _validate, launch_sol  # noqa: PLC0415 (device-side checks)

    with torch.no_grad(), torch.cuda.device(dev):
        cur = torch.cuda.current_stream(dev)
        s_in, s_run, s_out = _streams(dev)
        for s in (s_in, s_run, s_out):
            s.wait_stream(cur)
        slots = []
        with torch.cuda.stream(s_in):  # the input slots are written on s_in and read on s_run
            for _ in range(2):
                slots.append(dict(
                    q=torch.empty((B, Tq, hg, D), dtype=torch.bfloat16, device=dev),
                    k=torch.empty((B, Tk, hg, D), dtype=torch.bfloat16, device=dev),
                    v=torch.empty((B, Tk, hg, D), dtype=torch.bfloat16, device=dev),
                    inputs_free=torch.cuda.Event(), loaded=torch.cuda.Event(),
                    computed=torch.cuda.Event(), out=None))
        for sl in slots:
            for n in ("q", "k", "v"):
                sl[n].record_stream(s_run)
        counts = torch.empty((B, nqb, H), dtype=torch.int32, device=dev) if return_stats else None
        for gi, (h0, h1) in enumerate(groups):
            sl = slots[gi % 2]
            hc = h1 - h0
            dq, dk, dv = (sl[n][:, :, :hc] for n in ("q", "k", "v"))
            # inputs of this slot are free once the group two steps back has been computed
            if gi >= 2:
                s_in.wait_event(sl["inputs_free"])
            with torch.cuda.stream(s_in):
                for dst, src, T in ((dq, q, Tq), (dk, k, Tk), (dv, v, Tk)):
                    uniform = src.stride(0) == T * src.stride(1)
                    _copy_heads(dst.data_ptr(), dst.stride(1) * 2, src[:, :, h0:h1].data_ptr(),
                                src.stride(1) * 2, hc * D * 2, src, T, src.stride(0) * 2, uniform,
                                _H2D, s_in.cuda_stream)
            sl["loaded"].record(s_in)
            s_run.wait_event(sl["loaded"])
            with torch.cuda.stream(s_run):
                _validate(dq, dk, dv, scale)
                o, c = launch_sol(dq, dk, dv, dq.shape[-1] ** -0.5 if scale is None else float(scale),
                                  beta, local_blocks, kv_sink_tokens, query_sink_tokens,
                                  return_stats)
                sl["out"] = o
                if return_stats:
                    counts[:, :, h0:h1].copy_(c)
            sl["computed"].record(s_run)
            sl["inputs_free"].record(s_run)
            s_out.wait_event(sl["computed"])
            with torch.cuda.stream(s_out):
                o = sl["out"]
                uniform = out.stride(0) == Tq * out.stride(1)
                _copy_heads(out[:, :, h0:h1].data_ptr(), out.stride(1) * 2, o.data_ptr(),
                            hc * D * 2, hc * D * 2, out, Tq, out.stride(0) * 2, uniform, _D2H,
                            s_out.cuda_stream)
                o.record_stream(s_out)  # the output buffer is reused only after its copy
        cur.wait_stream(s_out)
        s_out.synchronize()
    if return_stats:
        return out, SolStats(counts, (Tk + BLOCK - 1) // BLOCK)
    return out
