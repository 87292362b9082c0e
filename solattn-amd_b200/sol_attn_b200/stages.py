"""Stage-by-stage driver of the C ABI (pool -> threshold -> attention) on preallocated buffers.

The public API (``sol_attention``) runs the three launches through ``solattn_sol_forward``.
This class issues them one by one so that benchmarks can time each kernel with CUDA events on
the launching stream and tests can read the intermediate pooled statistics and the kernel's
own routing bitmask.  Same arithmetic, same kernels.
"""

from __future__ import annotations

import math

import torch

from . import _lib

BLOCK = 64


class Stages:
    def __init__(self, q, k, v, *, beta, scale=None, local=1, kv_sink_blocks=0, q_sink_blocks=0,
                 protect=None, rows=None, keys=None, counts=True):
        self.L = _lib.load()
        self.indexed = rows is not None
        if self.indexed:
            B, Tq = rows.shape
            Tk = keys.shape[1]
            H, D = q.shape[1], q.shape[2]
        else:
            B, Tq, H, D = q.shape
            Tk = k.shape[1]
        self.q, self.k, self.v, self.rows, self.keys, self.protect = q, k, v, rows, keys, protect
        self.B, self.Tq, self.Tk, self.H, self.D = B, Tq, Tk, H, D
        self.scale = D ** -0.5 if scale is None else float(scale)
        self.beta = float(beta)
        self.force = 1 if beta == -math.inf else (2 if beta == math.inf else 0)
        self.local, self.kvs, self.qs = local, kv_sink_blocks, q_sink_blocks
        self.nqb, self.nkb = (Tq + BLOCK - 1) // BLOCK, (Tk + BLOCK - 1) // BLOCK
        dev = q.device
        f32, bf16 = torch.float32, torch.bfloat16
        self.qc = torch.zeros((B, H, self.nqb, D), dtype=f32, device=dev)
        self.kc = torch.zeros((B, H, self.nkb, D), dtype=bf16, device=dev)
        self.vc = torch.zeros_like(self.kc)
        self.mean = torch.zeros((B, H, D), dtype=f32, device=dev)
        self.var = torch.zeros_like(self.mean)
        self.cut = torch.zeros((B, H, self.nqb), dtype=f32, device=dev)
        self.status = torch.zeros(4, dtype=torch.int32, device=dev)
        self.out = torch.empty((B, Tq, H, D), dtype=bf16, device=dev)
        self.counts = torch.full((B, self.nqb, H), -1, dtype=torch.int32, device=dev) if counts else None
        # Routing decisions [B, H, nqb, ceil(nkb/32)] (bit kb % 32 of word kb / 32), written by
        # the attention call's routing pass, followed by the attention kernel's work counter and
        # the per-item tile lists (solattn_masks_bytes).
        nw = (self.nkb + 31) // 32
        nbytes = int(self.L.solattn_masks_bytes(B, Tq, Tk, H))
        self._mask_words = torch.zeros((nbytes + 3) // 4, dtype=torch.int32, device=dev)
        self.mask = self._mask_words[:B * H * self.nqb * nw].view(B, H, self.nqb, nw)

    def _strides(self, x):
        return (0, x.stride(0), x.stride(1)) if self.indexed else (x.stride(0), x.stride(1), x.stride(2))

    def _common(self):
        st = [*self._strides(self.q), *self._strides(self.k), *self._strides(self.v)]
        ridx = self.rows.data_ptr() if self.indexed else None
        kidx = self.keys.data_ptr() if self.indexed else None
        nrows = self.q.shape[0] if self.indexed else 0
        return st, ridx, kidx, nrows

    def pool(self, stream):
        st, ridx, kidx, nrows = self._common()
        rc = self.L.solattn_pool_qkv(self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                                     self.B, self.Tq, self.Tk, self.H, self.D, *st, ridx, kidx,
                                     nrows, int(self.force == 0), self.qc.data_ptr(),
                                     self.kc.data_ptr(), self.vc.data_ptr(),
                                     self.status.data_ptr(), stream)
        _lib.check(rc, "solattn_pool_qkv")

    def threshold(self, stream):
        if self.force != 0:
            return
        rc = self.L.solattn_threshold(self.kc.data_ptr(), self.qc.data_ptr(), self.B, self.H,
                                      self.nqb, self.nkb, self.D, self.scale, self.beta,
                                      self.mean.data_ptr(), self.var.data_ptr(),
                                      self.cut.data_ptr(), stream)
        _lib.check(rc, "solattn_threshold")

    def attention(self, stream):
        st, ridx, kidx, nrows = self._common()
        rc = self.L.solattn_attention(
            self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.B, self.Tq, self.Tk,
            self.H, self.D, *st, ridx, kidx, nrows, self.kc.data_ptr(), self.vc.data_ptr(),
            self.qc.data_ptr(), self.cut.data_ptr(),
            self.protect.data_ptr() if self.protect is not None else None, self.scale,
            self.force, self.local, self.kvs, self.qs, self.out.data_ptr(),
            self.counts.data_ptr() if self.counts is not None else None, self.status.data_ptr(),
            self.mask.data_ptr(), stream)
        _lib.check(rc, "solattn_attention")

    def run(self, stream=None):
        stream = torch.cuda.current_stream(self.q.device).cuda_stream if stream is None else stream
        self.pool(stream)
        self.threshold(stream)
        self.attention(stream)
        return self.out

    def launches(self) -> int:
        """Kernels one run() launches: pool, threshold (threshold mode only), the routing pass
        (tcgen05 path: at most 4096 key blocks) and the fused attention."""
        return 2 + (self.force == 0) + (self.nkb <= 4096)

    def public_launches(self) -> int:
        """Kernels one public call (solattn_sol_forward) launches for this problem: pooling, the
        routing pass and the fused attention on the tcgen05 path (the threshold is folded into
        the first two); with more than 4096 key blocks pooling, the threshold kernel (threshold
        mode only) and the mma.sync kernel."""
        if self.nkb <= 4096:
            return 3
        return 2 + (self.force == 0)
