"""Bit-exact CPU restatement of the pooled statistics and routing arithmetic of the CUDA
kernels (TEST INFRASTRUCTURE ONLY; see the header of ``sol_oracle.py`` for who may use it).

The reference (zihaomu/SolAttn-AMD) leaves the FP32 summation order of pooling, moments,
thresholds and the routing proxy to Triton/BLAS (``kernels.py:16-64, 129-135``;
``reference.py:13-15, 27-41``), so no implementation reproduces it bit for bit. The CUDA
kernels of this package fix one order and round every operation to nearest FP32 without
fused multiply-adds; this module restates that order in numpy float32 so tests can demand
bit identity:

* pooling (``solattn_pool_qkv``): 8 row groups, group g sums rows g, g+8, ..., g+56 of the
  block in order (rows past the ragged end skipped), the group sums are added in order
  g = 0..7, mean = sum / count; K/V means rounded to BF16 (nearest even);
* moments (``solattn_threshold``): eight slice sums per channel, slice j summing key blocks
  j, j+8, j+16, ... of x and x*x in order, combined as ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7));
  mean = s1/n, var = max(s2/n - mean*mean, 0);
* cutoff: eight partial sums over d = 8i + e (i increasing) of qc*mean and (qc*qc)*var,
  combined in the same tree; cutoff = (mu + beta*sqrt(sg)) * scale;
* routing (the routing pass): proxy = dot * scale where dot sums qc*kc as eight partial sums
  p_j over d = 8i + j (i increasing), each step one fused multiply-add
  p_j = fma(qc[d], kc[d], p_j) rounded once (``fma32``), combined as
  ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)); exact iff proxy > cutoff (force modes and the local /
  sink / protected rules as in ``reference.py:41-51``).

Routing decisions computed here from the GPU's own pooled statistics must equal the GPU's
bit for bit (the north-star routing criterion).
"""

from __future__ import annotations

import numpy as np
import torch

BLOCK = 64
F32 = np.float32


def _bf16_round(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()


def fma32(a, b, c) -> np.ndarray:
    """IEEE fusedMultiplyAdd in float32, a*b + c rounded once to nearest (ties to even),
    elementwise.  The product of two float32 values is exact in float64; the float64 sum s and
    its exact error e (Knuth's TwoSum) give a*b + c = s + e exactly, and rounding s to float32
    gives the correctly rounded result unless s lies exactly halfway between two float32
    values while e != 0 -- then the exact value lies on e's side of that midpoint."""
    a64 = np.asarray(a, F32).astype(np.float64)
    b64 = np.asarray(b, F32).astype(np.float64)
    c64 = np.asarray(c, F32).astype(np.float64)
    p = a64 * b64
    s = p + c64
    bb = s - p
    e = (p - (s - bb)) + (c64 - bb)
    r = s.astype(F32)
    r64 = r.astype(np.float64)
    d = s - r64  # exact: s and r are neighbours
    up = np.nextafter(r, F32(np.inf))
    dn = np.nextafter(r, F32(-np.inf))
    mid = ((d > 0) & (d == (up.astype(np.float64) - r64) / 2)) | \
          ((d < 0) & (-d == (r64 - dn.astype(np.float64)) / 2))
    away = mid & (e != 0) & (np.sign(e) == np.sign(d))
    return np.where(away, np.where(d > 0, up, dn), r).astype(F32)


def pool(x: torch.Tensor, out_bf16: bool) -> np.ndarray:
    """Block means of a BTHD tensor [B, T, H, D] -> [B, H, nb, D] float32 (BF16-rounded if asked)."""
    B, T, H, D = x.shape
    nb = (T + BLOCK - 1) // BLOCK
    pad = nb * BLOCK - T
    xf = x.float()
    if pad:
        xf = torch.cat((xf, torch.zeros((B, pad, H, D))), 1)
    a = xf.numpy().reshape(B, nb, BLOCK, H, D).transpose(0, 3, 1, 2, 4)  # [B,H,nb,64,D]
    total = np.zeros((B, H, nb, D), F32)
    for g in range(8):
        part = np.zeros((B, H, nb, D), F32)
        for i in range(8):
            part = part + a[:, :, :, g + 8 * i]  # zero rows past the end leave sums unchanged
        total = total + part
    counts = np.array([min(BLOCK, T - j * BLOCK) for j in range(nb)], F32)
    mean = total / counts[None, None, :, None]
    return _bf16_round(mean) if out_bf16 else mean.astype(F32)


def _tree8(p):
    """((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)) of eight float32 arrays."""
    return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]))


def moments(kc: np.ndarray):
    """kc [B, H, nkb, D] (BF16 values as float32) -> mean, var [B, H, D]."""
    nb = kc.shape[2]
    n = F32(nb)
    s1, s2 = [], []
    for j in range(8):
        a = np.zeros(kc.shape[:2] + kc.shape[3:], F32)
        b = np.zeros_like(a)
        for r in range(j, nb, 8):
            x = kc[:, :, r]
            a = a + x
            b = b + x * x
        s1.append(a)
        s2.append(b)
    mean = _tree8(s1) / n
    var = np.maximum(_tree8(s2) / n - mean * mean, F32(0))
    return mean, var


def cutoffs(qc: np.ndarray, mean: np.ndarray, var: np.ndarray, beta: float, scale: float):
    """qc [B, H, nqb, D] -> cutoff [B, H, nqb]."""
    D = qc.shape[3]
    mu, sg = [], []
    for e in range(8):
        a = np.zeros(qc.shape[:3], F32)
        b = np.zeros_like(a)
        for i in range(D // 8):
            d = 8 * i + e
            qv = qc[..., d]
            a = a + qv * mean[:, :, None, d]
            b = b + (qv * qv) * var[:, :, None, d]
        mu.append(a)
        sg.append(b)
    return (_tree8(mu) + F32(beta) * np.sqrt(_tree8(sg))) * F32(scale)


def route(qc, kc, cutoff, scale, force, local, kv_sink_blocks, q_sink_blocks, protect=None):
    """Exact-block selection [B, H, nqb, nkb] (bool) from pooled statistics."""
    B, H, nqb, D = qc.shape
    nkb = kc.shape[2]
    if force == 1:
        sel = np.ones((B, H, nqb, nkb), bool)
    elif force == 2:
        sel = np.zeros((B, H, nqb, nkb), bool)
    else:
        part = [np.zeros((B, H, nqb, nkb), F32) for _ in range(8)]
        for i in range(D // 8):
            for j in range(8):
                d = 8 * i + j
                part[j] = fma32(qc[:, :, :, None, d], kc[:, :, None, :, d], part[j])
        dot = ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]))
        sel = (dot * F32(scale)) > cutoff[..., None]
    qb = np.arange(nqb)[:, None]
    kb = np.arange(nkb)[None, :]
    forced = (kb < kv_sink_blocks) | (qb < q_sink_blocks)
    if local >= 0:
        forced = forced | (np.abs(kb - qb) <= local)
    sel = sel | forced[None, None]
    if protect is not None:
        sel = sel | np.asarray(protect, bool)[:, None]
    return sel


def pack_mask(sel: np.ndarray) -> np.ndarray:
    """bool [..., nkb] -> uint32 words [..., ceil(nkb/32)] (bit kb%32 of word kb//32)."""
    nkb = sel.shape[-1]
    nw = (nkb + 31) // 32
    padded = np.zeros(sel.shape[:-1] + (nw * 32,), bool)
    padded[..., :nkb] = sel
    bits = padded.reshape(sel.shape[:-1] + (nw, 32)).astype(np.uint64)
    return (bits << np.arange(32, dtype=np.uint64)).sum(-1).astype(np.uint32)
