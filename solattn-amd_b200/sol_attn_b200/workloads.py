"""Seeded synthetic inputs for the benchmark configurations and the parity tests.

Every generator draws on a CPU ``torch.Generator`` in a fixed order (Q, then K,
then V) so that the GPU path and the CPU oracle see identical bits. None of
these are captured model activations; the shapes and value distributions are
those of the reference's benchmark fixtures
(``benchmarks/bench_attention.py:35-45``) and of the configurations this
package is measured on:

* ``plumbing``      B=1, T=1024, H=4, D=64, i.i.d. N(0,1), seed 0.
* ``block_smooth``  per (64-token block, head) base ~ N(0,1), token = base + sigma*N(0,1).
* ``video_dit``     base_0 ~ N(0,1), base_b = 0.9*base_{b-1} + 0.44*N(0,1) along blocks,
                    token = base + 0.3*N(0,1).
* ``ragged_cross``  one packed [B, T, 3, H, D] N(0,1) buffer; q = buf[:, :, 0],
                    k = buf[:, :Tk, 1], v = buf[:, :Tk, 2] (non-contiguous views).
* ``indexed_windows`` the window plan rows/keys of the indexed configuration.
"""

from __future__ import annotations

import torch

BLOCK = 64


def reference_fixture(nq=193, nk=317, d=64, b=1, h=2, strided=False, seed=42):
    """The reference test fixture (``tests/test_attention.py:13-17``) on CPU."""
    gen = torch.Generator().manual_seed(seed)
    xs = [torch.randn((b, n, h * (2 if strided else 1), d), generator=gen,
                      dtype=torch.bfloat16) for n in (nq, nk, nk)]
    return tuple(x[:, :, ::2] if strided else x for x in xs)


def iid(shape, seed=0, n=3):
    gen = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(shape, generator=gen, dtype=torch.bfloat16) for _ in range(n))


def _smooth(shape, gen, sigma, drift):
    b, t, h, d = shape
    nb = (t + BLOCK - 1) // BLOCK
    base = torch.randn((b, nb, h, d), generator=gen, dtype=torch.float32)
    if drift:
        for i in range(1, nb):
            base[:, i] = 0.9 * base[:, i - 1] + 0.44 * base[:, i]
    noise = torch.randn(shape, generator=gen, dtype=torch.float32)
    x = base.repeat_interleave(BLOCK, dim=1)[:, :t] + sigma * noise
    return x.to(torch.bfloat16)


def block_smooth(b=1, t=4096, h=16, d=128, sigma=0.1, seed=0):
    gen = torch.Generator().manual_seed(seed)
    return tuple(_smooth((b, t, h, d), gen, sigma, False) for _ in range(3))


def video_dit(b=1, t=32768, h=24, d=128, sigma=0.3, seed=0):
    gen = torch.Generator().manual_seed(seed)
    return tuple(_smooth((b, t, h, d), gen, sigma, True) for _ in range(3))


def ragged_cross(b=2, tq=8192, tk=5000, h=16, d=64, seed=0):
    gen = torch.Generator().manual_seed(seed)
    buf = torch.randn((b, tq, 3, h, d), generator=gen, dtype=torch.bfloat16)
    return buf[:, :, 0], buf[:, :tk, 1], buf[:, :tk, 2]


def indexed_windows(seq_len=32768, window=512, halo=1024, anchor=256, stride=8):
    """Rows and allowed keys of each query window of the indexed configuration.

    Window w owns rows [w*window, (w+1)*window). Its allowed keys are the
    sorted union of the anchor range [0, anchor), its own window widened by
    ``halo`` tokens on both sides, and every ``stride``-th key elsewhere.
    Returns a list of (rows, keys) int64 CPU vectors, one per window.
    """
    out = []
    strided = torch.arange(0, seq_len, stride)
    for s in range(0, seq_len, window):
        e = min(seq_len, s + window)
        rows = torch.arange(s, e)
        keys = torch.cat((torch.arange(0, anchor),
                          torch.arange(max(0, s - halo), min(seq_len, e + halo)), strided))
        out.append((rows, torch.unique(keys)))
    return out


def group_windows(windows):
    """Group windows with equal (query, key) counts into rectangular plans.

    Returns a list of (window_ids, rows [W, nq], keys [W, nk]) in order of
    first appearance, since ``IndexedPlan`` is rectangular
    (``indexed.py:11-66``).
    """
    groups = {}
    for i, (rows, keys) in enumerate(windows):
        groups.setdefault((rows.numel(), keys.numel()), []).append(i)
    return [(ids, torch.stack([windows[i][0] for i in ids]), torch.stack([windows[i][1] for i in ids]))
            for ids in groups.values()]
