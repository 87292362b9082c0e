"""Latency receipts whose JSON fields match the reference's published receipts.

The reference publishes all-in latencies of its operator next to torch SDPA and its own dense
kernel as JSON receipts (``docs/benchmarks/r9700-synthetic-*.json``, written by
``benchmarks/bench_attention.py:70-113``).  This module produces a receipt with the same field
names for this package on a B200, so the two can be read side by side; the measurement itself is
this package's: inputs come from :mod:`sol_attn_b200.workloads` (seeded CPU generators, copied
to the GPU), every implementation is timed in every trial in a freshly shuffled order, and the
receipt file is written once, atomically, when the run ends (with ``"state": "failed"`` and the
error if it does not finish).  Synthetic inputs say nothing about model quality.

    python -m sol_attn_b200.bench_receipt receipt.json --tokens 1024 4096 8192 --heads 4
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import random
import statistics
import time
from pathlib import Path

import torch
import torch.nn.functional as F

from . import dense_attention, sol_attention, workloads

KINDS = ("block-smooth", "random")


def inputs(kind: str, tokens: int, heads: int, dim: int, seed: int):
    """BTHD BF16 Q/K/V on the GPU: block-smooth = per-64-token-block base vectors plus 0.05
    times N(0, 1) noise per token (the reference's smooth fixture's distribution), random =
    i.i.d. N(0, 1)."""
    if kind == "block-smooth":
        cpu = workloads.block_smooth(b=1, t=tokens, h=heads, d=dim, sigma=0.05, seed=seed)
    else:
        cpu = workloads.iid((1, tokens, heads, dim), seed=seed)
    return tuple(x.cuda() for x in cpu)


class EventTimer:
    """Mean device time of ``calls`` back-to-back calls of a function, by CUDA events."""

    def __init__(self, calls: int):
        self.calls = calls
        self.begin = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)

    def __call__(self, fn) -> float:
        self.begin.record()
        for _ in range(self.calls):
            fn()
        self.end.record()
        self.end.synchronize()
        return self.begin.elapsed_time(self.end) / self.calls


def summary(samples):
    mean = statistics.mean(samples)
    return {"median_ms": statistics.median(samples), "samples_ms": samples,
            "min_ms": min(samples), "max_ms": max(samples),
            "cv_percent": 100.0 * statistics.pstdev(samples) / mean if mean else 0.0}


def measure(kind, tokens, opts):
    q, k, v = inputs(kind, tokens, opts.heads, opts.dim, opts.seed)
    bhtd = lambda x: x.transpose(1, 2)  # noqa: E731
    impls = {
        "torch_sdpa_auto": lambda: F.scaled_dot_product_attention(bhtd(q), bhtd(k), bhtd(v)),
        "project_dense": lambda: dense_attention(q, k, v),
        "sol_all_in": lambda: sol_attention(q, k, v, beta=opts.beta),
    }
    for fn in impls.values():
        for _ in range(opts.warmup):
            fn()
    torch.cuda.synchronize()
    timer = EventTimer(opts.calls)
    order = random.Random(opts.seed)
    samples = {name: [] for name in impls}
    for _ in range(opts.trials):
        names = list(impls)
        order.shuffle(names)
        for name in names:
            samples[name].append(timer(impls[name]))
    timings = {name: summary(xs) for name, xs in samples.items()}
    out, stats = sol_attention(q, k, v, beta=opts.beta, return_stats=True)
    ref = bhtd(impls["torch_sdpa_auto"]()).float()
    diff = out.float() - ref
    sol_ms = timings["sol_all_in"]["median_ms"]
    return {"shape": list(q.shape), "timings": timings,
            "exact_block_density": stats.density(),
            "finite": bool(torch.isfinite(out).all()),
            "relative_l2_vs_sdpa": float(diff.norm() / ref.norm().clamp_min(1e-8)),
            "max_abs_vs_sdpa": float(diff.abs().max()),
            "cosine_vs_sdpa": float(F.cosine_similarity(out.float().flatten(), ref.flatten(), 0)),
            "speedup_vs_sdpa": timings["torch_sdpa_auto"]["median_ms"] / sol_ms,
            "speedup_vs_project_dense": timings["project_dense"]["median_ms"] / sol_ms}


def sources():
    """SHA-256 of the package's Python and CUDA sources (which build produced the receipt)."""
    pkg = Path(__file__).resolve().parent
    files = sorted(pkg.glob("*.py")) + sorted((pkg.parent / "csrc").glob("*.cu*"))
    return {p.name: hashlib.sha256(p.read_bytes()).hexdigest() for p in files}


def parse(argv):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("receipt", type=Path, help="new JSON file (an existing one is never replaced)")
    ap.add_argument("--tokens", type=int, nargs="+", default=[1024, 4096])
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--dim", type=int, choices=(64, 128), default=128)
    ap.add_argument("--input", choices=KINDS, default="block-smooth")
    ap.add_argument("--beta", type=float, default=1.0)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--calls", type=int, default=5, help="back-to-back calls per sample")
    ap.add_argument("--trials", type=int, default=5, help="samples per implementation")
    opts = ap.parse_args(argv)
    if not math.isfinite(opts.beta):
        ap.error("beta must be finite here (the force modes are covered by the tests)")
    if min(opts.tokens + [opts.heads, opts.warmup + 1, opts.calls, opts.trials]) <= 0:
        ap.error("token counts, heads, calls and trials must be positive")
    if opts.receipt.exists():
        ap.error(f"{opts.receipt} exists; receipts are kept, write a new one")
    return opts


def main(argv=None):
    opts = parse(argv)
    receipt = {"state": "running", "scope": "All-in GPU-event latency, warm; synthetic data only",
               "started_unix": time.time(), "torch": torch.__version__, "cuda": torch.version.cuda,
               "hip": None, "triton": None,
               "device": torch.cuda.get_device_name(0),
               "gpu_uuid": os.environ.get("CUDA_VISIBLE_DEVICES"),
               "configuration": {k: (str(v) if isinstance(v, Path) else v)
                                 for k, v in vars(opts).items()},
               "threshold_estimator": "diagonal_covariance", "source_sha256": sources(),
               "cases": []}
    try:
        for tokens in opts.tokens:
            case = measure(opts.input, tokens, opts)
            receipt["cases"].append(case)
            print(json.dumps({"shape": case["shape"],
                              "sol_ms": case["timings"]["sol_all_in"]["median_ms"]}), flush=True)
        receipt["state"] = "complete"
    except Exception as exc:
        receipt.update(state="failed", error=repr(exc))
        raise
    finally:
        opts.receipt.parent.mkdir(parents=True, exist_ok=True)
        tmp = opts.receipt.with_suffix(opts.receipt.suffix + ".tmp")
        tmp.write_text(json.dumps(receipt, indent=2, allow_nan=False) + "\n")
        os.replace(tmp, opts.receipt)


if __name__ == "__main__":
    main()
