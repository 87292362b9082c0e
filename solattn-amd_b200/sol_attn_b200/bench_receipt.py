"""All-in benchmark receipt in the reference's JSON shape (``benchmarks/bench_attention.py``).

Times torch SDPA, this package's ``dense_attention`` and ``sol_attention`` on the reference's
own synthetic fixtures (same flags, same input recipe, same rotation of the timing order, same
fields per case), so that a B200 receipt can be set beside the reference's published R9700
receipts (``docs/benchmarks/r9700-synthetic-*.json``).  Synthetic inputs are never
model-quality evidence.

    python -m sol_attn_b200.bench_receipt --tokens 1024 4096 8192 --out receipt.json
"""

import argparse
import hashlib
import json
import math
import os
import statistics
import time
from pathlib import Path

import torch
import torch.nn.functional as F

from . import dense_attention, sol_attention


def _samples(fn, repeats):
    """One trial: the mean of ``repeats`` back-to-back calls, timed with CUDA events."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(repeats):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / repeats


def make_inputs(tokens, heads, dimension, seed, kind):
    """The reference fixture (``bench_attention.py:35-45``): BTHD BF16 N(0,1) from a CUDA
    generator; "block-smooth" replaces each tensor by per-64-token-block centres plus 0.05
    times the noise."""
    generator = torch.Generator(device="cuda").manual_seed(seed)

    def rand(shape):
        return torch.randn(shape, device="cuda", dtype=torch.bfloat16, generator=generator)

    q, k, v = [rand((1, tokens, heads, dimension)) for _ in range(3)]
    if kind == "block-smooth":
        for x in (q, k, v):
            centres = rand((1, (tokens + 63) // 64, heads, dimension))
            x.copy_(centres.repeat_interleave(64, dim=1)[:, :tokens] + 0.05 * x)
    return q, k, v


def _source_hashes():
    pkg = Path(__file__).resolve().parent
    files = sorted(pkg.glob("*.py")) + sorted((pkg.parent / "csrc").glob("*.cu*"))
    root = pkg.parent
    return {str(p.relative_to(root)): hashlib.sha256(p.read_bytes()).hexdigest() for p in files}


def run_case(n, args):
    q, k, v = make_inputs(n, args.heads, args.head_dim, args.seed, args.input)

    def sdpa():
        return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                              v.transpose(1, 2)).transpose(1, 2)

    functions = {"torch_sdpa_auto": sdpa,
                 "project_dense": lambda: dense_attention(q, k, v),
                 "sol_all_in": lambda: sol_attention(q, k, v, beta=args.beta)}
    for fn in functions.values():  # warm-up
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    samples = {name: [] for name in functions}
    names = list(functions)
    for trial in range(args.trials):  # rotate the order between trials
        for name in names[trial % len(names):] + names[:trial % len(names)]:
            samples[name].append(_samples(functions[name], args.repeats))
    timings = {name: {"median_ms": statistics.median(xs), "samples_ms": xs, "min_ms": min(xs),
                      "max_ms": max(xs),
                      "cv_percent": statistics.pstdev(xs) / statistics.mean(xs) * 100}
               for name, xs in samples.items()}
    actual, stats = sol_attention(q, k, v, beta=args.beta, return_stats=True)
    reference = sdpa().float()
    delta = actual.float() - reference
    return {"shape": list(q.shape), "timings": timings, "exact_block_density": stats.density(),
            "finite": bool(torch.isfinite(actual).all()),
            "relative_l2_vs_sdpa": (delta.norm() / reference.norm().clamp_min(1e-8)).item(),
            "max_abs_vs_sdpa": delta.abs().max().item(),
            "cosine_vs_sdpa": F.cosine_similarity(actual.float().flatten(), reference.flatten(),
                                                  dim=0).item(),
            "speedup_vs_sdpa": timings["torch_sdpa_auto"]["median_ms"]
            / timings["sol_all_in"]["median_ms"],
            "speedup_vs_project_dense": timings["project_dense"]["median_ms"]
            / timings["sol_all_in"]["median_ms"]}


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--tokens", type=int, nargs="+", default=[1024, 4096])
    parser.add_argument("--heads", type=int, default=4)
    parser.add_argument("--head-dim", type=int, choices=[64, 128], default=128)
    parser.add_argument("--beta", type=float, default=1.0)
    parser.add_argument("--input", choices=["random", "block-smooth"], default="block-smooth")
    parser.add_argument("--seed", type=int, default=42)
    parser.add_argument("--repeats", type=int, default=5)
    parser.add_argument("--trials", type=int, default=5)
    parser.add_argument("--out", type=Path, required=True)
    args = parser.parse_args(argv)
    if min(*args.tokens, args.heads, args.repeats, args.trials) <= 0:
        parser.error("shape and repetition counts must be positive")
    if not math.isfinite(args.beta):
        parser.error("Benchmark beta must be finite; dense-limit cases are covered by tests")
    if args.out.exists():
        parser.error("Use a new output path to preserve experiment receipts")
    device = torch.cuda.get_device_properties(0)
    report = {"state": "running",
              "scope": "All-in GPU-event latency, warm; synthetic data only",
              "started_unix": time.time(), "torch": torch.__version__, "hip": None,
              "cuda": torch.version.cuda, "triton": None, "device": str(device),
              "gpu_uuid": os.environ.get("CUDA_VISIBLE_DEVICES"), "image": None,
              "configuration": {**vars(args), "out": str(args.out)},
              "threshold_estimator": "diagonal_covariance", "source_sha256": _source_hashes(),
              "cases": []}
    args.out.parent.mkdir(parents=True, exist_ok=True)

    def save():
        args.out.write_text(json.dumps(report, indent=2, allow_nan=False) + "\n")

    save()
    try:
        for n in args.tokens:
            case = run_case(n, args)
            report["cases"].append(case)
            save()
            print(json.dumps(case), flush=True)
        report["state"] = "complete"
        save()
    except Exception as exc:
        report.update(state="failed", error=repr(exc))
        save()
        raise


if __name__ == "__main__":
    main()
