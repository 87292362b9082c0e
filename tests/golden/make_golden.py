"""Generate golden fixtures from the reference's own FP32 oracle.

Run in a container that has the reference source tree (it is not present on
GPU boxes)::

    python tests/golden/make_golden.py --reference-src <path to reference>/src

The reference oracle ``sol_attn_amd.reference.sol_reference``
(``src/sol_attn_amd/reference.py:19-66``) is imported from that tree and run on
seeded inputs drawn by ``sol_attn_b200.workloads``; its outputs are stored as
compressed ``.npz`` next to this script together with a SHA-256 of the input
bytes, so that tests can regenerate the inputs from the seed and prove they
are the same. Large outputs are stored on a fixed row subsample only.
"""

from __future__ import annotations

import argparse
import hashlib
import math
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1] / "solattn-amd_b200"))

from sol_attn_b200 import workloads  # noqa: E402
from sol_attn_b200.indexed import build_protection  # noqa: E402

INF = math.inf


def digest(*xs):
    h = hashlib.sha256()
    for x in xs:
        h.update(x.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def subsample(t, every):
    """Token rows kept for large outputs: 0, every, 2*every, ... and the last row."""
    idx = list(range(0, t, every))
    if idx[-1] != t - 1:
        idx.append(t - 1)
    return np.asarray(idx, dtype=np.int64)


def save(name, **arrays):
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    size = (HERE / f"{name}.npz").stat().st_size
    print(f"{name}: {size / 1024:.0f} KiB", flush=True)


def bthd_cases():
    """(name, input factory, kwargs of sol_reference, row subsample step or None)."""
    cases = [("c1_plumbing", lambda: workloads.iid((1, 1024, 4, 64), seed=0),
              dict(beta=1.0, kv_sink_tokens=128, query_sink_tokens=128, local_blocks=1), None)]
    for d in (64, 128):
        for strided in (False, True):
            for beta, tag in ((-INF, "minf"), (INF, "pinf"), (1.0, "b1")):
                cases.append((f"ragged_d{d}_{'strided' if strided else 'dense'}_{tag}",
                              lambda d=d, s=strided: workloads.reference_fixture(d=d, b=2, strided=s),
                              dict(beta=beta), None))
    cases.append(("zero_sinks", lambda: tuple(x.zero_() if i < 2 else x for i, x in
                                              enumerate(workloads.reference_fixture())),
                  dict(beta=INF, local_blocks=0, kv_sink_tokens=65, query_sink_tokens=1), None))
    cases.append(("prefix_rounding", lambda: workloads.reference_fixture(),
                  dict(beta=INF, kv_sink_tokens=65, query_sink_tokens=1, local_blocks=0), None))
    for beta, tag in ((-INF, "minf"), (INF, "pinf"), (1.0, "b1")):
        cases.append((f"groups_tail_{tag}", lambda: workloads.reference_fixture(nq=1025, nk=1089, h=1),
                      dict(beta=beta), None))
    cases.append(("no_exact_rows", lambda: workloads.reference_fixture(nq=321, nk=65, h=1),
                  dict(beta=INF, local_blocks=0), None))
    cases.append(("single_token", lambda: workloads.reference_fixture(nq=1, nk=1), dict(beta=1.0), None))
    cases.append(("beta0_subsetq", lambda: (lambda g: (
        torch.randn((1, 129, 1, 64), generator=g, dtype=torch.bfloat16),
        torch.randn((1, 205, 1, 64), generator=g, dtype=torch.bfloat16),
        torch.randn((1, 205, 1, 64), generator=g, dtype=torch.bfloat16)))(torch.Generator().manual_seed(7)),
        dict(beta=0.0), None))
    for beta, tag in ((1.0, "b1"), (-INF, "minf"), (INF, "pinf")):
        cases.append((f"c2_block_smooth_{tag}", lambda: workloads.block_smooth(),
                      dict(beta=beta, kv_sink_tokens=128, query_sink_tokens=128, local_blocks=1), 97))
    cases.append(("c4_ragged_cross", lambda: workloads.ragged_cross(),
                  dict(beta=1.0, kv_sink_tokens=64, query_sink_tokens=0, local_blocks=0), 127))
    return cases


def indexed_cases():
    """The reference indexed test fixture (``tests/test_indexed.py:59-76``) for three betas."""
    g = torch.Generator().manual_seed(719)
    cpu = [torch.randn((1200, 4, 128), generator=g, dtype=torch.bfloat16)[:, ::2] for _ in range(3)]
    rows = torch.stack((torch.arange(231, 361), torch.arange(901, 1031)))
    keys = torch.stack((torch.cat((torch.arange(7), torch.arange(191, 703), torch.arange(1180, 1193))),
                        torch.cat((torch.arange(7), torch.arange(661, 1173), torch.arange(1180, 1193)))))
    return cpu, rows, keys


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    from sol_attn_amd.reference import sol_reference
    from sol_attn_amd.indexed import IndexedPlan
    torch.set_num_threads(8)

    for name, make, kw, every in bthd_cases():
        if args.only and args.only not in name:
            continue
        q, k, v = make()
        t0 = time.time()
        out, counts = sol_reference(q, k, v, **kw)
        arrays = dict(counts=counts.numpy(), sha256=np.array(digest(q, k, v)),
                      beta=np.float64(kw.get("beta", 1.0)))
        if every is None:
            arrays["out"] = out.numpy()
        else:
            idx = subsample(q.shape[1], every)
            arrays["rows"] = idx
            arrays["out_rows"] = out[:, idx].numpy()
        if name == "beta0_subsetq":
            part, pc = sol_reference(q, k, v, query_blocks=[0, 2], **kw)
            arrays["subset_out"] = part.numpy()
            arrays["subset_counts"] = pc.numpy()
        save(name, **arrays)
        print(f"  {time.time() - t0:.1f}s", flush=True)

    cpu, rows, keys = indexed_cases()
    plan = IndexedPlan.create(rows, keys, 1200, protected_ranges=((0, 7), (1180, 1193)), local_tokens=64)
    mine = build_protection(rows, keys, 1200, ((0, 7), (1180, 1193)), 64)
    assert torch.equal(plan.protected_blocks, mine)
    for beta, tag in ((-INF, "minf"), (INF, "pinf"), (1.0, "b1")):
        ref, counts = sol_reference(cpu[0][rows], cpu[1][keys], cpu[2][keys], beta=beta,
                                    local_blocks=-1, protected_blocks=plan.protected_blocks)
        save(f"indexed_{tag}", out=ref.numpy(), counts=counts.numpy(),
             protected=plan.protected_blocks.numpy(), sha256=np.array(digest(*cpu)))

    # Protection matrices of the reference's plan builder on the indexed configuration.
    wins = workloads.indexed_windows()
    prot = {}
    for ids, r, kk in workloads.group_windows(wins):
        p = IndexedPlan.create(r, kk, 32768, protected_ranges=((0, 256),), local_tokens=64)
        prot[f"w{ids[0]}_n{kk.shape[1]}"] = p.protected_blocks[:4].numpy()
    save("c5_protection", **prot)


if __name__ == "__main__":
    main()
