"""The full forward folds the threshold into the other launches (the pooling kernel computes each
head's key moments as its last K unit finishes, the routing pass forms the cutoffs): its key
moments, cutoffs, counts and outputs must equal, bit for bit, those of the stage-by-stage path,
which runs the threshold kernel (csrc/threshold.cu) between pooling and routing and whose
statistics are pinned to the CPU restatement (oracle/kernel_order.py) elsewhere."""

import ctypes

import numpy as np
import pytest
import torch

from helpers import CAbi, to_device
from make_golden import bthd_cases
from sol_attn_b200 import _lib, workloads

pytestmark = pytest.mark.gpu
CASES = {name: (make, kw) for name, make, kw, _ in bthd_cases()}


def _forward(q, k, v, *, beta, local, kv_sink_blocks, q_sink_blocks):
    """solattn_sol_forward on a workspace of our own, which is then read back."""
    L = _lib.load()
    B, Tq, H, D = q.shape
    Tk = k.shape[1]
    total, offs = _lib.workspace_layout(B, Tq, Tk, H, D)
    ws = torch.empty(total + 256, dtype=torch.uint8, device=q.device)
    base = (ws.data_ptr() + 255) // 256 * 256
    out = torch.empty((B, Tq, H, D), dtype=torch.bfloat16, device=q.device)
    nqb, nkb = (Tq + 63) // 64, (Tk + 63) // 64
    counts = torch.empty((B, nqb, H), dtype=torch.int32, device=q.device)
    st = [*q.stride()[:3], *k.stride()[:3], *v.stride()[:3]]
    rc = L.solattn_sol_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), B, Tq, Tk, H, D, *st,
                               None, None, 0, None, D ** -0.5, beta, local, kv_sink_blocks,
                               q_sink_blocks, ctypes.c_void_p(base), total, out.data_ptr(),
                               counts.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "solattn_sol_forward")
    torch.cuda.synchronize()
    skip = base - ws.data_ptr()

    def section(name, n, dtype):
        o = skip + offs[name]
        return ws[o:o + n * torch.empty((), dtype=dtype).element_size()].view(dtype)

    status = int(section("status", 1, torch.int32)[0])
    assert status == 0, status
    return dict(out=out, counts=counts, mean=section("mean", B * H * D, torch.float32),
                var=section("var", B * H * D, torch.float32),
                cut=section("cutoff", B * H * nqb, torch.float32))


@pytest.mark.parametrize("case,beta", [("c2_block_smooth_b1", 1.0), ("c2_block_smooth_b1", 0.5),
                                       ("c2_block_smooth_b1", 0.0), ("ragged_d64_strided_b1", 1.0),
                                       ("c4_ragged_cross", 0.5), ("groups_tail_b1", 1.5)])
def test_fused_threshold_equals_stage_path(case, beta):
    make, kw = CASES[case]
    q, k, v = (to_device(x) for x in make())
    args = dict(local=kw.get("local_blocks", 1),
                kv_sink_blocks=(kw.get("kv_sink_tokens", 0) + 63) // 64,
                q_sink_blocks=(kw.get("query_sink_tokens", 0) + 63) // 64)
    staged = CAbi().stages(q, k, v, beta=beta, **args)
    fused = _forward(q, k, v, beta=beta, **args)
    np.testing.assert_array_equal(fused["mean"].cpu().numpy(), staged["mean"].cpu().numpy().ravel())
    np.testing.assert_array_equal(fused["var"].cpu().numpy(), staged["var"].cpu().numpy().ravel())
    np.testing.assert_array_equal(fused["cut"].cpu().numpy(), staged["cut"].cpu().numpy().ravel())
    assert torch.equal(fused["counts"], staged["counts"])
    assert torch.equal(fused["out"], staged["out"])


def test_fused_threshold_headline_heads():
    """The bench workload's shape (T = 32768, 512 key blocks per head), three heads."""
    q, k, v = workloads.video_dit(b=1, t=32768, h=24, d=128, sigma=0.3, seed=0)
    q, k, v = (x[:, :, (0, 11, 23)].contiguous().cuda() for x in (q, k, v))
    args = dict(local=1, kv_sink_blocks=2, q_sink_blocks=2)
    staged = CAbi().stages(q, k, v, beta=1.0, **args)
    fused = _forward(q, k, v, beta=1.0, **args)
    np.testing.assert_array_equal(fused["cut"].cpu().numpy(), staged["cut"].cpu().numpy().ravel())
    assert torch.equal(fused["counts"], staged["counts"])
    assert torch.equal(fused["out"], staged["out"])
