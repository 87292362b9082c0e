"""Host-side API contract (``src/sol_attn_amd/attention.py:19-85``) without a GPU."""

import math

import pytest
import torch

from sol_attn_b200 import dense_attention, sol_attention, sol_attention_indexed, IndexedPlan
from sol_attn_b200 import workloads


def test_api_rejects_unsupported_input():
    """``tests/test_attention.py:149-156`` with the device message re-targeted to B200."""
    q, k, v = workloads.reference_fixture()
    with pytest.raises(ValueError, match="B200"):
        sol_attention(q, k, v)
    with pytest.raises(ValueError, match="Only BF16"):
        sol_attention(q.float(), k.float(), v.float())
    with pytest.raises(ValueError, match="Inference only"):
        sol_attention(q.clone().requires_grad_(), k, v)
    with pytest.raises(ValueError, match="B200"):
        dense_attention(q, k, v)


@pytest.mark.parametrize("shape_fix,msg", [
    (lambda q, k, v: (q[0], k, v), "rank-4"),
    (lambda q, k, v: (q, k[:, :10], v), "shapes must agree"),
    (lambda q, k, v: (q[..., :32], k[..., :32], v[..., :32]), "head dimensions"),
    (lambda q, k, v: (q.transpose(2, 3).contiguous().transpose(2, 3), k, v), "contiguous head"),
])
def test_api_rejects_bad_layouts(shape_fix, msg):
    q, k, v = workloads.reference_fixture()
    with pytest.raises(ValueError, match=msg):
        sol_attention(*shape_fix(q, k, v))


def test_api_rejects_masks_by_signature():
    q, k, v = workloads.reference_fixture()
    with pytest.raises(TypeError):
        sol_attention(q, k, v, attn_mask=torch.ones((193, 317)))


def test_indexed_api_validation_order():
    q = torch.zeros((20, 2, 64), dtype=torch.bfloat16)
    plan = IndexedPlan.create(torch.tensor([[1, 2]]), torch.arange(8).reshape(1, -1), 20)
    with pytest.raises(ValueError, match="matching NHD"):
        sol_attention_indexed(q, q[:10], q, plan)
    with pytest.raises(ValueError, match="B200"):
        sol_attention_indexed(q, q, q, plan)


def test_sink_and_beta_validation_is_reached_only_on_device():
    # On CPU the device check fires first, exactly like the reference's ordering.
    q, k, v = workloads.reference_fixture()
    with pytest.raises(ValueError):
        sol_attention(q, k, v, beta=math.nan)


def test_scatter_and_dense_rows_reject_bad_arguments_on_cpu():
    from sol_attn_b200 import dense_attention_rows
    q = torch.zeros((100, 2, 64), dtype=torch.bfloat16)
    rows = torch.arange(10)
    with pytest.raises(ValueError, match="B200"):
        dense_attention_rows(q, q, q, rows)
    with pytest.raises(ValueError, match="NHD"):
        dense_attention_rows(q, q[:50], q, rows)
    plan = IndexedPlan.create(torch.arange(64)[None], torch.arange(64)[None], 100)
    with pytest.raises(ValueError, match="B200"):
        sol_attention_indexed(q, q, q, plan, out=torch.zeros_like(q))


def test_bench_receipt_rejects_bad_runs_before_touching_the_gpu(tmp_path):
    """Receipts are comparable only for finite beta and positive counts, and a receipt that
    exists is never replaced (the reference keeps the same guards,
    ``benchmarks/bench_attention.py:61-66``); all of it is checked before any GPU work."""
    from sol_attn_b200 import bench_receipt
    out = tmp_path / "r.json"
    with pytest.raises(SystemExit):
        bench_receipt.main([str(out), "--beta", "inf"])
    with pytest.raises(SystemExit):
        bench_receipt.main([str(out), "--tokens", "0"])
    out.write_text("{}")
    with pytest.raises(SystemExit):
        bench_receipt.main([str(out)])
    assert out.read_text() == "{}"


def test_launch_counts_of_the_two_paths():
    """The kernels one call launches (the bench's gpu_launches): the public call folds the
    threshold into pooling and routing on the tcgen05 path; the stage path launches it apart;
    beyond 4096 key blocks the mma.sync kernel routes for itself."""
    from sol_attn_b200.stages import Stages
    q, k, v = (torch.zeros((1, 4096, 2, 64), dtype=torch.bfloat16) for _ in range(3))
    st = Stages(q, k, v, beta=1.0)
    assert (st.launches(), st.public_launches()) == (4, 3)
    st = Stages(q, k, v, beta=math.inf)
    assert (st.launches(), st.public_launches()) == (3, 3)
    t = 64 * 4097
    q, k, v = (torch.zeros((1, t, 1, 64), dtype=torch.bfloat16) for _ in range(3))
    st = Stages(q, k, v, beta=1.0)
    assert (st.launches(), st.public_launches()) == (3, 3)
