"""The host-buffer entry point ``sol_attention_host`` (no counterpart in the reference): head
groups streamed through the GPU with overlapped copies must give exactly ``sol_attention``'s
output on the same inputs, for strided host views, odd head groupings and stats."""

import math

import pytest
import torch

from helpers import to_device
from sol_attn_b200 import sol_attention, sol_attention_host, workloads


def test_host_api_rejects_device_tensors_and_bad_arguments():
    q = torch.zeros((1, 64, 2, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="host"):
        sol_attention_host(q.to("meta"), q, q)
    with pytest.raises(ValueError, match="Only BF16"):
        sol_attention_host(q.float(), q, q)
    with pytest.raises(ValueError, match="beta"):
        sol_attention_host(q, q, q, beta=math.nan)
    with pytest.raises(ValueError, match="Sink"):
        sol_attention_host(q, q, q, kv_sink_tokens=65)
    with pytest.raises(ValueError, match="contiguous heads"):
        sol_attention_host(q.transpose(1, 2).contiguous().transpose(1, 2), q, q)


@pytest.mark.gpu
@pytest.mark.parametrize("heads_per_group", [None, 3, 1])
def test_host_api_matches_device_api(heads_per_group):
    # packed [B, T, 3, H, D] host buffer: q/k/v are strided views of it
    B, T, H, D = 2, 1000, 7, 64
    g = torch.Generator().manual_seed(3)
    buf = torch.randn((B, T, 3, H, D), generator=g).to(torch.bfloat16).pin_memory()
    q, k, v = buf[:, :, 0], buf[:, :, 1], buf[:, :, 2]
    kw = dict(beta=0.5, local_blocks=1, kv_sink_tokens=64, query_sink_tokens=64)
    out_h, st_h = sol_attention_host(q, k, v, heads_per_group=heads_per_group, return_stats=True, **kw)
    out_d, st_d = sol_attention(*(to_device(x) for x in (q, k, v)), return_stats=True, **kw)
    assert out_h.device.type == "cpu"
    assert torch.equal(out_h, out_d.cpu())
    assert torch.equal(st_h.exact_blocks.cpu(), st_d.exact_blocks.cpu())


@pytest.mark.gpu
def test_host_api_into_preallocated_strided_output():
    q, k, v = workloads.iid((1, 2048, 8, 128), seed=5)
    q, k, v = (x.pin_memory() for x in (q, k, v))
    out = torch.full((1, 2048, 2, 8, 128), 7.0, dtype=torch.bfloat16).pin_memory()[:, :, 1]
    res = sol_attention_host(q, k, v, out=out, beta=1.0)
    assert res.data_ptr() == out.data_ptr()
    ref = sol_attention(*(to_device(x) for x in (q, k, v)), beta=1.0)
    assert torch.equal(out, ref.cpu())
