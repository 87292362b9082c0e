"""Device-side errors surface on the public path without a per-call synchronisation.

Every public call copies its status word to pinned host memory asynchronously; the next call
on the device (or ``SolStats.density()``) raises ``DeviceError`` for a nonzero word.  No kernel
is made to fail here: the nonzero word is written by the host into the slot the call's copy
filled, which is what a kernel's report would have produced.
"""

import pytest
import torch

from helpers import to_device
from sol_attn_b200 import dense_attention, sol_attention, workloads
from sol_attn_b200.status import DeviceError, check_device_errors, monitor

pytestmark = pytest.mark.gpu


def _inject(code):
    """Wait for the last call's status copy, then overwrite the copied word with ``code``."""
    mon = monitor(torch.device("cuda", torch.cuda.current_device()))
    assert mon.pending, "the call recorded no status copy"
    slot = mon.pending[-1]
    mon.events[slot].synchronize()
    assert int(mon.host[slot]) == 0, "a real device-side error"
    mon.host[slot] = code


def test_clean_calls_raise_nothing():
    q, k, v = (to_device(x) for x in workloads.reference_fixture())
    for _ in range(3):
        sol_attention(q, k, v)
    dense_attention(q, k, v)
    check_device_errors()


def test_injected_status_raises_on_next_call():
    q, k, v = (to_device(x) for x in workloads.reference_fixture())
    sol_attention(q, k, v)
    _inject(2)  # kStatusBadIndex
    with pytest.raises(DeviceError, match="status 2"):
        sol_attention(q, k, v)
    sol_attention(q, k, v)  # the error was reported once; later calls are clean
    check_device_errors()


def test_injected_status_raises_in_density():
    q, k, v = (to_device(x) for x in workloads.reference_fixture())
    _, stats = sol_attention(q, k, v, return_stats=True)
    _inject(1)  # kStatusWaitTimeout
    with pytest.raises(DeviceError, match="status 1"):
        stats.density()
    assert 0.0 < stats.density() <= 1.0


def test_dense_status_is_monitored():
    q, k, v = (to_device(x) for x in workloads.reference_fixture())
    dense_attention(q, k, v)
    _inject(1)
    with pytest.raises(DeviceError):
        dense_attention(q, k, v)
    check_device_errors()
