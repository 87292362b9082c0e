"""Device-side error reporting of the public calls, without a host synchronisation per call.

The kernels record errors that only the device can see - a bounded wait that ran out, a gather
or scatter index outside its tensor, a ragged key count outside [1, Tk] - in an int32 status
word (first error wins).  After every public call the Python layer enqueues, on the call's
stream, an asynchronous copy of that word into a slot of pinned host memory
(``solattn_status_to_host``) and records an event behind it; nothing blocks.  The words are
looked at

* at the start of the next public call on the same device: every slot whose event has
  completed is read, and a nonzero word raises :class:`DeviceError`;
* in ``SolStats.density()`` and :func:`check_device_errors`, which wait for every pending slot
  (both synchronise anyway).

So an error surfaces at the latest on the next call or the next synchronising read, and a
production call pays one 4-byte device-to-host copy, never a synchronisation.  The reference's
kernels report nothing of the kind; this is the negative-code path of the C ABI
(``SOLATTN_ERR_DEVICE``) carried through to Python.
"""

from __future__ import annotations

import collections
import threading

import torch

from . import _lib

# Device-side codes (csrc/common.cuh kStatus*).
CODES = {1: "a bounded wait inside a kernel ran out", 2: "an index outside its tensor",
         3: "TMEM allocation returned an unusable address",
         4: "a TMA tile coordinate outside its tensor"}


class DeviceError(_lib.SolAttnError):
    """A kernel of an earlier call reported a device-side error (its output is not valid)."""

    def __init__(self, code: int):
        self.code = code
        super().__init__(f"a previous SOL attention call on this device reported device-side "
                         f"status {code} ({CODES.get(code, 'unknown')}); its output is invalid")


class StatusMonitor:
    """Pending status copies of one device: a ring of pinned int32 slots and their events."""

    SLOTS = 256

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.host = torch.zeros(self.SLOTS, dtype=torch.int32).pin_memory()
        self.words = self.host.numpy()  # the same pinned memory, read without torch indexing
        self.host_ptr = self.host.data_ptr()
        self.events = [None] * self.SLOTS  # created on first use, then recorded again
        self.pending = collections.deque()
        self.next = 0
        self.lock = threading.Lock()

    def record(self, status_ptr: int, stream: torch.cuda.Stream) -> None:
        """Enqueue the copy of the device word at ``status_ptr`` on ``stream``.  A slot is
        read only after its event completed, i.e. after the copy has overwritten it."""
        with self.lock:
            if len(self.pending) == self.SLOTS:  # every slot in flight: wait for the oldest
                self._take(wait=True, limit=1)
            slot = self.next
            self.next = (slot + 1) % self.SLOTS
            rc = _lib.load().solattn_status_to_host(status_ptr, self.host_ptr + 4 * slot,
                                                    stream.cuda_stream)
            _lib.check(rc, "solattn_status_to_host")
            event = self.events[slot]
            if event is None:
                event = self.events[slot] = torch.cuda.Event()
            event.record(stream)
            self.pending.append(slot)

    def poll(self, wait: bool) -> None:
        """Read the completed slots (every pending slot when ``wait``); raise on a nonzero word."""
        with self.lock:
            self._take(wait=wait, limit=None)

    def _take(self, wait: bool, limit) -> None:
        first_error = 0
        taken = 0
        while self.pending and (limit is None or taken < limit):
            slot = self.pending[0]
            event = self.events[slot]
            if not wait and not event.query():
                break
            event.synchronize()
            value = int(self.words[slot])
            self.pending.popleft()
            taken += 1
            if value and not first_error:
                first_error = value
        if first_error:
            raise DeviceError(first_error)


_MONITORS: dict = {}
_MONITORS_LOCK = threading.Lock()


def monitor(device: torch.device) -> StatusMonitor:
    index = device.index if device.index is not None else torch.cuda.current_device()
    with _MONITORS_LOCK:
        if index not in _MONITORS:
            _MONITORS[index] = StatusMonitor(index)
        return _MONITORS[index]


def check_device_errors(device=None) -> None:
    """Wait for every pending status copy (of ``device``, or of every device used) and raise
    :class:`DeviceError` if a call reported a device-side error."""
    if device is not None:
        monitor(torch.device(device)).poll(wait=True)
        return
    for mon in list(_MONITORS.values()):
        mon.poll(wait=True)
