"""Device status words of the ops, read without stalling the host.

The kernels OR data-dependent errors (an index outside ``[0, n)``, a key code
outside the codebook, a corrupt code->key index, a pipeline wait that gave
up) into a 32-bit status word on the device.  Reading that word right after
the launch would synchronise the host with the GPU after every op, so by
default (``SSA_CHECKED`` unset or ``1``) the word is read lazily:

* each op takes one word of a per-device ring (zeroed), passes it to the
  library, then enqueues on its stream a 4-byte copy of the word into pinned
  host memory, a reset of the word, and an event;
* every later op first looks at the oldest pending events without waiting
  (``Event.query``) and raises for the first word that came back non-zero;
* :func:`check_errors` waits for every pending word and raises.

An error therefore surfaces at the next op call after the GPU has finished
the failing one, or at :func:`check_errors`, never silently, and the host
never waits for the GPU on the fast path.  ``SSA_CHECKED=sync`` reads the
word right after each op (one host synchronisation per op, the error raised
by the failing call itself); ``SSA_CHECKED=0`` passes no status word at all.
Inside a CUDA graph capture no word is used.
"""

from __future__ import annotations

import collections
import os
import threading
from typing import Callable, Optional

import torch

from . import _lib as L

_SLOTS = 256


def mode() -> str:
    v = os.environ.get("SSA_CHECKED", "1").strip().lower()
    if v in ("0", "off", "false", "no"):
        return "off"
    if v == "sync":
        return "sync"
    return "lazy"


class _Ring:
    def __init__(self, dev: torch.device):
        self.dev = dev
        self.words = torch.zeros(_SLOTS, dtype=torch.int32, device=dev)
        self.host = torch.zeros(_SLOTS, dtype=torch.int32).pin_memory()
        self.next = 0
        self.pending = collections.deque()      # (slot, event, op, decode), oldest first

    def _resolve(self, entry) -> Optional[Exception]:
        slot, ev, op, decode = entry
        bits = int(self.host[slot])
        return decode(op, bits) if bits else None


_rings = {}
_lock = threading.Lock()


def _ring(dev: torch.device) -> _Ring:
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    r = _rings.get(key)
    if r is None:
        r = _rings[key] = _Ring(torch.device("cuda", key))
    return r


def poll(dev: torch.device) -> None:
    """Raise for the first finished op whose status word came back non-zero
    (does not wait for the GPU)."""
    if not _rings:
        return
    with _lock:
        r = _ring(dev)
        while r.pending and r.pending[0][1].query():
            err = r._resolve(r.pending.popleft())
            if err is not None:
                raise err


class Slot:
    """One status word lent to one op call."""

    __slots__ = ("ring", "index", "ptr")

    def __init__(self, ring: _Ring, index: int):
        self.ring, self.index = ring, index
        self.ptr = ring.words[index].data_ptr()


def acquire(dev: torch.device) -> Optional[Slot]:
    """A zeroed device status word for the next launch, or None when no word
    is used (``SSA_CHECKED=0`` or a stream capture in progress)."""
    if mode() == "off" or torch.cuda.is_current_stream_capturing():
        return None
    poll(dev)
    with _lock:
        r = _ring(dev)
        if len(r.pending) == _SLOTS:             # every word in flight: wait for the oldest
            entry = r.pending.popleft()
            entry[1].synchronize()
            err = r._resolve(entry)
            if err is not None:
                raise err
        s = Slot(r, r.next)
        r.next = (r.next + 1) % _SLOTS
        return s


def release(slot: Optional[Slot], op: str, decode: Callable[[str, int], Optional[Exception]]) -> None:
    """Queue the read-back of ``slot`` after the launch just made on the
    current stream; with ``SSA_CHECKED=sync`` wait for it and raise now."""
    if slot is None:
        return
    r = slot.ring
    stream = torch.cuda.current_stream(r.dev)
    with torch.cuda.stream(stream):
        r.host[slot.index].copy_(r.words[slot.index], non_blocking=True)
        r.words[slot.index].zero_()
    ev = torch.cuda.Event()
    ev.record(stream)
    entry = (slot.index, ev, op, decode)
    if mode() == "sync":
        ev.synchronize()
        err = r._resolve(entry)
        if err is not None:
            raise err
        return
    with _lock:
        r.pending.append(entry)


def check_errors(device=None) -> None:
    """Wait for every op launched so far on ``device`` (default: all devices
    with pending words) and raise for the first error a kernel reported."""
    with _lock:
        rings = list(_rings.values()) if device is None else [_ring(torch.device(device))]
        first = None
        for r in rings:
            while r.pending:
                entry = r.pending.popleft()
                entry[1].synchronize()
                err = r._resolve(entry)
                if err is not None and first is None:
                    first = err
    if first is not None:
        raise first


# ---------------------------------------------------------------------------
# decoders: status bits -> the exception each op raises
# ---------------------------------------------------------------------------
def route_error(op: str, bits: int) -> Optional[Exception]:
    if bits & L.SSA_DEVICE_INDEX_FULL:
        return RuntimeError(f"{op}: a bucket of the decode index had no free slot (rebuild it first)")
    if bits & L.SSA_DEVICE_BAD_INDEX:
        return ValueError(f"{op}: the code->key index failed its check")
    if bits & L.SSA_DEVICE_BAD_CODE:
        return ValueError(f"{op}: a key code is outside the codebook [0, num_codebook)")
    if bits & L.SSA_DEVICE_TIMEOUT:
        return RuntimeError(f"{op}: a device pipeline wait timed out; results are undefined")
    return RuntimeError(f"{op}: device status 0x{bits:x}")


def attn_error(op: str, bits: int) -> Optional[Exception]:
    if bits & L.SSA_DEVICE_INDEX_OOB:
        return IndexError(f"{op}: an index is outside [0, seq_len)")
    return RuntimeError(f"{op}: device status 0x{bits:x}")
