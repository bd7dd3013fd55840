"""Asynchronous, bounded transfer submission: the API of the reference's
``reloc_torch.asynchronous`` (TransferQueue / TransferCompletion /
PrefetchWindow, libreloc/python/reloc_torch/asynchronous.py:41-374 -- the
class and method names, arguments and error messages are that interface).

The implementation is built on this executor's completion model: a submitted
group is one native dispatch group whose members run on one device context
and complete through ONE native event (``pyreloc.DispatchCompletion``:
``wait`` / ``query`` / ``wait_stream``). A queue only adds budgets and
ownership around it:

* budgets -- at most ``max_in_flight`` open completions and
  ``max_output_bytes`` of their outputs (the allocation sizes of the output
  descriptors, computed on the ``meta`` device without allocating);
* outputs -- allocated on the queue's own stream; every consumer stream that
  is ordered after the group (``wait_stream`` / ``wait``) is registered with
  the caching allocator (``record_stream``), and ``release()`` marks the end
  of their reads with one event per consumer stream, which ``close()`` waits
  for before the budget slot is given back;
* failures -- a consumer drain that cannot be proven complete sends the
  outputs and native handles to the package's process-lifetime quarantine
  (``pyreloc._QUARANTINED``) and closes the queue to new work.

Source buffers (CPU) must be ready and unchanged until ``wait()`` /
``done()`` reports the group complete.
"""
from __future__ import annotations

import operator
import os
from collections import OrderedDict, deque
from dataclasses import dataclass
from itertools import count
from threading import RLock
from types import MappingProxyType

from .. import pyreloc
from .group import GroupResult, PreparedTransferGroup, _execute_transfer_group

_COUNTED = ("source_bytes", "wire_bytes", "destination_bytes", "payload_bytes_transferred")


@dataclass(frozen=True)
class _Limits:
    """A queue's validated budgets and per-group options."""

    max_in_flight: int
    max_output_bytes: int
    max_scratch_bytes: int
    gather_threads: int
    pinning: str

    def __post_init__(self):
        for name in ("max_in_flight", "max_output_bytes", "max_scratch_bytes", "gather_threads"):
            raw = getattr(self, name)
            if isinstance(raw, bool):
                raise TypeError(f"{name} must be an integer")
            if operator.index(raw) <= 0:
                raise ValueError(f"{name} must be positive")
            object.__setattr__(self, name, operator.index(raw))
        if self.pinning not in ("pinned", "pageable"):
            raise ValueError("pinning must be pinned or pageable")


def _allocation_bytes(group):
    """Bytes the group's outputs will take: the storage of each destination
    descriptor, sized on the meta device."""
    import torch

    return sum(torch.empty_strided(d.shape, d.strides, dtype=getattr(torch, d.dtype), device="meta")
               .untyped_storage().nbytes() for d in group.destinations)


class TransferCompletion:
    """One submitted group, from submission to ``close()``. It keeps the
    group's sources and outputs referenced until the group and every
    released consumer are known to be done."""

    _OPEN, _RELEASED, _CLOSED = range(3)

    def __init__(self, queue, token, group, native, tensors, descriptors, nbytes):
        self._queue, self._token, self._group, self._native = queue, token, group, native
        self._tensors, self._descriptors, self.nbytes = tensors, descriptors, nbytes
        self._state = self._OPEN
        # consumer stream handle -> (stream, event recorded by release() or None)
        self._readers = OrderedDict()

    def _guard(self):
        self._queue._check_process()
        if self._state == self._CLOSED:
            raise RuntimeError("transfer completion is closed")

    def _read_on(self, stream):
        """Register `stream` as a reader of the outputs (the caching allocator
        will not recycle them under its pending work)."""
        if stream.cuda_stream not in self._readers:
            for tensor in self._tensors:
                tensor.record_stream(stream)
            self._readers[stream.cuda_stream] = (stream, None)

    def done(self):
        """True once the group completed on the GPU (polls; never blocks)."""
        with self._queue._lock:
            self._guard()
            return self._native.query()

    def wait(self):
        """Block the host until the group completed; outputs and CPU sources
        are then safe to use and change."""
        import torch

        with self._queue._lock:
            self._guard()
            self._native.wait()
            if self._state == self._OPEN:
                self._read_on(torch.cuda.current_stream(self._queue.device))
            return GroupResult(self._tensors, self._descriptors, MappingProxyType(dict(self._group.native.report)))

    def wait_stream(self, stream=None):
        """Order ``stream`` (default: the current stream) after the group on
        the GPU, without a host wait; returns the output tensors."""
        import torch

        with self._queue._lock:
            self._guard()
            if self._state != self._OPEN:
                raise RuntimeError("consumer use was already released")
            stream = torch.cuda.current_stream(self._queue.device) if stream is None else stream
            self._queue._check_stream(stream)
            self._native.wait_stream(stream.cuda_stream)
            self._read_on(stream)
            return self._tensors

    def release(self):
        """Mark the end of the consumers' use: call right after enqueueing the
        last kernel that reads the outputs. Later work on the same consumer
        streams does not delay this completion's retirement."""
        import torch

        with self._queue._lock:
            self._guard()
            if self._state == self._OPEN:
                for handle, (stream, _) in self._readers.items():
                    fence = torch.cuda.Event()
                    fence.record(stream)
                    self._readers[handle] = (stream, fence)
                self._state = self._RELEASED

    def _drain_readers(self):
        for stream, fence in self._readers.values():
            if fence is not None:
                fence.synchronize()
            else:  # never released: everything on the stream so far
                stream.synchronize()

    def close(self):
        """Wait for the group and its consumers, then free the budget slot."""
        with self._queue._lock:
            self._queue._check_process()
            if self._state == self._CLOSED:
                return
            failure = None
            try:
                self.release()
            except Exception as error:  # noqa: BLE001 - the drain continues
                failure = error
            try:
                self._native.wait()
                self._queue._tally(self._group.native.report)
            except Exception as error:  # noqa: BLE001
                failure = failure or error
            try:
                self._drain_readers()
            except Exception as error:  # noqa: BLE001
                # unproven reader completion: nothing here may be reused, ever
                pyreloc._QUARANTINED.append((self._tensors, self._group, self._native, tuple(self._readers.values())))
                self._queue._closed = True
                failure = failure or error
            self._state = self._CLOSED
            self._queue._give_back(self._token)
            self._native = self._group = None
            self._tensors = self._descriptors = ()
            self._readers.clear()
            if failure is not None:
                raise failure

    cancel = close

    def __enter__(self):
        self._guard()
        return self

    def __exit__(self, *exc):
        self.close()
        return False


class TransferQueue:
    """One CUDA device's bounded submission queue. Submissions serialize on
    the host; their GPU work runs on the typed context of the queue's
    resources, ordered after the queue's own allocation stream."""

    def __init__(self, device="cuda:0", *, max_in_flight=2, max_output_bytes=128 << 20,
                 max_scratch_bytes=64 << 20, gather_threads=8, pinning="pinned", resources=None):
        import torch

        from .resources import TransferResources

        if resources is not None:
            if not isinstance(resources, TransferResources):
                raise TypeError("resources must be TransferResources")
            resources.native_typed  # refuses resources of another process
            if resources.closed:
                raise RuntimeError("transfer resources are closed")
        self._limits = _Limits(max_in_flight, max_output_bytes, max_scratch_bytes, gather_threads, pinning)
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("a transfer queue requires a CUDA device")
        self.device = torch.device("cuda", torch.cuda.current_device() if device.index is None else device.index)
        self._pid, self._lock, self._closed = os.getpid(), RLock(), False
        self._open = OrderedDict()  # token -> open TransferCompletion
        self._tokens = count()
        self._stats = {"submitted": 0, "peak_output_bytes": 0, "peak_in_flight": 0}
        self._totals = {"groups": 0, "logical_transfers": 0, "dispatches": {}, **dict.fromkeys(_COUNTED, 0)}
        self._stream = torch.cuda.Stream(device=self.device)
        self._owns_resources = resources is None
        self._resources = resources or TransferResources(max_typed_retained_bytes=max_scratch_bytes,
                                                         max_typed_live_bytes=max_scratch_bytes)

    # budgets and limits, read-only views of the validated options
    max_in_flight = property(lambda self: self._limits.max_in_flight)
    max_output_bytes = property(lambda self: self._limits.max_output_bytes)
    max_scratch_bytes = property(lambda self: self._limits.max_scratch_bytes)
    gather_threads = property(lambda self: self._limits.gather_threads)
    pinning = property(lambda self: self._limits.pinning)

    def _check_process(self):
        if self._pid != os.getpid():
            raise RuntimeError("transfer queue belongs to another process")

    def _check_stream(self, stream):
        import torch

        if not isinstance(stream, torch.cuda.Stream) or stream.device != self.device:
            raise ValueError("stream must belong to the transfer queue device")

    def _held_bytes(self):
        return sum(c.nbytes for c in self._open.values())

    def _fits(self, nbytes):
        return (not self._closed and len(self._open) < self._limits.max_in_flight
                and self._held_bytes() + nbytes <= self._limits.max_output_bytes)

    def can_submit(self, group):
        self._check_process()
        with self._lock:
            return self._fits(_allocation_bytes(group))

    def submit(self, group, *, producer_stream=None):
        """Enqueue a fresh group; returns its ``TransferCompletion`` at once.
        ``producer_stream``: GPU work the group must follow (the queue's own
        stream otherwise; CPU sources need no ordering)."""
        import torch

        self._check_process()
        if not isinstance(group, PreparedTransferGroup):
            raise TypeError("submit expects a PreparedTransferGroup")
        with self._lock:
            if self._closed:
                raise RuntimeError("transfer queue is closed")
            if group.device != self.device:
                raise ValueError("group device differs from the transfer queue")
            nbytes = _allocation_bytes(group)
            if not self._fits(nbytes):
                raise BufferError("transfer queue output/slot budget exceeded; close a prior completion")
            if producer_stream is not None:
                self._check_stream(producer_stream)
                self._stream.wait_stream(producer_stream)
            with torch.cuda.stream(self._stream):
                native, tensors, descriptors = _execute_transfer_group(
                    group, submit=True, resources=self._resources, gather_threads=self._limits.gather_threads,
                    max_scratch_bytes=self._limits.max_scratch_bytes)
            token = next(self._tokens)
            completion = TransferCompletion(self, token, group, native, tensors, descriptors, nbytes)
            self._open[token] = completion
            s = self._stats
            s["submitted"] += 1
            s["peak_output_bytes"] = max(s["peak_output_bytes"], self._held_bytes())
            s["peak_in_flight"] = max(s["peak_in_flight"], len(self._open))
            return completion

    def _give_back(self, token):
        self._open.pop(token, None)

    def _tally(self, report):
        t = self._totals
        t["groups"] += 1
        t["logical_transfers"] += report["logical_transfers"]
        for item in report["items"]:
            for key in _COUNTED:
                t[key] += item[key]
            t["dispatches"][item["implementation"]] = t["dispatches"].get(item["implementation"], 0) + 1

    def stats(self):
        self._check_process()
        with self._lock:
            return {**self._stats, "held": len(self._open), "output_bytes": self._held_bytes(),
                    "closed": self._closed, "resources": self._resources.stats()["typed"],
                    "owns_resources": self._owns_resources,
                    "totals": {**self._totals, "dispatches": dict(self._totals["dispatches"])}}

    def prefetch(self, groups):
        """A ``PrefetchWindow`` over an iterable of prepared groups."""
        return PrefetchWindow(self, groups)

    def close(self):
        """Close every open completion (their work drained) and the resources
        this queue created; refuse new submissions."""
        self._check_process()
        with self._lock:
            self._closed = True
            failure = None
            for completion in tuple(self._open.values()):
                try:
                    completion.close()
                except Exception as error:  # noqa: BLE001
                    failure = failure or error
            try:
                if self._owns_resources:
                    self._resources.close()
            except Exception as error:  # noqa: BLE001
                failure = failure or error
            if failure is not None:
                raise failure

    def __enter__(self):
        self._check_process()
        if self._closed:
            raise RuntimeError("transfer queue is closed")
        return self

    def __exit__(self, *exc):
        self.close()
        return False


class PrefetchWindow:
    """Iterate over groups, keeping the next group's transfer in flight while
    the caller consumes the current one: each step releases the previous
    consumer, closes the oldest completions until the queue's budget admits
    the next group, submits it and yields its outputs ordered on the current
    stream. Groups are drawn lazily, one per step."""

    def __init__(self, queue, groups):
        self._queue = queue
        self._completions = deque()
        self._steps = self._walk(iter(groups))
        self._closed = False

    def _walk(self, groups):
        previous = None
        for group in groups:
            if previous is not None:
                previous.release()
            while self._completions and not self._queue.can_submit(group):
                self._completions.popleft().close()
            previous = self._queue.submit(group)
            self._completions.append(previous)
            yield previous.wait_stream()
        if previous is not None:
            previous.release()

    def __iter__(self):
        return self

    def __next__(self):
        if self._closed:
            raise StopIteration
        try:
            return next(self._steps)
        except StopIteration:
            self.close()
            raise

    def close(self):
        if self._closed:
            return
        self._closed = True
        self._steps.close()
        failure = None
        while self._completions:
            try:
                self._completions.popleft().close()
            except Exception as error:  # noqa: BLE001
                failure = failure or error
        if failure is not None:
            raise failure

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


__all__ = ("PrefetchWindow", "TransferCompletion", "TransferQueue")
