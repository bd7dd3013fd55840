"""Asynchronous, bounded transfer submission (reference
``reloc_torch.asynchronous``: TransferQueue / TransferCompletion /
PrefetchWindow, libreloc/python/reloc_torch/asynchronous.py:41-374).

A ``TransferQueue`` owns one CUDA device's submission order: ``submit(group)``
validates and enqueues a whole group (DMA into the context's HBM ring and the
fused kernels, see ``group.py``) and returns at once with a
``TransferCompletion``. Consumers either block (``wait()``) or, the point of
the API, make their own stream wait on the group's completion event
(``wait_stream()``) and keep the host free to submit the next layer. The queue
bounds what is outstanding: at most ``max_in_flight`` completions and
``max_output_bytes`` of outputs; ``PrefetchWindow`` keeps the next group in
flight while the caller consumes the current one.

Source buffers (CPU) must be ready and must not change until ``wait()`` /
``done()`` says the group completed. Outputs are allocated on the queue's own
stream and handed to consumer streams with ``record_stream``, so the caching
allocator never recycles them under pending work.
"""
from __future__ import annotations

import operator
import os
from collections import deque
from threading import RLock
from types import MappingProxyType

from .group import GroupResult, PreparedTransferGroup, _execute_transfer_group

# Completions whose consumer-side drain failed: their tensors and native
# handles stay referenced for the life of the process.
_QUARANTINE = []

_TOTAL_KEYS = ("source_bytes", "wire_bytes", "destination_bytes", "payload_bytes_transferred")


def _positive(value, name):
    if isinstance(value, bool):
        raise TypeError(f"{name} must be an integer")
    value = operator.index(value)
    if value <= 0:
        raise ValueError(f"{name} must be positive")
    return value


def _output_bytes(group):
    """Bytes of the fresh outputs a group will allocate."""
    import torch

    total = 0
    for d in group.destinations:
        if 0 in d.shape:
            continue
        elems = 1 + sum((n - 1) * s for n, s in zip(d.shape, d.strides))
        total += elems * getattr(torch, d.dtype).itemsize
    return total


class TransferCompletion:
    """One submitted group. Holds the group's sources and outputs until the
    group and every registered consumer are known to be done."""

    def __init__(self, queue, group, native, tensors, descriptors, size):
        self._queue, self._group, self._native = queue, group, native
        self._tensors, self._descriptors, self._size = tensors, descriptors, size
        self._consumers = {}   # cuda_stream handle -> torch stream
        self._retired = []     # events recorded at release() on each consumer
        self._released = False
        self._closed = False

    def _usable(self):
        self._queue._check_process()
        if self._closed:
            raise RuntimeError("transfer completion is closed")

    def done(self):
        """True once the group completed on the GPU (polls; never blocks)."""
        with self._queue._lock:
            self._usable()
            return self._native.query()

    def wait(self):
        """Block the host until the group completed; outputs and CPU sources
        are then safe to use / modify."""
        with self._queue._lock:
            self._usable()
            self._native.wait()
            if not self._released:
                import torch

                self._add_consumer(torch.cuda.current_stream(self._queue.device))
            return GroupResult(self._tensors, self._descriptors,
                               MappingProxyType(dict(self._group.native.report)))

    def wait_stream(self, stream=None):
        """Order ``stream`` (default: the current stream) after the group on the
        GPU, without a host wait; returns the output tensors."""
        import torch

        with self._queue._lock:
            self._usable()
            if self._released:
                raise RuntimeError("consumer use was already released")
            stream = torch.cuda.current_stream(self._queue.device) if stream is None else stream
            self._queue._check_stream(stream)
            self._native.wait_stream(stream.cuda_stream)
            self._add_consumer(stream)
            return self._tensors

    def _add_consumer(self, stream):
        for t in self._tensors:
            if t.is_cuda:
                t.record_stream(stream)
        self._consumers[stream.cuda_stream] = stream

    def release(self):
        """Mark the end of the consumers' use: call right after enqueueing the
        last kernel that reads the outputs. Later work on the same consumer
        streams does not delay this completion's retirement."""
        import torch

        with self._queue._lock:
            self._usable()
            if not self._released:
                for stream in self._consumers.values():
                    ev = torch.cuda.Event()
                    ev.record(stream)
                    self._retired.append(ev)
                self._released = True

    def close(self):
        """Wait for the group and its released consumers, then free the slot."""
        with self._queue._lock:
            self._queue._check_process()
            if self._closed:
                return
            error = None
            try:
                self.release()
            except Exception as failure:  # noqa: BLE001 - keep draining
                error = failure
            try:
                self._native.wait()
                self._queue._account(dict(self._group.native.report))
            except Exception as failure:  # noqa: BLE001
                error = error or failure
            try:
                if self._released:
                    for ev in self._retired:
                        ev.synchronize()
                else:
                    for stream in self._consumers.values():
                        stream.synchronize()
            except Exception as failure:  # noqa: BLE001
                _QUARANTINE.append((self._tensors, self._group, self._native, tuple(self._consumers.values()),
                                    tuple(self._retired)))
                self._queue._closed = True
                error = error or failure
            self._closed = True
            self._native = self._group = None
            self._tensors = self._descriptors = ()
            self._consumers.clear()
            self._retired.clear()
            self._queue._release(self)
            if error is not None:
                raise error

    cancel = close

    def __enter__(self):
        self._usable()
        return self

    def __exit__(self, *exc):
        self.close()
        return False


class TransferQueue:
    """One CUDA device's bounded submission queue. Submissions serialize on
    the host (a lock); their GPU work runs on the shared typed context's
    streams, ordered after the queue's own allocation stream."""

    def __init__(self, device="cuda:0", *, max_in_flight=2, max_output_bytes=128 << 20,
                 max_scratch_bytes=64 << 20, gather_threads=8, pinning="pinned", resources=None):
        import torch

        from .resources import TransferResources

        if resources is not None:
            if not isinstance(resources, TransferResources):
                raise TypeError("resources must be TransferResources")
            resources.native_typed  # rejects use from another process
            if resources.closed:
                raise RuntimeError("transfer resources are closed")
        self.max_in_flight = _positive(max_in_flight, "max_in_flight")
        self.max_output_bytes = _positive(max_output_bytes, "max_output_bytes")
        self.max_scratch_bytes = _positive(max_scratch_bytes, "max_scratch_bytes")
        self.gather_threads = _positive(gather_threads, "gather_threads")
        if pinning not in ("pinned", "pageable"):
            raise ValueError("pinning must be pinned or pageable")
        self.pinning = pinning
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("a transfer queue requires a CUDA device")
        self.device = torch.device("cuda", torch.cuda.current_device() if device.index is None else device.index)
        self._pid, self._lock = os.getpid(), RLock()
        self._closed = False
        self._held, self._bytes = set(), 0
        self._submitted = self._peak_bytes = self._peak_handles = 0
        self._totals = {"groups": 0, "logical_transfers": 0, "dispatches": {}, **{k: 0 for k in _TOTAL_KEYS}}
        self._stream = torch.cuda.Stream(device=self.device)  # output allocations live on this stream
        self._owns_resources = resources is None
        self._resources = resources if resources is not None else TransferResources(
            max_typed_retained_bytes=max_scratch_bytes, max_typed_live_bytes=max_scratch_bytes)

    def _check_process(self):
        if self._pid != os.getpid():
            raise RuntimeError("transfer queue belongs to another process")

    def _check_stream(self, stream):
        import torch

        if not isinstance(stream, torch.cuda.Stream) or stream.device != self.device:
            raise ValueError("stream must belong to the transfer queue device")

    def can_submit(self, group):
        self._check_process()
        with self._lock:
            return (not self._closed and len(self._held) < self.max_in_flight
                    and self._bytes + _output_bytes(group) <= self.max_output_bytes)

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
            size = _output_bytes(group)
            if not self.can_submit(group):
                raise BufferError("transfer queue output/slot budget exceeded; close a prior completion")
            if producer_stream is not None:
                self._check_stream(producer_stream)
                self._stream.wait_stream(producer_stream)
            with torch.cuda.stream(self._stream):
                native, tensors, descriptors = _execute_transfer_group(
                    group, submit=True, resources=self._resources, gather_threads=self.gather_threads,
                    pinning=self.pinning, max_scratch_bytes=self.max_scratch_bytes)
            handle = TransferCompletion(self, group, native, tensors, descriptors, size)
            self._held.add(handle)
            self._bytes += size
            self._submitted += 1
            self._peak_bytes = max(self._peak_bytes, self._bytes)
            self._peak_handles = max(self._peak_handles, len(self._held))
            return handle

    def _release(self, handle):
        self._held.discard(handle)
        self._bytes -= handle._size

    def _account(self, report):
        t = self._totals
        t["groups"] += 1
        t["logical_transfers"] += report["logical_transfers"]
        for item in report["items"]:
            for k in _TOTAL_KEYS:
                t[k] += item[k]
            t["dispatches"][item["implementation"]] = t["dispatches"].get(item["implementation"], 0) + 1

    def stats(self):
        self._check_process()
        with self._lock:
            return {"submitted": self._submitted, "held": len(self._held), "output_bytes": self._bytes,
                    "peak_output_bytes": self._peak_bytes, "peak_in_flight": self._peak_handles,
                    "closed": self._closed, "resources": self._resources.stats()["typed"],
                    "owns_resources": self._owns_resources,
                    "totals": {**self._totals, "dispatches": dict(self._totals["dispatches"])}}

    def prefetch(self, groups):
        """A ``PrefetchWindow`` over an iterable of prepared groups."""
        return PrefetchWindow(self, groups)

    def close(self):
        """Drain every held completion; close resources this queue created."""
        self._check_process()
        with self._lock:
            self._closed = True
            error = None
            for handle in tuple(self._held):
                try:
                    handle.close()
                except Exception as failure:  # noqa: BLE001
                    error = error or failure
            try:
                if self._owns_resources:
                    self._resources.close()
            except Exception as failure:  # noqa: BLE001
                error = error or failure
            if error is not None:
                raise error

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
    the caller consumes the current one. Each step releases the previous
    consumer, retires the oldest completion when the queue is full, submits
    the next group and yields its outputs ordered on the current stream
    (``wait_stream``). Groups are prepared lazily, one per step."""

    def __init__(self, queue, groups):
        self._queue = queue
        self._groups = iter(groups)
        self._handles = deque()
        self._last = None
        self._closed = False

    def __iter__(self):
        return self

    def __next__(self):
        if self._closed:
            raise StopIteration
        if self._last is not None:
            self._last.release()
            self._last = None
        try:
            group = next(self._groups)
        except StopIteration:
            self.close()
            raise
        while self._handles and not self._queue.can_submit(group):
            self._handles.popleft().close()
        handle = self._queue.submit(group)
        self._handles.append(handle)
        self._last = handle
        return handle.wait_stream()

    def close(self):
        if self._closed:
            return
        error = None
        while self._handles:
            try:
                self._handles.popleft().close()
            except Exception as failure:  # noqa: BLE001
                error = error or failure
        self._last, self._closed = None, True
        if error is not None:
            raise error

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


__all__ = ("PrefetchWindow", "TransferCompletion", "TransferQueue")
