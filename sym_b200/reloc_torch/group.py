"""Consumer-sized transfer groups (reference ``reloc_torch.group``,
libreloc/python/reloc_torch/group.py:41-147).

A group holds 1..256 fresh typed preparations for one CUDA device. Executing
it allocates every output, validates all members together at the native
boundary (``pyreloc.prepare_dispatch_group``: one device, no destination
aliasing another destination or any source) and then runs all members behind
ONE wait on the caller's current stream with ONE completion: on the B200 the
members' DMA chunks and kernels queue back to back on the context's copy and
compute streams, so a layer's seven matrices cost one caller-stream round
trip instead of seven. Any failure consumes the whole group; members are
never retried.
"""
from __future__ import annotations

import operator
from contextlib import ExitStack
from dataclasses import dataclass, field
from threading import Lock
from types import MappingProxyType

from .. import pyreloc
from .dispatch import PreparedTypedTransfer, storage_view

MAX_MEMBERS = 256


@dataclass
class PreparedTransferGroup:
    requests: tuple
    device: object
    consumed: bool = field(default=False, init=False)
    native: object = field(default=None, init=False, repr=False)
    _execution_lock: object = field(default_factory=Lock, init=False, repr=False)

    @property
    def destinations(self):
        """One output descriptor per member, in member order."""
        return tuple(r.destination for r in self.requests)


@dataclass(frozen=True)
class GroupResult:
    tensors: tuple
    descriptors: tuple
    report: MappingProxyType


def prepare_transfer_group(requests):
    """Group fresh typed preparations that target one CUDA device. Launches
    nothing; the group owns its members from here on."""
    import torch

    requests = tuple(requests)
    if not 1 <= len(requests) <= MAX_MEMBERS:
        raise ValueError(f"a group must contain between 1 and {MAX_MEMBERS} requests")
    if len({id(r) for r in requests}) != len(requests):
        raise ValueError("a request cannot occur twice in a group")
    device = None
    for r in requests:
        if not isinstance(r, PreparedTypedTransfer):
            raise TypeError("group members must be prepared typed transfers")
        if r.consumed:
            raise RuntimeError("group member was already executed")
        if r.template is None:
            raise ValueError("typed group members require an immutable dispatch template")
        here = torch.device(r.device)
        if here.type != "cuda" or here.index is None:
            raise ValueError("group members need a canonical CUDA device")
        if device is not None and here != device:
            raise ValueError("group members must use the same CUDA device")
        device = here
    return PreparedTransferGroup(requests, device)


def execute_transfer_group(group, *, resources=None, gather_threads=8, gather_pool=None, pinning="auto",
                           min_pinned_bytes=None, max_scratch_bytes=64 << 20):
    """Complete one group (blocking for the host: outputs are ready on return)."""
    return _execute_transfer_group(group, resources=resources, gather_threads=gather_threads,
                                   gather_pool=gather_pool, pinning=pinning, min_pinned_bytes=min_pinned_bytes,
                                   max_scratch_bytes=max_scratch_bytes)


def _execute_transfer_group(group, *, resources=None, gather_threads=8, gather_pool=None, pinning="auto",
                            min_pinned_bytes=None, max_scratch_bytes=64 << 20, submit=False):
    """Allocate the outputs, validate and run the group. ``submit``: return
    ``(DispatchCompletion, outputs, descriptors)`` without waiting."""
    import torch

    from .resources import TransferResources

    if not isinstance(group, PreparedTransferGroup):
        raise TypeError("group must be a PreparedTransferGroup")
    max_scratch_bytes = operator.index(max_scratch_bytes)
    if not 0 < max_scratch_bytes < 1 << 64:
        raise ValueError("max_scratch_bytes must be positive and fit size_t")
    if not 0 < operator.index(gather_threads) < 1 << 31:
        raise ValueError("gather_threads must be positive and fit a native int")
    if resources is not None and not isinstance(resources, TransferResources):
        raise TypeError("resources must be TransferResources or None")
    owner = None if resources is None else resources.native_typed
    with ExitStack() as locks:
        for item in (group, *group.requests):
            if not item._execution_lock.acquire(blocking=False):
                raise RuntimeError("group or member is already executing")
            locks.callback(item._execution_lock.release)
            if item.consumed:
                raise RuntimeError("group or member was already executed")
        for r in group.requests:  # stale sources / parameters fail before any allocation
            r.recheck()
        descriptors = group.destinations
        outputs = tuple(torch.empty_strided(d.shape, d.strides, dtype=getattr(torch, d.dtype), device=d.device)
                        for d in descriptors)
        entries = [(r.template, r.source_view, storage_view(out, "cuda", out.device.index), "h2d")
                   for r, out in zip(group.requests, outputs)]
        try:
            native = pyreloc.prepare_dispatch_group(entries)
        except pyreloc.TransferError as error:
            raise RuntimeError(f"transfer group rejected: {error}") from error
        group.native = native
        group.consumed = True
        for r in group.requests:
            r.consumed = True
        stream = torch.cuda.current_stream(group.device).cuda_stream
        owners = (tuple(r.source for r in group.requests), outputs)
        run = pyreloc.submit_dispatch_group if submit else pyreloc.execute_dispatch_group
        try:
            result = run(native, caller_stream=stream, resources=owner, owners=owners,
                         max_scratch_bytes=max_scratch_bytes)
        except pyreloc.TransferError as error:
            raise RuntimeError(f"transfer group failed: {error}") from error
    if submit:
        return result, outputs, descriptors
    return GroupResult(outputs, descriptors, MappingProxyType(dict(result)))


__all__ = ("GroupResult", "PreparedTransferGroup", "execute_transfer_group", "prepare_transfer_group")
