"""Consumer-sized transfer groups: the API of the reference's
``reloc_torch.group`` (libreloc/python/reloc_torch/group.py:41-147 -- the
names, fields and error messages below are that interface).

On this executor a group is one native dispatch group
(``pyreloc.prepare_dispatch_group`` / ``execute_dispatch_group``): its
members' DMA chunks and fused kernels queue back to back on one device
context's copy and compute streams, after ONE wait on the caller's stream,
and complete through ONE event. A layer's seven weight matrices therefore
cost one caller-stream round trip instead of seven. Any failure consumes the
whole group; members are never retried.
"""
from __future__ import annotations

import operator
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
        return tuple(member.destination for member in self.requests)


@dataclass(frozen=True)
class GroupResult:
    tensors: tuple
    descriptors: tuple
    report: MappingProxyType


def _member_device(member):
    """The canonical CUDA device of one fresh typed member."""
    import torch

    if not isinstance(member, PreparedTypedTransfer):
        raise TypeError("group members must be prepared typed transfers")
    if member.consumed:
        raise RuntimeError("group member was already executed")
    if member.template is None:
        raise ValueError("typed group members require an immutable dispatch template")
    device = torch.device(member.device)
    if device.type != "cuda" or device.index is None:
        raise ValueError("group members need a canonical CUDA device")
    return device


def prepare_transfer_group(requests):
    """Group fresh typed preparations that target one CUDA device. Launches
    nothing; the group owns its members from here on."""
    members = tuple(requests)
    if not 1 <= len(members) <= MAX_MEMBERS:
        raise ValueError(f"a group must contain between 1 and {MAX_MEMBERS} requests")
    if len(set(map(id, members))) != len(members):
        raise ValueError("a request cannot occur twice in a group")
    devices = {_member_device(m) for m in members}
    if len(devices) != 1:
        raise ValueError("group members must use the same CUDA device")
    return PreparedTransferGroup(members, devices.pop())


class _Claim:
    """Exclusive use of a group and of each of its members for one
    execution: all of them are claimed, or none (a partial claim is given
    back before the error propagates)."""

    def __init__(self, group):
        self._locks = [group._execution_lock, *(m._execution_lock for m in group.requests)]
        self._items = [group, *group.requests]
        self._held = []

    def __enter__(self):
        for lock, item in zip(self._locks, self._items):
            if not lock.acquire(blocking=False):
                self.__exit__()
                raise RuntimeError("group or member is already executing")
            self._held.append(lock)
            if item.consumed:
                self.__exit__()
                raise RuntimeError("group or member was already executed")
        return self

    def __exit__(self, *exc):
        while self._held:
            self._held.pop().release()
        return False


def _checked_options(group, resources, gather_threads, max_scratch_bytes):
    from .resources import TransferResources

    if not isinstance(group, PreparedTransferGroup):
        raise TypeError("group must be a PreparedTransferGroup")
    scratch = operator.index(max_scratch_bytes)
    if not 0 < scratch < 1 << 64:
        raise ValueError("max_scratch_bytes must be positive and fit size_t")
    if not 0 < operator.index(gather_threads) < 1 << 31:
        raise ValueError("gather_threads must be positive and fit a native int")
    if resources is not None and not isinstance(resources, TransferResources):
        raise TypeError("resources must be TransferResources or None")
    return scratch, None if resources is None else resources.native_typed


def execute_transfer_group(group, *, resources=None, gather_threads=8, gather_pool=None, pinning="auto",
                           min_pinned_bytes=None, max_scratch_bytes=64 << 20):
    """Complete one group (blocking for the host: outputs are ready on return).
    The host-worker knobs of the reference are accepted and unused: no member
    is transformed on the CPU."""
    return _execute_transfer_group(group, resources=resources, gather_threads=gather_threads,
                                   max_scratch_bytes=max_scratch_bytes)


def _execute_transfer_group(group, *, resources=None, gather_threads=8, gather_pool=None, pinning="auto",
                            min_pinned_bytes=None, max_scratch_bytes=64 << 20, submit=False):
    """Allocate the outputs, validate the members together at the native
    boundary and run them as one native group. ``submit``: return
    ``(DispatchCompletion, outputs, descriptors)`` without waiting."""
    import torch

    scratch, owner = _checked_options(group, resources, gather_threads, max_scratch_bytes)
    with _Claim(group):
        # stale sources or parameters fail here, before anything is allocated
        for member in group.requests:
            member.recheck()
        descriptors = group.destinations
        outputs = tuple(torch.empty_strided(d.shape, d.strides, dtype=getattr(torch, d.dtype), device=d.device)
                        for d in descriptors)
        native = pyreloc.prepare_dispatch_group(
            [(m.template, m.source_view, storage_view(o, "cuda", o.device.index), "h2d")
             for m, o in zip(group.requests, outputs)])
        # From here the group is spent, whatever happens next.
        group.native = native
        for item in (group, *group.requests):
            item.consumed = True
        launch = pyreloc.submit_dispatch_group if submit else pyreloc.execute_dispatch_group
        try:
            outcome = launch(native, caller_stream=torch.cuda.current_stream(group.device).cuda_stream,
                             resources=owner, max_scratch_bytes=scratch,
                             owners=(tuple(m.source for m in group.requests), outputs))
        except pyreloc.TransferError as error:
            raise RuntimeError(f"transfer group failed: {error}") from error
    if submit:
        return outcome, outputs, descriptors
    return GroupResult(outputs, descriptors, MappingProxyType(dict(outcome)))


__all__ = ("GroupResult", "PreparedTransferGroup", "execute_transfer_group", "prepare_transfer_group")
