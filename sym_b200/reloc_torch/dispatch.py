"""Typed dispatch bridge for Torch tensors (reference
``reloc_torch.dispatch``, libreloc/python/reloc_torch/dispatch.py:156-362).

``prepare_typed_transfer`` validates a compiled TYPED recipe against a real
source tensor and its runtime parameters without allocating or launching:
exact symbol binding from the source shape, parameter snapshots (CPU values
only), the binder, the destination descriptor, storage views, capability and
the policy decision. ``execute_typed_transfer`` allocates the fresh CUDA
destination, rechecks the source storage and parameter values, orders the
runtime's private streams after the caller's current CUDA stream, runs the
selected B200 row and returns the tensor with an immutable scalar report.
Requests are single-use.
"""
from __future__ import annotations

import operator
from dataclasses import dataclass, field
from threading import Lock
from types import MappingProxyType

from .. import pyreloc
from .compiler import UnsupportedRecipe

POLICIES = ("auto", "original_cpu")

_TORCH_DTYPES = {"float32": "float32", "float16": "float16", "bfloat16": "bfloat16", "int8": "int8",
                 "int32": "int32", "int64": "int64"}


def dtype_name(dtype):
    name = str(dtype).replace("torch.", "")
    if name not in _TORCH_DTYPES:
        raise UnsupportedRecipe("unsupported_dtype", name)
    return name


def _current_stream(device):
    """The raw handle of the current CUDA stream of ``device`` (the cheap
    accessor when this Torch build has it)."""
    import torch

    index = device.index if device.index is not None else torch.cuda.current_device()
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(index)
    return torch.cuda.current_stream(index).cuda_stream


def storage_span(tensor):
    """Allocation base, capacity and the byte offset of element 0."""
    storage = tensor.untyped_storage()
    return int(storage.data_ptr()), int(storage.nbytes()), int(tensor.storage_offset()) * tensor.element_size()


def storage_snapshot(tensor):
    base, capacity, offset = storage_span(tensor)
    return (tuple(tensor.shape), tuple(tensor.stride()), offset, str(tensor.dtype), str(tensor.device), base,
            capacity)


def storage_view(tensor, kind, device):
    base, capacity, offset = storage_span(tensor)
    return pyreloc.BufferView(base=base, capacity_bytes=capacity, offset_bytes=offset,
                              extents=[int(d) for d in tensor.shape], strides=[int(s) for s in tensor.stride()],
                              element_size=tensor.element_size(), kind=kind, device=device)


def _parameter_snapshot(name, value, declared):
    import torch

    if not isinstance(value, torch.Tensor):
        raise UnsupportedRecipe("parameter_subclass", f"parameter {name!r} is not a tensor")
    if value.device.type != "cpu":
        raise UnsupportedRecipe("device_parameters_unavailable",
                                f"parameter {name!r} lives on {value.device}; only CPU parameter values are supported")
    data = value.detach().contiguous()
    dtype = dtype_name(data.dtype)
    if declared[0] == "int32" and data.dtype in (torch.int64, torch.int16, torch.int8):
        if data.numel() and (int(data.min()) < -(2 ** 31) or int(data.max()) >= 2 ** 31):
            raise UnsupportedRecipe("bind_error", f"parameter {name!r} does not fit int32")
        data = data.to(torch.int32)
        dtype = "int32"
    if dtype != declared[0]:
        raise UnsupportedRecipe("parameter_dtype", f"parameter {name!r} is {dtype}, declared {declared[0]}")
    return dtype, [int(d) for d in data.shape], data.numpy().tobytes()


@dataclass(frozen=True)
class DispatchResult:
    tensor: object
    report: MappingProxyType


@dataclass
class PreparedTypedTransfer:
    compiled: object
    source: object
    bindings: dict
    bound: object
    template: object
    device: object
    source_view: object
    parameters: dict
    snapshots: dict
    selected: dict
    consumed: bool = False
    direction: str = "h2d"
    _storage: tuple = field(default=(), repr=False)
    _execution_lock: object = field(default_factory=Lock, repr=False, compare=False)

    def __post_init__(self):
        self._storage = storage_snapshot(self.source)

    @property
    def capability(self):
        """The capability table of the selected template (a fresh copy)."""
        return self.template.capability

    def recheck(self):
        if storage_snapshot(self.source) != self._storage:
            raise RuntimeError("stale typed transfer: source storage or metadata changed after preflight")
        if not self.parameters:
            return
        declared = self.compiled.parameter_extents(self.bindings)
        for name, value in self.parameters.items():
            if _parameter_snapshot(name, value, declared[name]) != self.snapshots[name]:
                raise RuntimeError(f"stale typed transfer: parameter {name!r} changed after preflight")

    @property
    def report(self):
        return MappingProxyType(dict(self.selected))

    @property
    def destination(self):
        """The fresh output this request produces: dense, on ``device``."""
        shape = tuple(int(e) for e in self.bound.result_extents)
        strides, run = [], 1
        for e in reversed(shape):
            strides.append(run)
            run *= e
        return TensorDescriptor(shape, tuple(reversed(strides)), self.bound.result_dtype, self.device)


@dataclass(frozen=True)
class TensorDescriptor:
    """Shape, strides (elements), dtype name and device of a transfer output."""

    shape: tuple
    strides: tuple
    dtype: str
    device: object


def prepare_typed_transfer(compiled, source, device, *, parameters=None, policy="auto", calibration=None,
                           threads=8, implementation=""):
    import torch

    if not getattr(compiled, "typed", False):
        raise UnsupportedRecipe("not_typed_recipe", "the compiled recipe has no value transform")
    if policy not in POLICIES:
        raise ValueError(f"policy must be one of {POLICIES}, got {policy!r}")
    threads = operator.index(threads)
    device = torch.device(device)
    direction = compiled.recipe.direction
    ends = {"h2d": ("cpu", "cuda"), "d2h": ("cuda", "cpu")}.get(direction)
    if ends is None or source.device.type != ends[0] or device.type != ends[1]:
        raise UnsupportedRecipe("direction_mismatch",
                                f"{compiled.recipe.direction} recipe cannot move {source.device} -> {device}")
    if dtype_name(source.dtype) != compiled.recipe.source.dtype:
        raise UnsupportedRecipe("source_dtype", f"source is {source.dtype}, recipe expects "
                                                f"{compiled.recipe.source.dtype}")
    if not source.is_contiguous():
        raise UnsupportedRecipe("non_dense_source", "typed transfers take dense row-major sources")
    bindings, declared = compiled.bind_shape(tuple(source.shape))
    parameters = dict(parameters or {})
    missing, extra = sorted(set(declared) - set(parameters)), sorted(set(parameters) - set(declared))
    if missing or extra:
        raise UnsupportedRecipe("parameter_binding",
                                f"declared parameters {sorted(declared)}; missing {missing}, unexpected {extra}")
    snapshots = {n: _parameter_snapshot(n, parameters[n], declared[n]) for n in declared}
    gpu = source.device if direction == "d2h" else device
    index = gpu.index if gpu.index is not None else torch.cuda.current_device()
    key = ("typed", direction, tuple(sorted(bindings.items())),
           tuple((n, d, tuple(e), b) for n, (d, e, b) in sorted(snapshots.items())), index, policy, implementation)
    cache = compiled._execution_templates
    hit = cache.get(key)
    if hit is None:
        try:
            bound = pyreloc.bind_typed(compiled.decoded_plan, bindings, snapshots)
        except pyreloc.BindError as error:
            raise UnsupportedRecipe("bind_error", str(error)) from error
        try:
            template = pyreloc.prepare_dispatch_template(bound, direction, "cuda", policy=policy,
                                                         implementation=implementation)
        except pyreloc.TransferError as error:
            raise UnsupportedRecipe(error.code, str(error)) from error
        hit = cache.put(key, (bound, template))
    bound, template = hit
    if list(source.shape) != list(bound.source_extents):
        raise UnsupportedRecipe("shape_mismatch", f"source shape {list(source.shape)} vs {bound.source_extents}")
    if direction == "d2h":
        return PreparedTypedTransfer(compiled, source, bindings, bound, template, torch.device("cpu"),
                                     storage_view(source, "cuda", index), parameters, snapshots,
                                     template.selection, direction="d2h")
    return PreparedTypedTransfer(compiled, source, bindings, bound, template, torch.device("cuda", index),
                                 storage_view(source, "host", -1), parameters, snapshots, template.selection)


def execute_typed_transfer(request, *, n_buffers=4, n_streams=2, gather_threads=None, gather_pool=None,
                           pinning="auto", min_pinned_bytes=None, direct_dense_upload=True, pipeline=True,
                           chunk_size=None, resources=None, route="auto", out=None):
    """Complete a typed transfer into a fresh CUDA tensor (or ``out``)."""
    import torch

    from .resources import TransferResources

    if resources is not None and not isinstance(resources, TransferResources):
        raise TypeError("resources must be TransferResources or None")
    if not request._execution_lock.acquire(blocking=False):
        raise RuntimeError("typed transfer request is already executing")
    try:
        if request.consumed:
            raise RuntimeError("typed transfer request was already executed")
        request.recheck()
        shape = list(request.bound.result_extents)
        dtype = getattr(torch, request.bound.result_dtype)
        d2h = request.direction == "d2h"
        if out is None:
            out = torch.empty(shape, dtype=dtype, pin_memory=True) if d2h else \
                torch.empty(shape, dtype=dtype, device=request.device)
        elif list(out.shape) != shape or out.dtype != dtype or out.device != request.device \
                or not out.is_contiguous():
            raise ValueError("out must be a dense tensor of the result shape, dtype and device")
        dst_view = storage_view(out, "host", -1) if d2h else storage_view(out, "cuda", out.device.index)
        try:
            native = pyreloc.prepare_dispatch_from_template(request.template, request.source_view, dst_view)
        except pyreloc.TransferError as error:
            raise RuntimeError(f"typed dispatch rejected at execution: {error}") from error
        request.consumed = True
        stream = _current_stream(request.source.device if d2h else request.device)
        try:
            report = pyreloc.execute_dispatch(
                native, caller_stream=stream, n_buffers=n_buffers, chunk_size=chunk_size or 0,
                resources=None if resources is None else resources.native_typed,
                owners=(request.source, out), route=route)
        except pyreloc.TransferError as error:
            raise RuntimeError(f"{request.direction} typed dispatch failed: {error}") from error
        report = dict(report)
        report["placement_reason"] = request.selected["placement_reason"]
        report["policy"] = request.selected["policy"]
        return DispatchResult(out, MappingProxyType(report))
    finally:
        request._execution_lock.release()


__all__ = ("POLICIES", "DispatchResult", "PreparedTypedTransfer", "execute_typed_transfer", "prepare_typed_transfer")
