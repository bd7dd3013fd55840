"""``pyreloc`` for the B200 executor: the reference binding's names, keywords
and error behaviour (libreloc/python/PyReloc.cpp, PyDispatch.cpp,
PyTransfer.cpp) for the typed host->device path, bound through ctypes to the
drop-in C-ABI of ``include/sym_b200.h``.

Buffers are described by ``BufferView`` (allocation base, capacity, logical
offset, extents, strides, element size, kind, device) exactly as the
reference's ``pyreloc.BufferView``. Execution is GPU-only: every supported plan
runs in the fused sm_100a kernels; there is no CPU execution entry point.
"""
from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass, field
from types import MappingProxyType

from . import _native
from ._native import SbError, SbOptions, SbView, error_of, json_call

cuda_enabled = True


class DecodeError(ValueError):
    """Wire decoding failed; ``offset`` is the byte offset of the violated item."""

    def __init__(self, message, offset=-1):
        super().__init__(message)
        self.offset = offset


class BindError(ValueError):
    pass


class TransferError(RuntimeError):
    """A dispatch/transfer failure with a stable ``code``."""

    def __init__(self, code, message):
        super().__init__(f"{code}: {message}")
        self.code = code
        self.detail = message


# Owners of executions whose completion could not be proven
# (completion_unknown): kept alive for the life of the process, because work
# that may still touch their memory has no proven end.
_QUARANTINED = []


def _raise_transfer(err: SbError, owners=None):
    code, message, _ = error_of(err)
    if code == "completion_unknown" and owners is not None:
        _QUARANTINED.append(owners)
    raise TransferError(code, message)


def version() -> str:
    return _native.lib().sb_version().decode()


def kernel_launches() -> int:
    """Kernels this process launched through the native library."""
    return int(_native.lib().sb_kernel_launches())


def wire_version(data: bytes):
    v = _native.lib().sb_wire_version(bytes(data), len(data))
    return None if v < 0 else v


class _Handle:
    _free = None

    def __init__(self, ptr):
        self._ptr = ctypes.c_void_p(ptr) if not isinstance(ptr, ctypes.c_void_p) else ptr

    @property
    def ptr(self):
        return self._ptr

    def __del__(self):
        ptr = getattr(self, "_ptr", None)
        native = globals().get("_native")  # None once the interpreter tears modules down
        lib = getattr(native, "_lib", None)
        if ptr and ptr.value and self._free and lib is not None:
            getattr(lib, self._free)(ptr)
            ptr.value = None


class PlanHandle(_Handle):
    _free = "sb_plan_free"

    def __init__(self, ptr):
        super().__init__(ptr)
        self._info = json_call(_native.lib().sb_plan_describe, self._ptr)

    symbols = property(lambda self: list(self._info["symbols"]))
    num_axes = property(lambda self: self._info["num_axes"])
    element_size = property(lambda self: self._info["element_size"])
    no_copy = property(lambda self: self._info["no_copy"])

    def __repr__(self):
        return (f"PlanHandle(symbols={self.symbols}, axes={self.num_axes}, "
                f"element_size={self.element_size}, no_copy={self.no_copy})")


class TypedPlanHandle(PlanHandle):
    source_dtype = property(lambda self: self._info["source_dtype"])
    result_dtype = property(lambda self: self._info["result_dtype"])
    source_rank = property(lambda self: self._info["source_rank"])
    result_rank = property(lambda self: self._info["result_rank"])
    num_stages = property(lambda self: len(self._info["stages"]))
    layout_axes = property(lambda self: self._info["num_axes"])
    stages = property(lambda self: [dict(s) for s in self._info["stages"]])
    parameters = property(lambda self: [dict(p) for p in self._info["parameters"]])
    fills = property(lambda self: self._info["fills"])

    def __repr__(self):
        return (f"TypedPlanHandle({self.source_dtype} -> {self.result_dtype}, stages={self.num_stages}, "
                f"symbols={self.symbols})")


def _load(fn, data, cls):
    data = bytes(data)
    out = ctypes.c_void_p()
    err = SbError()
    if fn(data, len(data), ctypes.byref(out), ctypes.byref(err)):
        _, message, offset = error_of(err)
        raise DecodeError(f"decode error at byte offset {offset}: {message}", offset)
    return cls(out)


def load_plan(data) -> PlanHandle:
    """Decode a wire v0 (layout-only) plan."""
    return _load(_native.lib().sb_load_plan, data, PlanHandle)


def load_typed_plan(data) -> TypedPlanHandle:
    """Decode a wire v1 typed plan."""
    return _load(_native.lib().sb_load_typed_plan, data, TypedPlanHandle)


class BoundPlan(_Handle):
    _free = "sb_bound_free"

    def __init__(self, ptr, info=None):
        super().__init__(ptr)
        self._info = info if info is not None else json_call(_native.lib().sb_bound_describe, self._ptr)

    extents = property(lambda self: list(self._info["extents"]))
    src_strides = property(lambda self: list(self._info["src_strides"]))
    dst_strides = property(lambda self: list(self._info["dst_strides"]))
    element_size = property(lambda self: self._info["element_size"])
    total_bytes = property(lambda self: self._info["total_bytes"])
    no_copy = property(lambda self: self._info["no_copy"])
    typed = property(lambda self: self._info["typed"])
    strategy = property(lambda self: self._info["strategy"])
    pads = property(lambda self: [dict(p) for p in self._info["pads"]])

    def describe(self):
        return dict(self._info)

    def __repr__(self):
        return f"BoundPlan(extents={self.extents}, total_bytes={self.total_bytes}, strategy='{self.strategy}')"


class _LayoutView:
    """The layout part of a TypedBoundPlan (read-only)."""

    def __init__(self, info):
        self._info = info

    def __getattr__(self, name):
        info = self.__dict__["_info"]
        if name in info:
            return info[name]
        raise AttributeError(name)


class TypedBoundPlan(_Handle):
    _free = "sb_bound_free"

    def __init__(self, ptr):
        super().__init__(ptr)
        self._info = json_call(_native.lib().sb_bound_describe, self._ptr, cap=1 << 18)

    source_bytes = property(lambda self: self._info["source_bytes"])
    destination_bytes = property(lambda self: self._info["destination_bytes"])
    parameter_bytes = property(lambda self: self._info["parameter_bytes"])
    cuts = property(lambda self: [dict(c) for c in self._info["cuts"]])
    requirements = property(lambda self: list(self._info["requirements"]))
    layout = property(lambda self: _LayoutView(self._info["layout"]))
    source_extents = property(lambda self: list(self._info["source_extents"]))
    result_extents = property(lambda self: list(self._info["result_extents"]))
    source_dtype = property(lambda self: self._info["source_dtype"])
    result_dtype = property(lambda self: self._info["result_dtype"])
    stages = property(lambda self: [dict(s) for s in self._info["stages"]])

    def wire_bytes(self, boundary):
        cuts = self._info["cuts"]
        if not 0 <= boundary < len(cuts):
            raise ValueError("boundary out of range")
        return cuts[boundary]["bytes"]

    def describe(self):
        """Bound layout, footprints and checked stage arithmetic as a dict."""
        return dict(self._info)

    def __repr__(self):
        return (f"TypedBoundPlan(source_bytes={self.source_bytes}, destination_bytes={self.destination_bytes}, "
                f"parameter_bytes={self.parameter_bytes}, stages={len(self._info['stages'])})")


def _symbol_arrays(symbols):
    names = list(symbols)
    n = len(names)
    arr_n = (ctypes.c_char_p * max(1, n))(*[str(k).encode() for k in names])
    arr_v = (ctypes.c_int64 * max(1, n))(*[int(symbols[k]) for k in names])
    return n, arr_n, arr_v


def bind(plan: PlanHandle, symbols, strategy="auto", **_):
    """Bind a wire v0 plan against ``{symbol: value}``."""
    if isinstance(plan, TypedPlanHandle):
        raise BindError("bind expects a layout-only (v0) plan; use bind_typed")
    n, names, values = _symbol_arrays(symbols)
    out = ctypes.c_void_p()
    err = SbError()
    if _native.lib().sb_bind(plan.ptr, n, names, values, ctypes.byref(out), ctypes.byref(err)):
        raise BindError(error_of(err)[1])
    return BoundPlan(out)


def bind_typed(plan: TypedPlanHandle, symbols, parameters=None):
    """Bind a typed plan against ``{symbol: value}`` and
    ``{parameter name: (dtype, extents, bytes)}``; the bytes are copied."""
    parameters = dict(parameters or {})
    n, names, values = _symbol_arrays(symbols)
    pn = list(parameters)
    m = max(1, len(pn))
    pnames = (ctypes.c_char_p * m)(*[p.encode() for p in pn])
    pdt = (ctypes.c_char_p * m)(*[str(parameters[p][0]).encode() for p in pn])
    for p in pn:
        if len(parameters[p][1]) > 1:
            raise BindError(f"parameter '{p}' rank differs from its declaration")
    pranks = (ctypes.c_int32 * m)(*[len(parameters[p][1]) for p in pn])
    pext = (ctypes.c_int64 * m)(*[int(parameters[p][1][0]) if parameters[p][1] else 0 for p in pn])
    keep = [ctypes.create_string_buffer(bytes(parameters[p][2]), max(1, len(parameters[p][2]))) for p in pn]
    pbytes = (ctypes.c_void_p * m)(*[ctypes.cast(b, ctypes.c_void_p) for b in keep])
    plens = (ctypes.c_size_t * m)(*[len(parameters[p][2]) for p in pn])
    out = ctypes.c_void_p()
    err = SbError()
    if _native.lib().sb_bind_typed(plan.ptr, n, names, values, len(pn), pnames, pdt, pranks, pext, pbytes, plens,
                                   ctypes.byref(out), ctypes.byref(err)):
        raise BindError(error_of(err)[1])
    return TypedBoundPlan(out)


_DIRECTIONS = {"h2d": 0, "d2h": 1}


def query_capability(bound: TypedBoundPlan, direction="h2d", device="cuda"):
    """Eligible and excluded rows for ``direction`` with a ``device`` end."""
    err = SbError()
    buf = ctypes.create_string_buffer(1 << 16)
    if _native.lib().sb_query_capability(bound.ptr, _DIRECTIONS[direction], 1 if device == "cuda" else 0, buf,
                                         1 << 16, ctypes.byref(err)):
        _raise_transfer(err)
    import json

    return json.loads(buf.value.decode())


class DispatchTemplate(_Handle):
    """Immutable: checked arithmetic, capability and the selected row."""

    _free = "sb_template_free"

    def __init__(self, ptr, bound):
        super().__init__(ptr)
        self.bound = bound
        self._info = json_call(_native.lib().sb_template_describe, self._ptr)

    capability = property(lambda self: {k: [dict(r) for r in v] for k, v in self._info["capability"].items()})
    selection = property(lambda self: dict(self._info["selection"]))
    program = property(lambda self: self)
    device_kernel = property(lambda self: self._info.get("device_kernel"))
    padded_rows = property(lambda self: self._info.get("padded_rows"))
    row_bytes = property(lambda self: self._info.get("row_bytes"))

    def describe(self):
        return dict(self._info)


def prepare_dispatch_template(bound: TypedBoundPlan, direction="h2d", device="cuda", *, policy="auto",
                              calibration=None, threads=8, implementation=""):
    """Validate the program, query capability and apply the policy (no buffers)."""
    if policy not in ("auto", "original_cpu"):
        raise ValueError("policy must be 'auto' or 'original_cpu'")
    if not isinstance(implementation, str):
        raise TypeError("implementation must be a string")
    out = ctypes.c_void_p()
    err = SbError()
    if _native.lib().sb_prepare_dispatch_template(bound.ptr, _DIRECTIONS[direction],
                                                  1 if policy == "original_cpu" else 0,
                                                  implementation.encode(), ctypes.byref(out), ctypes.byref(err)):
        _raise_transfer(err)
    return DispatchTemplate(out, bound)


@dataclass
class BufferView:
    """A caller buffer: allocation, capacity, logical offset and view."""

    base: int
    capacity_bytes: int
    offset_bytes: int
    extents: list
    strides: list
    element_size: int
    kind: str = "host"
    device: int = -1

    def native(self) -> SbView:
        rank = len(self.extents)
        if rank > 8:
            raise TransferError("invalid_view", "views have at most 8 dimensions")
        v = SbView(int(self.base), int(self.capacity_bytes), int(self.offset_bytes), 1 if self.kind == "cuda" else 0,
                   int(self.device), rank, int(self.element_size))
        pairs = list(zip(self.extents, self.strides))
        if pairs:
            v.extents[:len(pairs)] = [int(e) for e, _ in pairs]
            v.strides[:len(pairs)] = [int(x) for _, x in pairs]
        return v


class DispatchRequest(_Handle):
    """A single-use prepared request (template + validated views)."""

    _free = "sb_request_free"

    def __init__(self, ptr, template):
        super().__init__(ptr)
        self.template = template
        self.consumed = False
        sel = template._info["selection"]
        self.report = MappingProxyType({"implementation": sel["implementation"], "policy": sel["policy"],
                                        "placement_reason": sel["placement_reason"]})


def prepare_dispatch_from_template(prepared: DispatchTemplate, source: BufferView, destination: BufferView):
    out = ctypes.c_void_p()
    err = SbError()
    s, d = source.native(), destination.native()
    if _native.lib().sb_prepare_dispatch(prepared.ptr, ctypes.byref(s), ctypes.byref(d), ctypes.byref(out),
                                         ctypes.byref(err)):
        _raise_transfer(err)
    return DispatchRequest(out, prepared)


def prepare_dispatch(bound, source, destination, direction="h2d", *, policy="auto", calibration=None, threads=8,
                     implementation=""):
    tmpl = prepare_dispatch_template(bound, direction, "cuda", policy=policy, implementation=implementation)
    return prepare_dispatch_from_template(tmpl, source, destination)


def _options(n_buffers=4, route="auto", chunk_size=0, caller_stream=None, async_completion=False):
    o = SbOptions()
    o.n_buffers = int(n_buffers)
    if route not in _native.ROUTES:
        raise ValueError(f"route must be one of {sorted(_native.ROUTES)}")
    o.route = _native.ROUTES[route]
    o.chunk_bytes = int(chunk_size or 0)
    if caller_stream is not None:
        o.caller_stream = ctypes.c_void_p(int(caller_stream))
        o.has_caller_stream = 1
    o.async_completion = 1 if async_completion else 0
    return o


_TLS = threading.local()


def _call_scratch():
    """This thread's error record and report buffer for execute calls (the
    native call fills them; reused so each call does not allocate 8 KiB)."""
    scratch = getattr(_TLS, "scratch", None)
    if scratch is None:
        scratch = _TLS.scratch = (SbError(), ctypes.create_string_buffer(8192))
    return scratch


def execute_dispatch(request: DispatchRequest, *, caller_stream=None, n_buffers=4, n_streams=2, gather_threads=None,
                     gather_pool=None, pinning="pinned", min_pinned_bytes=None, direct_dense_upload=True,
                     pipeline=True, chunk_size=0, resources=None, owners=(), route="auto",
                     async_completion=False):
    """Run the prepared request on the destination device's context.

    Blocks until complete unless ``async_completion`` (then ``caller_stream``
    is ordered after the work). ``owners`` are kept alive for the call.
    Host-worker knobs of the reference (gather threads/pools, pinning) are
    accepted and ignored: no data is transformed on the CPU.
    """
    if request.consumed:
        raise TransferError("already_executed", "dispatch requests are single-use")
    request.consumed = True
    opts = _options(n_buffers, route, chunk_size, caller_stream, async_completion)
    err, buf = _call_scratch()
    native_res = resources.handle if resources is not None else None
    _keep = owners
    rc = _native.lib().sb_execute_dispatch(request.ptr, native_res, ctypes.byref(opts), buf, 8192,
                                           ctypes.byref(err))
    del _keep
    import json

    report = json.loads(buf.value.decode())
    request.report = MappingProxyType(report)
    if rc:
        _raise_transfer(err, owners)
    return MappingProxyType(report)


def execute_rows(prepared: DispatchTemplate, source_ptr: int, destination_ptr: int, row_begin: int, row_end: int,
                 *, device: int, host_source: bool = True, resources=None, caller_stream=None, n_buffers=4,
                 route="dma_ring", chunk_size=0, async_completion=False):
    """Produce physical result rows [row_begin, row_end) into the window's own
    device storage (a shard). ``host_source``: the source pointer is host
    memory (only the rows' bytes cross PCIe); otherwise it is device memory."""
    opts = _options(n_buffers, route, chunk_size, caller_stream, async_completion)
    err = SbError()
    buf = ctypes.create_string_buffer(8192)
    rc = _native.lib().sb_execute_rows(prepared.ptr, resources.handle if resources is not None else None,
                                       int(device), ctypes.c_void_p(int(source_ptr)), 1 if host_source else 0,
                                       ctypes.c_void_p(int(destination_ptr)), int(row_begin), int(row_end),
                                       ctypes.byref(opts), buf, 8192, ctypes.byref(err))
    import json

    report = json.loads(buf.value.decode())
    if rc:
        _raise_transfer(err)
    return MappingProxyType(report)


def execute_source_rows(prepared: DispatchTemplate, source_ptr: int, row_begin: int, row_end: int,
                        destination_ptr: int, *, device: int, resources=None, caller_stream=None,
                        async_completion=False):
    """Transform a window of source rows held in device memory (this GPU's or
    a peer's mapped with ``ipc_open``) into the full destination: the window
    ``[row_begin, row_end)`` of the plan's source-outer axis starts at
    ``source_ptr``; only the result cells those rows produce are written."""
    opts = _options(4, "auto", 0, caller_stream, async_completion)
    err = SbError()
    buf = ctypes.create_string_buffer(8192)
    rc = _native.lib().sb_execute_source_rows(prepared.ptr, resources.handle if resources is not None else None,
                                              int(device), ctypes.c_void_p(int(source_ptr)), int(row_begin),
                                              int(row_end), ctypes.c_void_p(int(destination_ptr)),
                                              ctypes.byref(opts), buf, 8192, ctypes.byref(err))
    import json

    report = json.loads(buf.value.decode())
    if rc:
        _raise_transfer(err)
    return MappingProxyType(report)


def execute_source_shards(prepared: DispatchTemplate, source_ptrs, row_bounds, destination_ptr: int, *,
                          device: int, resources=None, caller_stream=None, async_completion=False):
    """All source rows as consecutive blocks in device memory (this GPU's or
    peers'): block j at ``source_ptrs[j]`` holds rows
    ``[row_bounds[j], row_bounds[j + 1])``; writes the whole result to
    ``destination_ptr``, in one tile launch where the plan allows."""
    n = len(source_ptrs)
    if len(row_bounds) != n + 1:
        raise ValueError("row_bounds needs one more entry than source_ptrs")
    ptrs = (ctypes.c_void_p * n)(*[int(p) for p in source_ptrs])
    bounds = (ctypes.c_int64 * (n + 1))(*[int(b) for b in row_bounds])
    opts = _options(4, "auto", 0, caller_stream, async_completion)
    err = SbError()
    buf = ctypes.create_string_buffer(8192)
    rc = _native.lib().sb_execute_source_shards(prepared.ptr, resources.handle if resources is not None else None,
                                                int(device), ptrs, bounds, n, ctypes.c_void_p(int(destination_ptr)),
                                                ctypes.byref(opts), buf, 8192, ctypes.byref(err))
    import json

    report = json.loads(buf.value.decode())
    if rc:
        _raise_transfer(err)
    return MappingProxyType(report)


def ipc_handle(device_ptr: int):
    """``(handle, offset)``: the 64-byte CUDA IPC handle of the allocation
    holding ``device_ptr`` and the pointer's byte offset in it."""
    h = (ctypes.c_uint8 * 64)()
    off = ctypes.c_uint64()
    err = SbError()
    if _native.lib().sb_ipc_handle(ctypes.c_void_p(int(device_ptr)), h, ctypes.byref(off), ctypes.byref(err)):
        _raise_transfer(err)
    return bytes(h), int(off.value)


def ipc_open(handle: bytes, device: int) -> int:
    """Map another process's allocation (its IPC handle) on ``device``;
    returns the allocation's base (add the offset from ``ipc_handle``)."""
    if len(handle) != 64:
        raise ValueError("CUDA IPC handles are 64 bytes")
    h = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
    out = ctypes.c_void_p()
    err = SbError()
    if _native.lib().sb_ipc_open(h, int(device), ctypes.byref(out), ctypes.byref(err)):
        _raise_transfer(err)
    return int(out.value)


def ipc_close(device_ptr: int):
    err = SbError()
    if _native.lib().sb_ipc_close(ctypes.c_void_p(int(device_ptr)), ctypes.byref(err)):
        _raise_transfer(err)


def execute_h2d_static(prepared: DispatchTemplate, source_ptr: int, destination_ptr: int, stream=None):
    """Host -> device execution that allocates nothing, for callers that cannot
    allocate device memory: staging and parameters live in a statically
    allocated 32 MiB device array (see include/sym_b200.h). Work is ordered on
    ``stream`` (a cudaStream_t handle; None/0 = the legacy default stream).
    Calls that overlap on the GPU share that array and race."""
    err = SbError()
    if _native.lib().sb_execute_h2d_static(prepared.ptr, ctypes.c_void_p(int(source_ptr)),
                                           ctypes.c_void_p(int(destination_ptr)),
                                           ctypes.c_void_p(int(stream or 0)), ctypes.byref(err)):
        _raise_transfer(err)


class DispatchResources:
    """Typed contexts: per-device streams, HBM ring and parameter buffers,
    retained across calls (reference ``pyreloc.DispatchResources``)."""

    def __init__(self, *, max_retained_bytes=64 << 20, max_live_bytes=0, max_background_workers=64,
                 max_streams=8, max_contexts=1, max_contexts_per_device=1, acquire_timeout_ms=None):
        out = ctypes.c_void_p()
        err = SbError()
        if acquire_timeout_ms is not None and int(acquire_timeout_ms) < 0:
            raise ValueError("acquire_timeout_ms must be None or non-negative")
        # Caps that a context here meets by construction (2 streams, one
        # context per device, no background transform workers): only their
        # range is checked.
        for name, value, least in (("max_streams", max_streams, 2), ("max_contexts_per_device",
                                                                     max_contexts_per_device, 1),
                                   ("max_background_workers", max_background_workers, 1), ("max_contexts",
                                                                                           max_contexts, 1)):
            if int(value) < least:
                raise ValueError(f"{name} must be at least {least} on this executor")
        _native.lib().sb_resources_create(int(max_retained_bytes), int(max_live_bytes or 0), int(max_contexts),
                                          ctypes.byref(out), ctypes.byref(err))
        self.handle = out
        self._closed = False
        if acquire_timeout_ms is not None:
            _native.lib().sb_resources_set_acquire_timeout(self.handle, int(acquire_timeout_ms))

    def stats(self):
        return json_call(_native.lib().sb_resources_stats, self.handle)

    def streams(self, device: int):
        """(copy stream, compute stream) handles of ``device``'s context."""
        a, b = ctypes.c_void_p(), ctypes.c_void_p()
        err = SbError()
        if _native.lib().sb_resources_streams(self.handle, int(device), ctypes.byref(a), ctypes.byref(b),
                                              ctypes.byref(err)):
            _raise_transfer(err)
        return a.value or 0, b.value or 0

    def clear(self):
        err = SbError()
        if _native.lib().sb_resources_clear(self.handle, ctypes.byref(err)):
            _raise_transfer(err)

    def close(self):
        if self._closed:
            return
        err = SbError()
        rc = _native.lib().sb_resources_close(self.handle, ctypes.byref(err))
        self._closed = True
        if rc:
            _raise_transfer(err)

    @property
    def closed(self):
        return self._closed

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False

    def __del__(self):
        h = getattr(self, "handle", None)
        native = globals().get("_native")  # None once the interpreter tears modules down
        lib = getattr(native, "_lib", None)
        if h and h.value and lib is not None:
            lib.sb_resources_free(h)
            self.handle = ctypes.c_void_p()


# ---- wire v0 layout transfers (reference pyreloc.make_transfer / execute_transfer,
# libreloc/python/PyTransfer.cpp:440-461) --------------------------------------------

def prepare_transfer_template(bound: BoundPlan) -> DispatchTemplate:
    """A reusable template for a bound v0 plan (no buffers)."""
    out = ctypes.c_void_p()
    err = SbError()
    if _native.lib().sb_prepare_transfer_template(bound.ptr, ctypes.byref(out), ctypes.byref(err)):
        _raise_transfer(err)
    return DispatchTemplate(out, bound)


def _span_view(view: BufferView, elements: int) -> BufferView:
    return BufferView(view.base, view.capacity_bytes, view.offset_bytes, [int(elements)], [1], view.element_size,
                      view.kind, view.device)


def make_transfer(bound: BoundPlan, source: BufferView, destination: BufferView, direction="h2d"):
    """Validate a v0 plan against the caller's buffers; a single-use request.
    The source is read as the dense span the plan addresses, the destination
    written as the dense padded result."""
    if direction != "h2d":
        raise TransferError("implementation_unavailable", "device-to-host transfers are outside this executor")
    tmpl = prepare_transfer_template(bound)
    span = 1 + sum((e - 1) * s for e, s in zip(bound.extents, bound.src_strides))
    return prepare_dispatch_from_template(tmpl, _span_view(source, span),
                                          _span_view(destination, bound.total_bytes // bound.element_size))


def execute_transfer(request: DispatchRequest, caller_stream=None, n_buffers=4, n_streams=2, gather_threads=None,
                     *, resources=None, route="auto", chunk_size=0, async_completion=False):
    """Run a prepared layout transfer (GPU-only, like execute_dispatch)."""
    return execute_dispatch(request, caller_stream=caller_stream, n_buffers=n_buffers, resources=resources,
                            route=route, chunk_size=chunk_size, async_completion=async_completion)


# ---------------------------------------------------------------------------
# consumer-sized groups and asynchronous completion
# (reference pyreloc: prepare_dispatch_group / execute_dispatch_group /
# submit_dispatch_group / DispatchCompletion, PyDispatch.cpp:625-700)
# ---------------------------------------------------------------------------

class DispatchGroup(_Handle):
    """A validated, single-use group of requests on one CUDA device."""

    _free = "sb_group_free"

    def __init__(self, ptr, templates):
        super().__init__(ptr)
        self.templates = templates  # kept alive with the group
        self.consumed = False
        self.failed = False
        self._executing = False

    @property
    def report(self):
        if self._executing:
            raise ValueError("report is unavailable during execution")
        return MappingProxyType(json_call(_native.lib().sb_group_report, self._ptr))


def prepare_dispatch_group(entries):
    """Validate ``(plan, source_view, destination_view, direction)`` entries
    together. ``plan`` is a typed ``DispatchTemplate`` or a layout
    ``BoundPlan`` (read through its transfer template, with the views spanned
    like ``make_transfer``). Launches nothing."""
    from ._native import SbGroupEntry

    entries = list(entries)
    if not 1 <= len(entries) <= 256:
        raise TransferError("invalid_options", "a group must contain between 1 and 256 members")
    arr = (SbGroupEntry * len(entries))()
    templates = []
    for i, (plan, source, destination, direction) in enumerate(entries):
        if direction not in _DIRECTIONS:
            raise ValueError("direction must be 'h2d' or 'd2h'")
        if isinstance(plan, BoundPlan):
            tmpl = prepare_transfer_template(plan)
            span = 1 + sum((e - 1) * s for e, s in zip(plan.extents, plan.src_strides))
            source = _span_view(source, span)
            destination = _span_view(destination, plan.total_bytes // plan.element_size)
        elif isinstance(plan, DispatchTemplate):
            tmpl = plan
        else:
            raise TypeError("group plans are dispatch templates or layout bound plans")
        templates.append(tmpl)
        arr[i].plan = tmpl.ptr
        arr[i].source = source.native()
        arr[i].destination = destination.native()
        arr[i].direction = _DIRECTIONS[direction]
    out = ctypes.c_void_p()
    err = SbError()
    if _native.lib().sb_prepare_dispatch_group(arr, len(entries), ctypes.byref(out), ctypes.byref(err)):
        _raise_transfer(err)
    return DispatchGroup(out, templates)


def _group_call(group):
    if not isinstance(group, DispatchGroup):
        raise TypeError("expected a DispatchGroup")
    if group.consumed or group._executing:
        raise TransferError("already_executed", "dispatch groups are single-use")


def execute_dispatch_group(group, *, caller_stream=None, gather_threads=8, gather_pool=None, pinning="auto",
                           min_pinned_bytes=None, max_scratch_bytes=64 << 20, resources=None, owners=None,
                           device_layout=False, n_buffers=4, chunked_members=False, route="auto", chunk_size=0):
    """Run every member after one wait on ``caller_stream`` and complete once
    (blocking). Host-worker knobs of the reference are accepted and ignored."""
    _group_call(group)
    group._executing = True
    opts = _options(n_buffers, route, chunk_size, caller_stream, False)
    err = SbError()
    buf = ctypes.create_string_buffer(1 << 20)
    _keep = owners
    try:
        rc = _native.lib().sb_execute_dispatch_group(group.ptr, resources.handle if resources is not None else None,
                                                     ctypes.byref(opts), buf, 1 << 20, ctypes.byref(err))
    finally:
        group._executing = False
        group.consumed = True
        del _keep
    if rc:
        group.failed = True
        _raise_transfer(err, owners)
    import json

    return MappingProxyType(json.loads(buf.value.decode()))


class DispatchCompletion(_Handle):
    """The pending completion of a submitted group. ``wait()`` blocks the
    host; ``wait_stream(stream)`` orders a consumer stream after the group
    without blocking; ``query()`` polls. Buffer owners are held until the
    group is known complete. Dropping the handle waits for the group."""

    _free = "sb_completion_free"

    def __init__(self, ptr, group, owners):
        super().__init__(ptr)
        self._group = group
        self._owners = owners

    def _done(self):
        self._owners = None

    def wait(self):
        err = SbError()
        if _native.lib().sb_completion_wait(self._ptr, ctypes.byref(err)):
            owners = self._owners
            self._done()
            _raise_transfer(err, owners)
        self._done()

    def query(self):
        done = ctypes.c_int32()
        err = SbError()
        if _native.lib().sb_completion_query(self._ptr, ctypes.byref(done), ctypes.byref(err)):
            owners = self._owners
            self._done()
            _raise_transfer(err, owners)
        if done.value:
            self._done()
        return bool(done.value)

    def wait_stream(self, stream):
        err = SbError()
        if _native.lib().sb_completion_wait_stream(self._ptr, ctypes.c_void_p(int(stream or 0)),
                                                   ctypes.byref(err)):
            _raise_transfer(err)

    def __reduce_ex__(self, protocol):
        raise TypeError("dispatch completions cannot be serialized")


def submit_dispatch_group(group, *, caller_stream=None, gather_threads=8, gather_pool=None, pinning="auto",
                          min_pinned_bytes=None, max_scratch_bytes=64 << 20, resources=None, owners=None,
                          device_layout=False, n_buffers=4, chunked_members=False, route="auto", chunk_size=0):
    """Enqueue the group and return its ``DispatchCompletion`` without waiting."""
    _group_call(group)
    group._executing = True
    opts = _options(n_buffers, route, chunk_size, caller_stream, True)
    err = SbError()
    out = ctypes.c_void_p()
    try:
        rc = _native.lib().sb_submit_dispatch_group(group.ptr, resources.handle if resources is not None else None,
                                                    ctypes.byref(opts), ctypes.byref(out), ctypes.byref(err))
    finally:
        group._executing = False
        group.consumed = True
    if rc:
        group.failed = True
        _raise_transfer(err, owners)
    return DispatchCompletion(out, group, owners)
