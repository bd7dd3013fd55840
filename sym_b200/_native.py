"""ctypes binding of the drop-in C-ABI (include/sym_b200.h, libsb_runtime.so).

The product path has no fallback: if the native library is missing, importing
anything that executes plans raises ``NativeLibraryMissing`` instead of
running elsewhere.
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "_lib"
RUNTIME_LIB = LIB_DIR / "libsb_runtime.so"
CUDA_LIB = LIB_DIR / "libsb_cuda.so"


class NativeLibraryMissing(ImportError):
    pass


class SbError(ctypes.Structure):
    _fields_ = [("code", ctypes.c_char * 48), ("message", ctypes.c_char * 456), ("offset", ctypes.c_int64)]


class SbView(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_uint64), ("capacity_bytes", ctypes.c_uint64), ("offset_bytes", ctypes.c_uint64),
        ("kind", ctypes.c_int32), ("device", ctypes.c_int32), ("rank", ctypes.c_int32),
        ("element_size", ctypes.c_uint32), ("extents", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8),
    ]


class SbOptions(ctypes.Structure):
    _fields_ = [
        ("n_buffers", ctypes.c_int32), ("route", ctypes.c_int32), ("chunk_bytes", ctypes.c_uint64),
        ("caller_stream", ctypes.c_void_p), ("has_caller_stream", ctypes.c_int32),
        ("async_completion", ctypes.c_int32),
    ]


class SbGroupEntry(ctypes.Structure):
    _fields_ = [("plan", ctypes.c_void_p), ("source", SbView), ("destination", SbView), ("direction", ctypes.c_int32)]


ROUTES = {"auto": 0, "dma_ring": 1, "zero_copy": 2, "staged": 3}

_lib = None


def lib():
    """The loaded runtime library (built in-tree by ``python -m sym_b200.build``)."""
    global _lib
    if _lib is not None:
        return _lib
    if not RUNTIME_LIB.exists() or not CUDA_LIB.exists():
        raise NativeLibraryMissing(
            f"sym_b200 native libraries are not built ({RUNTIME_LIB}); run `python -m sym_b200.build`")
    L = ctypes.CDLL(str(RUNTIME_LIB))
    vp, sz, i32, i64, u64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64
    ep = ctypes.POINTER(SbError)
    cpp = ctypes.POINTER(ctypes.c_char_p)
    pp = ctypes.POINTER(ctypes.c_void_p)
    sig = {
        "sb_version": (ctypes.c_char_p, []),
        "sb_kernel_launches": (u64, []),
        "sb_wire_version": (ctypes.c_int, [ctypes.c_char_p, sz]),
        "sb_load_plan": (ctypes.c_int, [ctypes.c_char_p, sz, pp, ep]),
        "sb_load_typed_plan": (ctypes.c_int, [ctypes.c_char_p, sz, pp, ep]),
        "sb_plan_describe": (ctypes.c_int, [vp, ctypes.c_char_p, sz]),
        "sb_plan_free": (None, [vp]),
        "sb_bind": (ctypes.c_int, [vp, i32, cpp, ctypes.POINTER(i64), pp, ep]),
        "sb_bind_typed": (ctypes.c_int, [vp, i32, cpp, ctypes.POINTER(i64), i32, cpp, cpp,
                                         ctypes.POINTER(i32), ctypes.POINTER(i64), pp,
                                         ctypes.POINTER(sz), pp, ep]),
        "sb_bound_describe": (ctypes.c_int, [vp, ctypes.c_char_p, sz]),
        "sb_bound_free": (None, [vp]),
        "sb_query_capability": (ctypes.c_int, [vp, i32, i32, ctypes.c_char_p, sz, ep]),
        "sb_prepare_dispatch_template": (ctypes.c_int, [vp, i32, i32, ctypes.c_char_p, pp, ep]),
        "sb_template_describe": (ctypes.c_int, [vp, ctypes.c_char_p, sz]),
        "sb_prepare_transfer_template": (ctypes.c_int, [vp, pp, ep]),
        "sb_template_free": (None, [vp]),
        "sb_prepare_dispatch": (ctypes.c_int, [vp, ctypes.POINTER(SbView), ctypes.POINTER(SbView), pp, ep]),
        "sb_execute_dispatch": (ctypes.c_int, [vp, vp, ctypes.POINTER(SbOptions), ctypes.c_char_p, sz, ep]),
        "sb_request_free": (None, [vp]),
        "sb_execute_rows": (ctypes.c_int, [vp, vp, i32, vp, i32, vp, i64, i64, ctypes.POINTER(SbOptions),
                                           ctypes.c_char_p, sz, ep]),
        "sb_execute_h2d_static": (ctypes.c_int, [vp, vp, vp, vp, ep]),
        "sb_execute_source_rows": (ctypes.c_int, [vp, vp, i32, vp, i64, i64, vp, ctypes.POINTER(SbOptions),
                                                  ctypes.c_char_p, sz, ep]),
        "sb_execute_source_shards": (ctypes.c_int, [vp, vp, i32, ctypes.POINTER(vp), ctypes.POINTER(i64), i32, vp,
                                                    ctypes.POINTER(SbOptions), ctypes.c_char_p, sz, ep]),
        "sb_ipc_handle": (ctypes.c_int, [vp, ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(u64), ep]),
        "sb_ipc_open": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint8), i32, pp, ep]),
        "sb_ipc_close": (ctypes.c_int, [vp, ep]),
        "sb_resources_create": (ctypes.c_int, [u64, u64, ctypes.c_uint32, pp, ep]),
        "sb_resources_stats": (ctypes.c_int, [vp, ctypes.c_char_p, sz]),
        "sb_resources_streams": (ctypes.c_int, [vp, i32, pp, pp, ep]),
        "sb_resources_clear": (ctypes.c_int, [vp, ep]),
        "sb_resources_set_acquire_timeout": (None, [vp, ctypes.c_int64]),
        "sb_resources_close": (ctypes.c_int, [vp, ep]),
        "sb_resources_free": (None, [vp]),
        "sb_prepare_dispatch_group": (ctypes.c_int, [ctypes.POINTER(SbGroupEntry), sz, pp, ep]),
        "sb_execute_dispatch_group": (ctypes.c_int, [vp, vp, ctypes.POINTER(SbOptions), ctypes.c_char_p, sz, ep]),
        "sb_submit_dispatch_group": (ctypes.c_int, [vp, vp, ctypes.POINTER(SbOptions), pp, ep]),
        "sb_group_report": (ctypes.c_int, [vp, ctypes.c_char_p, sz]),
        "sb_group_free": (None, [vp]),
        "sb_completion_wait": (ctypes.c_int, [vp, ep]),
        "sb_completion_query": (ctypes.c_int, [vp, ctypes.POINTER(i32), ep]),
        "sb_completion_wait_stream": (ctypes.c_int, [vp, vp, ep]),
        "sb_completion_free": (None, [vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


_cuda = None


def cuda_layer():
    """The thin CUDA layer (libsb_cuda.so, include/sb_cuda.h), loaded by the
    runtime library; for its wait-limit setting and the test hooks that
    inject failures (``sbc_test_fault_mode``, ``sbc_test_withhold_tile``)."""
    global _cuda
    if _cuda is not None:
        return _cuda
    lib()
    L = ctypes.CDLL(str(CUDA_LIB))
    L.sbc_test_fault_mode.restype = ctypes.c_int
    L.sbc_test_fault_mode.argtypes = [ctypes.c_int]
    L.sbc_test_withhold_tile.restype = None
    L.sbc_test_withhold_tile.argtypes = [ctypes.c_uint32, ctypes.c_uint64]
    L.sbc_set_wait_limit_ns.restype = None
    L.sbc_set_wait_limit_ns.argtypes = [ctypes.c_uint64]
    L.sbc_wait_launch_count.restype = ctypes.c_uint64
    L.sbc_wait_launch_count.argtypes = []
    _cuda = L
    return L


def error_of(err: SbError):
    return err.code.decode(), err.message.decode(), err.offset


def json_call(fn, *args, cap=1 << 16):
    """Call a describe-style function, growing the buffer until the JSON fits."""
    while True:
        buf = ctypes.create_string_buffer(cap)
        n = fn(*args, buf, cap)
        if n < cap:
            return json.loads(buf.value.decode())
        cap = n + 1
