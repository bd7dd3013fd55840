"""Test infrastructure only: ctypes access to the reference libreloc CPU runtime.

``oracle/_ref/libreloc_ref.so`` is the reference's own C++ runtime compiled from
its sources by ``oracle/Makefile`` together with ``oracle/ref_driver.cpp``. It is
the strongest checker the parity tests have: the reference decoder
(``libreloc/src/Decode.cpp:868-1014``), binder (``libreloc/src/Bind.cpp:176-700``)
and typed CPU executor (``libreloc/src/TypedExecute.cpp:293-937``) run unmodified.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
use this module; the product never imports it.
"""
from __future__ import annotations

import ctypes
import json
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_ref" / "libreloc_ref.so"

_lib = None


class RefError(RuntimeError):
    pass


def available() -> bool:
    return LIB_PATH.exists()


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RefError(f"reference runtime not built: {LIB_PATH} (run make -C oracle ref)")
        L = ctypes.CDLL(str(LIB_PATH))
        vp, sz, i64p = ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int64)
        cpp = ctypes.POINTER(ctypes.c_char_p)
        L.ref_wire_version.argtypes = [ctypes.c_char_p, sz]
        L.ref_decode.argtypes = [ctypes.c_char_p, sz, ctypes.c_int,
                                 ctypes.POINTER(ctypes.c_uint64), ctypes.c_char_p, sz]
        L.ref_typed_prepare.restype = vp
        L.ref_typed_prepare.argtypes = [ctypes.c_char_p, sz, ctypes.c_int, cpp, i64p,
                                        ctypes.c_int, cpp, cpp, ctypes.POINTER(ctypes.c_int),
                                        i64p, ctypes.POINTER(ctypes.c_void_p),
                                        ctypes.POINTER(ctypes.c_size_t), ctypes.c_char_p, sz]
        L.ref_typed_describe.argtypes = [vp, ctypes.c_char_p, sz]
        L.ref_typed_execute.argtypes = [vp, vp, vp, ctypes.c_uint, ctypes.c_char_p, sz]
        L.ref_typed_execute_pool.argtypes = [vp, vp, vp, vp, ctypes.c_char_p, sz]
        L.ref_typed_execute_rows.argtypes = [vp, ctypes.c_int64, ctypes.c_int64, vp, vp,
                                             ctypes.c_uint, ctypes.c_char_p, sz]
        L.ref_typed_free.argtypes = [vp]
        L.ref_layout_prepare.restype = vp
        L.ref_layout_prepare.argtypes = [ctypes.c_char_p, sz, ctypes.c_int, cpp, i64p,
                                         ctypes.c_char_p, sz]
        L.ref_layout_describe.argtypes = [vp, ctypes.c_char_p, sz]
        L.ref_layout_execute.argtypes = [vp, vp, vp, ctypes.c_uint]
        L.ref_layout_free.argtypes = [vp]
        L.ref_pool_create.restype = vp
        L.ref_pool_create.argtypes = [ctypes.c_uint]
        L.ref_pool_threads.argtypes = [vp]
        L.ref_pool_free.argtypes = [vp]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def wire_version(blob: bytes):
    v = lib().ref_wire_version(blob, len(blob))
    return None if v < 0 else v


def decode_error(blob: bytes, typed: bool):
    """(offset, message) of the reference decoder's rejection, or None."""
    off = ctypes.c_uint64(0)
    buf = ctypes.create_string_buffer(512)
    rc = lib().ref_decode(blob, len(blob), 1 if typed else 0, ctypes.byref(off), buf, 512)
    return None if rc == 0 else (off.value, buf.value.decode())


def _symbols(symbols):
    names = list(symbols)
    arr_n = (ctypes.c_char_p * max(1, len(names)))(*[n.encode() for n in names])
    arr_v = (ctypes.c_int64 * max(1, len(names)))(*[int(symbols[n]) for n in names])
    return len(names), arr_n, arr_v


class TypedProgram:
    """decodeTypedPlan + bindTyped + prepareProgram of the reference."""

    def __init__(self, blob: bytes, symbols: dict, parameters: dict | None = None):
        parameters = parameters or {}
        n, names, values = _symbols(symbols)
        pn = list(parameters)
        m = max(1, len(pn))
        self._keep = []
        pnames = (ctypes.c_char_p * m)(*[p.encode() for p in pn])
        pdt = (ctypes.c_char_p * m)(*[parameters[p][0].encode() for p in pn])
        pranks = (ctypes.c_int * m)(*[len(parameters[p][1]) for p in pn])
        pext = (ctypes.c_int64 * m)(*[(parameters[p][1][0] if parameters[p][1] else 0) for p in pn])
        pbytes = (ctypes.c_void_p * m)()
        plens = (ctypes.c_size_t * m)()
        for i, p in enumerate(pn):
            data = bytes(parameters[p][2])
            buf = ctypes.create_string_buffer(data, max(1, len(data)))
            self._keep.append(buf)
            pbytes[i] = ctypes.cast(buf, ctypes.c_void_p)
            plens[i] = len(data)
        err = ctypes.create_string_buffer(1024)
        self._h = lib().ref_typed_prepare(blob, len(blob), n, names, values, len(pn), pnames,
                                          pdt, pranks, pext, pbytes, plens, err, 1024)
        if not self._h:
            raise RefError(err.value.decode())
        self.info = self.describe()

    def describe(self):
        buf = ctypes.create_string_buffer(1 << 20)
        lib().ref_typed_describe(self._h, buf, 1 << 20)
        return json.loads(buf.value.decode())

    def execute(self, src: np.ndarray, threads: int = 1) -> np.ndarray:
        src = np.ascontiguousarray(src)
        dst = np.empty(self.info["destination_bytes"], dtype=np.uint8)
        err = ctypes.create_string_buffer(512)
        if lib().ref_typed_execute(self._h, _ptr(src), _ptr(dst), threads, err, 512):
            raise RefError(err.value.decode())
        return dst

    def execute_into(self, src: np.ndarray, dst: np.ndarray, pool=None, threads: int = 1):
        err = ctypes.create_string_buffer(512)
        if pool is not None:
            rc = lib().ref_typed_execute_pool(self._h, _ptr(src), _ptr(dst), pool.handle, err, 512)
        else:
            rc = lib().ref_typed_execute(self._h, _ptr(src), _ptr(dst), threads, err, 512)
        if rc:
            raise RefError(err.value.decode())

    def execute_rows(self, src: np.ndarray, begin: int, end: int, threads: int = 1) -> np.ndarray:
        """executeHostChunk over physical outer rows [begin, end) of the bound layout."""
        layout = self.info["layout"]
        width = self.info["cuts"][-1]["bytes"] // self.info["cuts"][-1]["elements"]
        row_bytes = layout["dst_strides"][0] * width
        dst = np.empty((end - begin) * row_bytes, dtype=np.uint8)
        err = ctypes.create_string_buffer(512)
        if lib().ref_typed_execute_rows(self._h, begin, end, _ptr(np.ascontiguousarray(src)),
                                        _ptr(dst), threads, err, 512):
            raise RefError(err.value.decode())
        return dst

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.ref_typed_free(self._h)
            self._h = None


class LayoutPlan:
    """decodePlan + bind of the reference (wire v0)."""

    def __init__(self, blob: bytes, symbols: dict):
        n, names, values = _symbols(symbols)
        err = ctypes.create_string_buffer(1024)
        self._h = lib().ref_layout_prepare(blob, len(blob), n, names, values, err, 1024)
        if not self._h:
            raise RefError(err.value.decode())
        buf = ctypes.create_string_buffer(1 << 16)
        lib().ref_layout_describe(self._h, buf, 1 << 16)
        self.info = json.loads(buf.value.decode())

    def execute(self, src: np.ndarray, threads: int = 1) -> np.ndarray:
        dst = np.empty(self.info["total_bytes"], dtype=np.uint8)
        lib().ref_layout_execute(self._h, _ptr(np.ascontiguousarray(src)), _ptr(dst), threads)
        return dst

    def execute_into(self, src: np.ndarray, dst: np.ndarray, threads: int = 0):
        lib().ref_layout_execute(self._h, _ptr(src), _ptr(dst), threads)

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.ref_layout_free(self._h)
            self._h = None


class GatherPool:
    """The reference's persistent worker pool (libreloc/include/reloc/GatherPool.h:27)."""

    def __init__(self, threads: int = 0):
        self.handle = ctypes.c_void_p(lib().ref_pool_create(threads))
        self.threads = lib().ref_pool_threads(self.handle)

    def close(self):
        if self.handle:
            lib().ref_pool_free(self.handle)
            self.handle = None

    def __del__(self):
        if getattr(self, "handle", None) and _lib is not None:
            self.close()


def default_threads() -> int:
    return len(os.sched_getaffinity(0))
