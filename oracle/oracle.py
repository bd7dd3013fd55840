"""Test infrastructure only: ctypes access to the C restatement of the reference
typed executor (``oracle/typed_oracle.c``, built into ``oracle/liboracle.so``).

``Program.from_description`` takes a bound-plan description in the JSON shape
that ``oracle/ref.py`` (the reference binder) and ``sym_b200`` (this
repository's binder) both produce: the coalesced layout (extents, strides, pad
regions, fused fill), the logical result extents and, per stage, the transform,
its declared scales and zero points and the channel map. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use it.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

MAX_RANK, MAX_STAGES, MAX_TOKENS, MAX_SYMBOLS = 8, 8, 64, 32


class OracleError(RuntimeError):
    pass


class Stage(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32), ("per_channel", ctypes.c_int32),
        ("channel_is_dim", ctypes.c_int32), ("channel_dim", ctypes.c_int32),
        ("channel_length", ctypes.c_int64),
        ("scale", ctypes.POINTER(ctypes.c_float)),
        ("zero_point", ctypes.POINTER(ctypes.c_int32)),
        ("zero_point_count", ctypes.c_int64),
        ("ntokens", ctypes.c_int32),
        ("token_op", ctypes.c_int32 * MAX_TOKENS),
        ("token_value", ctypes.c_int64 * MAX_TOKENS),
    ]


class CProgram(ctypes.Structure):
    _fields_ = [
        ("rank", ctypes.c_int32),
        ("extents", ctypes.c_int64 * MAX_RANK), ("src_strides", ctypes.c_int64 * MAX_RANK),
        ("dst_strides", ctypes.c_int64 * MAX_RANK), ("pad_lo", ctypes.c_int64 * MAX_RANK),
        ("pad_hi", ctypes.c_int64 * MAX_RANK),
        ("src_width", ctypes.c_int32), ("dst_width", ctypes.c_int32),
        ("has_fill", ctypes.c_int32), ("fill_bits", ctypes.c_uint64),
        ("result_rank", ctypes.c_int32), ("result_extents", ctypes.c_int64 * MAX_RANK),
        ("nsymbols", ctypes.c_int32), ("symbols", ctypes.c_int64 * MAX_SYMBOLS),
        ("nstages", ctypes.c_int32), ("stages", Stage * MAX_STAGES),
    ]


_lib = None


def available() -> bool:
    return LIB_PATH.exists()


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OracleError(f"oracle not built: {LIB_PATH} (run make -C oracle oracle)")
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.POINTER(CProgram)
        L.orc_execute.argtypes = [P, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
        L.orc_execute_rows.argtypes = [P, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_char_p, ctypes.c_size_t]
        L.orc_narrow_f16.restype = ctypes.c_uint16
        L.orc_narrow_f16.argtypes = [ctypes.c_uint32]
        L.orc_narrow_bf16.restype = ctypes.c_uint16
        L.orc_narrow_bf16.argtypes = [ctypes.c_uint32]
        L.orc_widen_f16.restype = ctypes.c_uint32
        L.orc_widen_f16.argtypes = [ctypes.c_uint16]
        L.orc_widen_bf16.restype = ctypes.c_uint32
        L.orc_widen_bf16.argtypes = [ctypes.c_uint16]
        L.orc_quantize.restype = ctypes.c_int8
        L.orc_quantize.argtypes = [ctypes.c_uint32, ctypes.c_float]
        L.orc_dequantize.restype = ctypes.c_uint32
        L.orc_dequantize.argtypes = [ctypes.c_int8, ctypes.c_int32, ctypes.c_float]
        L.orc_reciprocal.restype = ctypes.c_float
        L.orc_reciprocal.argtypes = [ctypes.c_float]
        _lib = L
    return _lib


# Stage op codes (typed_oracle.h) from (transform, input width, output width).
def _stage_op(stage, in_dtype, out_dtype):
    t = stage["transform"]
    if t == 0:  # cast
        if in_dtype == "float32":
            return 1 if out_dtype == "bfloat16" else 0
        return 3 if in_dtype == "bfloat16" else 2
    return 4 if t == 1 else 5


class Program:
    """A bound typed program as the C oracle executes it."""

    def __init__(self, cprog: CProgram, keep, dst_bytes: int, row_bytes: int):
        self._c = cprog
        self._keep = keep
        self.destination_bytes = dst_bytes
        self.row_bytes = row_bytes

    @classmethod
    def from_description(cls, desc: dict, dtypes: list[str], symbols: list[int] | None = None):
        """``desc``: bound-plan description; ``dtypes``: the dtype at every stage
        boundary (source first, result last)."""
        widths = {"float32": 4, "float16": 2, "bfloat16": 2, "int8": 1}
        layout = desc["layout"]
        p = CProgram()
        r = len(layout["extents"])
        if r > MAX_RANK:
            raise OracleError("rank too large")
        p.rank = r
        for k in range(r):
            p.extents[k] = layout["extents"][k]
            p.src_strides[k] = layout["src_strides"][k]
            p.dst_strides[k] = layout["dst_strides"][k]
        fills = set()
        for pad in layout["pads"]:
            p.pad_lo[pad["axis"]] = pad["lo"]
            p.pad_hi[pad["axis"]] = pad["hi"]
            fills.add(pad["fill"])
        if len(fills) > 1:
            raise OracleError("mixed fills")
        if fills:
            p.has_fill = 1
            p.fill_bits = fills.pop()
        p.src_width = widths[dtypes[0]]
        p.dst_width = widths[dtypes[-1]]
        res = desc["result_extents"]
        p.result_rank = len(res)
        for j, e in enumerate(res):
            p.result_extents[j] = e
        symbols = symbols or []
        p.nsymbols = len(symbols)
        for i, s in enumerate(symbols):
            p.symbols[i] = s
        keep = []
        p.nstages = len(desc["stages"])
        for k, st in enumerate(desc["stages"]):
            s = p.stages[k]
            s.op = _stage_op(st, dtypes[k], dtypes[k + 1])
            s.per_channel = 1 if st["per_channel"] else 0
            s.channel_is_dim = 1 if st["channel_is_dim"] else 0
            s.channel_dim = st["channel_dim"]
            s.channel_length = st["channel_length"]
            if st.get("channel_tokens"):
                toks = st["channel_tokens"]
                s.ntokens = len(toks)
                for i, (op, val) in enumerate(toks):
                    s.token_op[i] = op
                    s.token_value[i] = val
            scale = np.array(st.get("scale_bits") or [0], dtype=np.uint32).view(np.float32).copy()
            zp = np.array(st.get("zero_point") or [0], dtype=np.int32).copy()
            keep += [scale, zp]
            s.scale = scale.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
            s.zero_point = zp.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
            s.zero_point_count = len(st.get("zero_point") or [])
        row_bytes = layout["dst_strides"][0] * p.dst_width
        return cls(p, keep, desc["destination_bytes"], row_bytes)

    def execute(self, src: np.ndarray) -> np.ndarray:
        src = np.ascontiguousarray(src)
        dst = np.empty(self.destination_bytes, dtype=np.uint8)
        err = ctypes.create_string_buffer(256)
        if lib().orc_execute(ctypes.byref(self._c), src.ctypes.data, dst.ctypes.data, err, 256):
            raise OracleError(err.value.decode())
        return dst

    def execute_rows(self, src: np.ndarray, begin: int, end: int) -> np.ndarray:
        src = np.ascontiguousarray(src)
        dst = np.empty((end - begin) * self.row_bytes, dtype=np.uint8)
        err = ctypes.create_string_buffer(256)
        if lib().orc_execute_rows(ctypes.byref(self._c), src.ctypes.data, dst.ctypes.data,
                                  begin, end, err, 256):
            raise OracleError(err.value.decode())
        return dst
