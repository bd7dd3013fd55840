"""Recipe -> wire plan encoder (in-process replacement for ``sym-reloc-export``).

The reference compiles recipes by shelling out to its MLIR exporter
(libreloc/python/reloc_torch/compiler.py:94-134), which needs LLVM/MLIR 21.
This module folds a recipe into ONE relocation plan directly and serializes
it in the frozen wire format (docs/reloc-plan-format.md: v0 layout plans, v1
typed plans), following the reference fold semantics
(sym/dialect/reloc/Transforms/PlanBuilder.cpp):

* the identity seed: one axis per source dim, row-major source strides;
* transpose permutes axes (pads and channel coordinates travel with them);
* reshape keeps, splits (one symbolic entry ``X floordiv C`` allowed, which
  records the divisibility guard ``X mod C``) or merges contiguous runs, then
  renumbers the view (perm resets to the identity);
* pad records lo/hi and the fill with the stage it entered at;
* cast/quantize/dequantize append a value stage whose channel map is the
  operand coordinate of its axis, rewritten through later layout folds;
* finalize: destination extents = extent + lo + hi, dense destination
  strides, the inverse permutation, fused fills folded through later stages.

Every blob this encoder produces is checked by the test-suite against the
reference decoder and binder (oracle/_ref); for the reference corpus recipes
it reproduces the committed blobs.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

from . import symbolic as sx
from .recipe import (BindingParam, Cast, Dequantize, InlineParam, Pad, Quantize, Recipe, Reshape, Transpose)


class UnsupportedRecipe(ValueError):
    def __init__(self, reason, detail=""):
        super().__init__(f"{reason}: {detail}" if detail else reason)
        self.reason = reason


_TYPES = {"float32": (0, 32), "float16": (0, 16), "float64": (0, 64), "bfloat16": (1, 16), "int8": (2, 8),
          "int16": (2, 16), "int32": (2, 32), "int64": (2, 64)}
_WIDTH = {"float32": 4, "float16": 2, "bfloat16": 2, "int8": 1, "int32": 4}
_TRANSFORM = {"cast": 0, "quantize": 1, "dequantize": 2}
_POLICY = {"ieee_rne": 0, "exact": 1, "symmetric_rne": 2, "affine": 3}


# ---------------------------------------------------------------------------
# Host folding of constant fills through stages (scalar C1 contract). Only
# constants: the encoder must write the fused fill bits into the layout.
# ---------------------------------------------------------------------------

def _f32(bits):
    return struct.unpack("<f", struct.pack("<I", bits & 0xFFFFFFFF))[0]


def _bits(f):
    return struct.unpack("<I", struct.pack("<f", f))[0]


def _narrow_f16(x):
    import numpy as np

    v = np.array([x], dtype=np.uint32).view(np.float32)
    if (x & 0x7FFFFFFF) > 0x7F800000:
        return ((x >> 16) & 0x8000) | 0x7E00 | ((x >> 13) & 0x3FF)
    return int(v.astype(np.float16).view(np.uint16)[0])


def _narrow_bf16(x):
    a = x & 0x7FFFFFFF
    if a > 0x7F800000:
        return ((x >> 16) | 0x40) & 0xFFFF
    lsb = (x >> 16) & 1
    return ((x + 0x7FFF + lsb) >> 16) & 0xFFFF


def _widen_f16(h):
    import numpy as np

    if (h & 0x7C00) == 0x7C00 and (h & 0x3FF):
        return ((h & 0x8000) << 16) | 0x7F800000 | ((h & 0x3FF) << 13)
    return int(np.array([h], dtype=np.uint16).view(np.float16).astype(np.float32).view(np.uint32)[0])


def _quantize(x, scale_bits):
    import numpy as np

    inv = np.float32(1.0) / np.array([scale_bits], dtype=np.uint32).view(np.float32)[0]
    t = np.array([x], dtype=np.uint32).view(np.float32)[0] * inv
    t = np.fmax(t, np.float32(-128.0))
    t = np.fmin(t, np.float32(127.0))
    return int(np.rint(t)) & 0xFF


def _dequantize(q, zp, scale_bits):
    import numpy as np

    d = np.float32(((q ^ 0x80) - 0x80) - zp)
    y = d * np.array([scale_bits], dtype=np.uint32).view(np.float32)[0]
    return int(np.array([y], dtype=np.float32).view(np.uint32)[0])


def _sext(bits, width):
    bits &= (1 << width) - 1
    return bits - (1 << width) if bits >> (width - 1) else bits


def fold_fill(bits, stage):
    t = stage["transform"]
    if t == "cast":
        i, o = stage["in"], stage["out"]
        if i == "float32" and o == "float16":
            return _narrow_f16(bits)
        if i == "float32" and o == "bfloat16":
            return _narrow_bf16(bits)
        if i == "float16" and o == "float32":
            return _widen_f16(bits)
        if i == "bfloat16" and o == "float32":
            return (bits & 0xFFFF) << 16
        raise UnsupportedRecipe("fill_fold", f"cast {i}->{o}")
    scale = stage["scale"]
    if not isinstance(scale, InlineParam) or scale.shape != () or stage["axis"] is not None:
        raise UnsupportedRecipe("fill_fold", "a pad fill cannot fold through a per-channel or runtime-parameter stage")
    if t == "quantize":
        return _quantize(bits, scale.bits[0])
    zp = 0
    z = stage["zero_point"]
    if isinstance(z, InlineParam):
        if z.shape != ():
            raise UnsupportedRecipe("fill_fold", "per-channel zero point")
        zp = _sext(z.bits[0], {"int8": 8, "int32": 32}.get(z.dtype, 32))
    elif z is not None:
        raise UnsupportedRecipe("fill_fold", "runtime zero point")
    return _dequantize(bits, zp, scale.bits[0])


# ---------------------------------------------------------------------------
# Folding state
# ---------------------------------------------------------------------------

@dataclass
class _Axis:
    name: str
    extent: sx.Expr
    stride: sx.Expr


@dataclass
class _State:
    axes: list
    perm: list
    dtype: str
    pads: list = field(default_factory=list)     # dicts: axis, lo, hi, fill(dtype,bits), stage
    stages: list = field(default_factory=list)   # dicts
    divisibility: list = field(default_factory=list)


def _const(e):
    return e.value if isinstance(e, sx.Const) else None


def _equal(a, b):
    ka, kb = sx.product_key([a]), sx.product_key([b])
    return ka is not None and ka == kb


def _padded(st, k):
    for p in st.pads:
        if p["axis"] == k:
            return sx.add(sx.add(st.axes[k].extent, p["lo"]), p["hi"])
    return st.axes[k].extent


def _has_pad(st, k):
    return any(p["axis"] == k for p in st.pads)


def _channel_dims(st):
    return {s["channel"] for s in st.stages if s["channel"] is not None}


def _fold_transpose(st, perm):
    r = len(st.axes)
    if sorted(perm) != list(range(r)):
        raise UnsupportedRecipe("invalid_transpose", f"perm {perm} for rank {r}")
    new_of_old = [0] * r
    for k, src in enumerate(perm):
        new_of_old[src] = k
    st.axes = [st.axes[s] for s in perm]
    st.perm = [st.perm[s] for s in perm]
    for p in st.pads:
        p["axis"] = new_of_old[p["axis"]]
    for s in st.stages:
        if s["channel"] is not None:
            s["channel"] = new_of_old[s["channel"]]


def _split_axes(targets, stride):
    out = []
    running = stride
    strides = [None] * len(targets)
    for t in range(len(targets) - 1, -1, -1):
        strides[t] = running
        running = sx.mul(running, targets[t])
    for e, s in zip(targets, strides):
        out.append(_Axis("", e, s))
    return out


def _matches_split(extent, targets):
    """(ok, divisor): targets decompose extent (all constant, or one entry
    equal to extent floordiv C)."""
    cprod = 1
    symbolic = None
    for t in targets:
        c = _const(t)
        if c is not None:
            cprod *= c
            continue
        if symbolic is not None:
            return False, 0
        symbolic = t
    ev = _const(extent)
    if symbolic is None:
        return ev is not None and ev == cprod, 0
    if ev is not None:
        return False, 0
    if cprod == 1:
        return _equal(symbolic, extent), 0
    if isinstance(symbolic, sx.FloorDiv) and symbolic.divisor == cprod and symbolic.lhs == extent:
        return True, cprod
    return False, 0


def _fold_reshape(st, shape):
    targets = [sx.expression(d) for d in shape]
    old = st.axes
    chan = _channel_dims(st)
    for t in targets:
        c = _const(t)
        if c is not None and c <= 0:
            raise UnsupportedRecipe("invalid_reshape", "non-positive extent")
    new_axes, emitted, new_of_old = [], [], [-1] * len(old)
    i = j = 0
    while i < len(old) and j < len(targets):
        i_end, j_end = i + 1, j + 1
        old_prod, new_prod = [_padded(st, i)], [targets[j]]
        divisor = 0
        split_ok = False
        while sx.product_key(old_prod) != sx.product_key(new_prod) or sx.product_key(old_prod) is None:
            if i_end == i + 1:
                ok, divisor = _matches_split(_padded(st, i), targets[j:j_end])
                if ok:
                    split_ok = True
                    break
            co = [_const(x) for x in old_prod]
            cn = [_const(x) for x in new_prod]
            if None not in co and None not in cn:
                po, pn = 1, 1
                for x in co:
                    po *= x
                for x in cn:
                    pn *= x
                if po < pn:
                    if i_end == len(old):
                        raise UnsupportedRecipe("invalid_reshape", "element counts differ")
                    old_prod.append(_padded(st, i_end))
                    i_end += 1
                else:
                    if j_end == len(targets):
                        raise UnsupportedRecipe("invalid_reshape", "element counts differ")
                    new_prod.append(targets[j_end])
                    j_end += 1
            elif i_end == i + 1 and j_end < len(targets):
                new_prod.append(targets[j_end])
                j_end += 1
            elif i_end < len(old):
                old_prod.append(_padded(st, i_end))
                i_end += 1
            else:
                raise UnsupportedRecipe("invalid_reshape", "cannot match extents")
        n_old, n_new = i_end - i, j_end - j
        if not split_ok and n_old == 1 and n_new > 1:
            # products matched symbolically (X floordiv C times C): the split
            # still needs its divisibility guard
            split_ok, divisor = _matches_split(_padded(st, i), targets[j:j_end])
            if not split_ok:
                raise UnsupportedRecipe("invalid_reshape", "cannot split the axis into the target run")
        if split_ok or (n_old == 1 and n_new > 1):
            if _has_pad(st, i):
                raise UnsupportedRecipe("reshape_pad", "splitting a padded axis")
            if i in chan:
                raise UnsupportedRecipe("reshape_channel", "reshaping a per-channel axis")
            new_axes += _split_axes(targets[j:j_end], old[i].stride)
            if divisor > 1:
                entry = (old[i].extent, divisor)
                if entry not in st.divisibility and entry not in emitted:
                    emitted.append(entry)
        elif n_old == 1 and n_new == 1:
            new_of_old[i] = len(new_axes)
            new_axes.append(_Axis("", old[i].extent, old[i].stride))
        else:
            for p in range(i, i_end):
                if _has_pad(st, p):
                    raise UnsupportedRecipe("reshape_pad", "pad folded into a merged axis")
                if p in chan:
                    raise UnsupportedRecipe("reshape_channel", "reshaping a per-channel axis")
            for p in range(i, i_end - 1):
                if not _equal(old[p].stride, sx.mul(old[p + 1].stride, old[p + 1].extent)):
                    raise UnsupportedRecipe("reshape_noncontiguous", "merging non-contiguous axes")
            stride = old[i_end - 1].stride
            if n_new == 1:
                new_axes.append(_Axis("", targets[j], stride))
            else:
                new_axes += _split_axes(targets[j:j_end], stride)
        i, j = i_end, j_end
    while i < len(old) and _const(_padded(st, i)) == 1:
        if _has_pad(st, i) or i in chan:
            raise UnsupportedRecipe("invalid_reshape", "unit axis with a pad or channel")
        i += 1
    while j < len(targets) and _const(targets[j]) == 1:
        new_axes.append(_Axis("", targets[j], sx.Const(1)))
        j += 1
    if i != len(old) or j != len(targets):
        raise UnsupportedRecipe("invalid_reshape", "extents do not match")
    for k, a in enumerate(new_axes):
        a.name = f"d{k}"
    for p in st.pads:
        p["axis"] = new_of_old[p["axis"]]
    for s in st.stages:
        if s["channel"] is not None:
            s["channel"] = new_of_old[s["channel"]]
    st.axes = new_axes
    st.perm = list(range(len(new_axes)))
    st.divisibility += emitted


def _fold_pad(st, op: Pad):
    if not 0 <= op.axis < len(st.axes):
        raise UnsupportedRecipe("invalid_pad", "axis out of range")
    if _has_pad(st, op.axis):
        raise UnsupportedRecipe("invalid_pad", "two pads on one axis")
    if op.fill.dtype != st.dtype:
        raise UnsupportedRecipe("fill_type", f"fill {op.fill.dtype} on a {st.dtype} tensor")
    if op.axis in _channel_dims(st):
        raise UnsupportedRecipe("pad_channel", "pad on a per-channel axis after its stage")
    st.pads.append({"axis": op.axis, "lo": sx.expression(op.lo), "hi": sx.expression(op.hi),
                    "fill": (op.fill.dtype, op.fill.bits), "stage": len(st.stages)})


def _fold_stage(st, op):
    shape = [_padded(st, k) for k in range(len(st.axes))]
    if isinstance(op, Cast):
        stage = {"transform": "cast", "policy": op.policy, "in": st.dtype, "out": op.dtype, "shape": shape,
                 "scale": None, "zero_point": None, "axis": None, "channel": None}
    else:
        kind = "quantize" if isinstance(op, Quantize) else "dequantize"
        if op.axis is not None:
            if op.axis >= len(st.axes):
                raise UnsupportedRecipe("invalid_axis", "channel axis out of range")
            if _has_pad(st, op.axis):
                raise UnsupportedRecipe("pad_channel", "per-channel stage on a padded axis")
        stage = {"transform": kind, "policy": op.policy, "in": st.dtype, "out": op.dtype, "shape": shape,
                 "scale": op.scale, "zero_point": op.zero_point, "axis": op.axis, "channel": op.axis}
    st.stages.append(stage)
    st.dtype = op.dtype


def fold(recipe: Recipe) -> _State:
    src = recipe.source
    shape = [sx.expression(d) for d in src.shape]
    strides = sx.dense_strides(shape)
    st = _State([_Axis(f"d{k}", e, s) for k, (e, s) in enumerate(zip(shape, strides))],
                list(range(len(shape))), src.dtype)
    for op in recipe.operations:
        if isinstance(op, Transpose):
            _fold_transpose(st, list(op.perm))
        elif isinstance(op, Reshape):
            _fold_reshape(st, op.shape)
        elif isinstance(op, Pad):
            _fold_pad(st, op)
        elif isinstance(op, (Cast, Quantize, Dequantize)):
            _fold_stage(st, op)
        else:
            raise UnsupportedRecipe("unsupported_operation", type(op).__name__)
    return st


# ---------------------------------------------------------------------------
# Serialization
# ---------------------------------------------------------------------------

class _Writer:
    def __init__(self):
        self.buf = bytearray()
        self.symbols = []

    def u8(self, v):
        self.buf += struct.pack("<B", v)

    def u32(self, v):
        self.buf += struct.pack("<I", v)

    def i64(self, v):
        self.buf += struct.pack("<q", v)

    def u64(self, v):
        self.buf += struct.pack("<Q", v & 0xFFFFFFFFFFFFFFFF)

    def string(self, s):
        b = s.encode()
        self.u32(len(b))
        self.buf += b

    def sym(self, name):
        if name not in self.symbols:
            self.symbols.append(name)
        return self.symbols.index(name)

    def expr(self, e, dims=None):
        ops = []

        def walk(x):
            if isinstance(x, sx.Const):
                ops.append((0x01, x.value))
            elif isinstance(x, sx.Symbol):
                ops.append((0x00, self.sym(x.name)))
            elif isinstance(x, _Dim):
                ops.append((0x07, x.index))
            elif isinstance(x, sx.Add):
                walk(x.lhs), walk(x.rhs), ops.append((0x02, None))
            elif isinstance(x, sx.Mul):
                walk(x.lhs), walk(x.rhs), ops.append((0x04, None))
            elif isinstance(x, sx.FloorDiv):
                walk(x.lhs), ops.append((0x01, x.divisor)), ops.append((0x05, None))
            elif isinstance(x, sx.Mod):
                walk(x.lhs), ops.append((0x01, x.divisor)), ops.append((0x06, None))
            else:
                raise UnsupportedRecipe("unsupported_expression", repr(x))

        walk(sx.expression(e) if not isinstance(e, _Dim) else e)
        self.u32(len(ops))
        for code, val in ops:
            self.u8(code)
            if code == 0x01:
                self.i64(val)
            elif code in (0x00, 0x07):
                self.u32(val)

    def dtype(self, name):
        kind, bits = _TYPES[name]
        self.u8(kind)
        self.u32(bits)

    def tensor(self, extents, elem):
        self.u32(len(extents))
        for e in extents:
            self.expr(e)
        self.u32(0)  # canonical row-major
        self.expr(sx.Const(0))
        self.dtype(elem)


@dataclass(frozen=True)
class _Dim:
    index: int


def _collect_symbols(w: _Writer, st: _State, src_shape, dst_extents):
    """Pre-assign the symbol table in first-use order of the wire sections."""


def _canonical_layout(st: _State):
    """The layout in the exporter's canonical form (the reference's
    PlanCanonicalize.cpp, canonicalizePlan): adjacent axes merge to a fixpoint
    when they are neighbours in the view order (perm[k+1] == perm[k] + 1),
    contiguous on the source side (stride_k == stride_{k+1} * extent_{k+1};
    the row-major destination side then holds too) and neither carries a
    pad. Returns (axes, perm, pads) with pad axes remapped; the logical
    result and the value stages keep the unmerged dims."""
    axes = [(_Axis(a.name, a.extent, a.stride)) for a in st.axes]
    perm = list(st.perm)
    pads = [dict(p) for p in st.pads]
    changed = True
    while changed:
        changed = False
        for k in range(len(axes) - 1):
            if any(p["axis"] in (k, k + 1) for p in pads):
                continue
            if perm[k + 1] != perm[k] + 1:
                continue
            if not _equal(axes[k].stride, sx.mul(axes[k + 1].stride, axes[k + 1].extent)):
                continue
            axes[k] = _Axis(axes[k].name, sx.mul(axes[k].extent, axes[k + 1].extent), axes[k + 1].stride)
            del axes[k + 1]
            removed = perm[k] + 1
            del perm[k + 1]
            perm = [v - 1 if v > removed else v for v in perm]
            for p in pads:
                if p["axis"] > k:
                    p["axis"] -= 1
            changed = True
            break
    return axes, perm, pads


def _layout_body(w: _Writer, st: _State, src_shape, src_dtype, dst_extents, dst_dtype, fused_fills, canon):
    axes, perm, pads = canon
    layout_extents = [a.extent for a in axes]
    for p in pads:
        k = p["axis"]
        layout_extents[k] = sx.add(sx.add(layout_extents[k], p["lo"]), p["hi"])
    w.tensor(src_shape, src_dtype)
    w.tensor(layout_extents, dst_dtype)
    w.u32(len(perm))
    for p in perm:
        w.u32(p)
    dst_strides = sx.dense_strides(layout_extents)
    w.u32(len(axes))
    for k, (a, ds) in enumerate(zip(axes, dst_strides)):
        w.string(f"d{k}")  # positional names, as the exporter emits them
        w.expr(a.extent)
        w.expr(a.stride)
        w.expr(ds)
    w.u32(len(pads))
    for p, bits in zip(sorted(pads, key=lambda p: p["axis"]), fused_fills):
        w.u32(p["axis"])
        w.expr(p["lo"])
        w.expr(p["hi"])
        w.dtype(dst_dtype)
        w.u64(bits)
    w.u32(len(st.divisibility))
    for e, d in st.divisibility:
        w.expr(e)
        w.i64(d)
    w.u32(0)  # alignment
    w.u32(len(axes))
    for a in axes:
        w.u8(1 if _const(a.stride) == 1 else 0)
    # a pad's range needs a check at bind time only when its widths are
    # symbolic (their sign is unknown); the padded extent is built as
    # extent + lo + hi, so it always matches
    symbolic_pad = any(_const(p["lo"]) is None or _const(p["hi"]) is None for p in pads)
    w.u8(0)  # no_copy
    w.u8(1 if symbolic_pad else 0)
    r = len(axes)
    w.u32(r)
    w.u32(r)
    inv = [0] * r
    for k, p in enumerate(perm):
        inv[p] = k
    for k in range(r):
        w.expr(_Dim(inv[k]))


def _param(w: _Writer, p):
    if p is None:
        w.u8(0)
        return
    if isinstance(p, InlineParam):
        w.u8(1)
        w.u8(len(p.shape))
        w.dtype(p.dtype)
        w.u32(len(p.bits))
        for b in p.bits:
            w.u64(b)
        return
    w.u8(2)
    w.string(p.name)
    w.u8(len(p.extents))
    for e in p.extents:
        w.expr(e)
    w.dtype(p.dtype)


def encode(recipe: Recipe) -> bytes:
    """Fold and serialize; wire v1 when the recipe has a value stage, else v0."""
    st = fold(recipe)
    src_shape = [sx.expression(d) for d in recipe.source.shape]
    dst_extents = [_padded(st, k) for k in range(len(st.axes))]
    # fused fills in the result dtype (pads sorted by axis, as written)
    pads = sorted(st.pads, key=lambda p: p["axis"])
    fused = []
    for p in pads:
        bits = p["fill"][1]
        for s in st.stages[p["stage"]:]:
            bits = fold_fill(bits, s)
        fused.append(bits)
    w = _Writer()
    body = _Writer()
    body.symbols = w.symbols  # one shared table, first use order
    typed = bool(st.stages)
    if typed:
        body.tensor(src_shape, recipe.source.dtype)
        body.tensor(dst_extents, st.dtype)
    canon = _canonical_layout(st)
    _layout_body(body, st, src_shape, recipe.source.dtype, dst_extents, st.dtype, fused, canon)
    if typed:
        body.u32(len(st.stages))
        for s in st.stages:
            body.u8(_TRANSFORM[s["transform"]])
            body.u8(_POLICY[s["policy"]])
            body.dtype(s["in"])
            body.u8(1 if s["transform"] == "dequantize" else 0)
            body.dtype(s["out"])
            body.u8(1 if s["transform"] == "quantize" else 0)
            body.u32(len(s["shape"]))
            for e in s["shape"]:
                body.expr(e)
            _param(body, s["scale"])
            _param(body, s["zero_point"])
            body.i64(-1 if s["axis"] is None else s["axis"])
            if s["channel"] is None:
                body.u8(0)
            else:
                body.u8(1)
                body.u32(len(st.axes))
                body.expr(_Dim(s["channel"]))
        # fills name the (merged) layout axes; merging keeps the pads' order
        body.u32(len(pads))
        for p, cp in zip(pads, sorted(canon[2], key=lambda p: p["axis"])):
            body.u32(cp["axis"])
            body.u32(p["stage"])
            body.dtype(p["fill"][0])
            body.u64(p["fill"][1])
    w.buf += b"RPLN"
    w.u32(1 if typed else 0)
    w.u32(len(w.symbols))
    for name in w.symbols:
        w.string(name)
    return bytes(w.buf + body.buf)


# ---------------------------------------------------------------------------
# CompiledRecipe / CompilerClient
# ---------------------------------------------------------------------------

class CompiledRecipe:
    """A recipe with its wire plan, decoded once by the native decoder."""

    def __init__(self, recipe: Recipe, blob: bytes):
        from .. import pyreloc

        self.recipe = recipe
        self.plan_bytes = blob
        self.wire_version = pyreloc.wire_version(blob)
        self.typed = self.wire_version == 1
        self.decoded_plan = pyreloc.load_typed_plan(blob) if self.typed else pyreloc.load_plan(blob)
        self._execution_templates = _TemplateCache()

    @property
    def symbols(self):
        return self.decoded_plan.symbols

    def parameter_extents(self, bindings):
        """{name: (dtype, [concrete extents])} of every runtime parameter."""
        out = {}
        for p in self.recipe.parameter_bindings:
            out[p.name] = (p.dtype, [sx.expression(e).evaluate(bindings) for e in p.extents])
        return out

    def bind_shape(self, shape):
        """(symbol bindings, declared parameter extents) of a source shape,
        cached per shape (the per-call hot path of typed transfers)."""
        cache = self.__dict__.setdefault("_shape_cache", {})
        hit = cache.get(shape)
        if hit is None:
            bindings = self.source_symbols(shape)
            hit = (bindings, self.parameter_extents(bindings))
            if len(cache) >= 256:
                cache.clear()
            cache[shape] = hit
        bindings, declared = hit
        return dict(bindings), {k: (d, list(e)) for k, (d, e) in declared.items()}

    def source_symbols(self, shape):
        """Bind symbols from a concrete source shape (each symbol must appear
        as a bare source extent)."""
        bindings = {}
        for spec, actual in zip(self.recipe.source.shape, shape):
            e = sx.expression(spec)
            if isinstance(e, sx.Symbol):
                prev = bindings.setdefault(e.name, int(actual))
                if prev != int(actual):
                    raise UnsupportedRecipe("symbol_conflict", e.name)
        for name in self.symbols:
            if name not in bindings:
                raise UnsupportedRecipe("unbound_symbol", name)
        return bindings


class _TemplateCache:
    def __init__(self, max_entries=256):
        self._entries = {}
        self.max_entries = max_entries

    def get(self, key, _nbytes=0):
        return self._entries.get(key)

    def put(self, key, value, _nbytes=0):
        if len(self._entries) >= self.max_entries:
            self._entries.pop(next(iter(self._entries)))
        self._entries[key] = value
        return value


class CompilerClient:
    """Compile recipes in-process (no exporter subprocess)."""

    def __init__(self, *_, **__):
        self._cache = {}

    @classmethod
    def from_environment(cls, environ=None, **options):
        return cls(**options)

    @property
    def identity(self):
        return "sym_b200.reloc_torch.compiler@1"

    def compile(self, recipe: Recipe) -> CompiledRecipe:
        key = repr(recipe)
        hit = self._cache.get(key)
        if hit is None:
            hit = self._cache[key] = CompiledRecipe(recipe, encode(recipe))
        return hit
