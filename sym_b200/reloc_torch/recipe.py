"""Immutable relocation recipes, independent of Torch and of compiled plans.

Same dataclasses and validation rules as the reference frontend's
``reloc_torch.recipe`` (libreloc/python/reloc_torch/recipe.py:23-188):
layout operations (Transpose, Reshape, Pad) and typed value operations (Cast,
Quantize, Dequantize) over a source TensorSpec, with stage parameters given
as exact bit patterns (InlineParam) or runtime bindings (BindingParam). A
recipe never holds a pointer.
"""
from __future__ import annotations

from dataclasses import dataclass

from .symbolic import Expr

_TENSOR_DTYPES = {"float32": 32, "float16": 16, "bfloat16": 16, "int8": 8}
_PARAM_DTYPES = {**_TENSOR_DTYPES, "int32": 32}
_CAST_POLICIES = ("ieee_rne", "exact")
_QUANT_POLICIES = ("symmetric_rne", "affine")


@dataclass(frozen=True)
class TensorSpec:
    shape: tuple
    strides: tuple
    offset: Expr | int
    dtype: str


@dataclass(frozen=True)
class Transpose:
    perm: tuple


@dataclass(frozen=True)
class Reshape:
    shape: tuple


@dataclass(frozen=True)
class Fill:
    dtype: str
    bits: int

    def __post_init__(self):
        width = _TENSOR_DTYPES.get(self.dtype)
        if width is None or type(self.bits) is not int or not 0 <= self.bits < 1 << width:
            raise ValueError("invalid fill dtype or bit pattern")


@dataclass(frozen=True)
class Pad:
    axis: int
    lo: Expr | int
    hi: Expr | int
    fill: Fill


@dataclass(frozen=True)
class InlineParam:
    dtype: str
    shape: tuple
    bits: tuple

    def __post_init__(self):
        width = _PARAM_DTYPES.get(self.dtype)
        if (width is None or type(self.shape) is not tuple or len(self.shape) > 1
                or any(type(d) is not int or d <= 0 for d in self.shape)):
            raise ValueError("invalid parameter dtype or shape")
        count = 1
        for d in self.shape:
            count *= d
        if (type(self.bits) is not tuple or len(self.bits) != count
                or any(type(b) is not int or not 0 <= b < 1 << width for b in self.bits)):
            raise ValueError("invalid parameter bit patterns")


@dataclass(frozen=True)
class BindingParam:
    name: str
    dtype: str
    extents: tuple

    def __post_init__(self):
        if (type(self.name) is not str or not self.name or self.dtype not in _PARAM_DTYPES
                or type(self.extents) is not tuple or len(self.extents) > 1):
            raise ValueError("invalid parameter binding")


@dataclass(frozen=True)
class Cast:
    dtype: str
    policy: str

    def __post_init__(self):
        if self.dtype not in _TENSOR_DTYPES or self.policy not in _CAST_POLICIES:
            raise ValueError("invalid cast dtype or policy")


def _check_quant(op):
    if op.dtype not in _TENSOR_DTYPES or op.policy not in _QUANT_POLICIES:
        raise ValueError("invalid quantization dtype or policy")
    if not isinstance(op.scale, (InlineParam, BindingParam)):
        raise ValueError("quantization scale must be an InlineParam or BindingParam")
    if op.zero_point is not None and not isinstance(op.zero_point, (InlineParam, BindingParam)):
        raise ValueError("quantization zero point must be an InlineParam, BindingParam or None")
    if op.axis is not None and (type(op.axis) is not int or op.axis < 0):
        raise ValueError("quantization axis must be None (per tensor) or a non-negative int")


@dataclass(frozen=True)
class Quantize:
    dtype: str
    scale: InlineParam | BindingParam
    zero_point: InlineParam | BindingParam | None
    axis: int | None
    policy: str

    def __post_init__(self):
        _check_quant(self)


@dataclass(frozen=True)
class Dequantize:
    dtype: str
    scale: InlineParam | BindingParam
    zero_point: InlineParam | BindingParam | None
    axis: int | None
    policy: str

    def __post_init__(self):
        _check_quant(self)


TYPED_OPERATIONS = (Cast, Quantize, Dequantize)
LAYOUT_OPERATIONS = (Transpose, Reshape, Pad)


@dataclass(frozen=True)
class Recipe:
    source: TensorSpec
    operations: tuple
    destination: TensorSpec
    direction: str

    @property
    def typed(self):
        return any(isinstance(op, TYPED_OPERATIONS) for op in self.operations)

    @property
    def indexed(self):
        return False

    @property
    def parameter_bindings(self):
        seen = []
        for op in self.operations:
            for param in (getattr(op, "scale", None), getattr(op, "zero_point", None)):
                if isinstance(param, BindingParam) and all(p.name != param.name for p in seen):
                    seen.append(param)
        return tuple(seen)


def from_json(recipe_json) -> Recipe:
    """Build a Recipe from the reference manifest's recipe JSON."""
    from .symbolic import from_json as ex

    def spec(j):
        return TensorSpec(tuple(ex(d) for d in j["shape"]), tuple(ex(d) for d in j["strides"]),
                          ex(j["offset"]), j["dtype"])

    def param(j):
        if j is None:
            return None
        if j["kind"] == "inline":
            return InlineParam(j["dtype"], tuple(j["shape"]), tuple(j["bits"]))
        return BindingParam(j["name"], j["dtype"], tuple(ex(e) for e in j["extents"]))

    ops = []
    for o in recipe_json["operations"]:
        k = o["kind"]
        if k == "transpose":
            ops.append(Transpose(tuple(o["perm"])))
        elif k == "reshape":
            ops.append(Reshape(tuple(ex(d) for d in o["shape"])))
        elif k == "pad":
            ops.append(Pad(o["axis"], ex(o["lo"]), ex(o["hi"]), Fill(o["fill"]["dtype"], o["fill"]["bits"])))
        elif k == "cast":
            ops.append(Cast(o["dtype"], o["policy"]))
        elif k == "quantize":
            ops.append(Quantize(o["dtype"], param(o["scale"]), param(o["zero_point"]), o["axis"], o["policy"]))
        elif k == "dequantize":
            ops.append(Dequantize(o["dtype"], param(o["scale"]), param(o["zero_point"]), o["axis"], o["policy"]))
        else:
            raise ValueError(f"unknown operation {k!r}")
    return Recipe(spec(recipe_json["source"]), tuple(ops), spec(recipe_json["destination"]),
                  recipe_json["direction"])
