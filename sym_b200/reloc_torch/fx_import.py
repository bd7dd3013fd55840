"""FX region discovery for ``RelocBackend`` (reference
``reloc_torch.fx_import.import_graph``, libreloc/python/reloc_torch/fx_import.py:551-625).

A region is a single-user chain in a Dynamo (torch-level) FX graph that
starts at a CPU tensor input, applies relocation ops, crosses to a CUDA
device exactly once (``.cuda()`` / ``.to(device)``), and may continue with
relocation ops on the device side. Its recipe is built from the ops'
semantics and the example inputs' static shapes -- nothing in the graph is
executed. Supported ops:

* layout: ``permute``, ``transpose``, ``t``, ``reshape``/``view``,
  ``flatten``, ``squeeze``, ``unsqueeze``, ``contiguous``, constant
  ``torch.nn.functional.pad``;
* values (the scalar contract's stages, bit-exact with the Torch ops they
  replace): f32 -> f16/bf16 (RNE), f16/bf16 -> f32 (exact); int8 -> f32/f16
  as a dequantize with scale 1; ``int8.float() * scale`` as a dequantize
  with that scale (a Python number, or a CPU f32 tensor input that broadcasts
  along one axis or is a single value).

The result must be dense row-major (torch's ``preserve_format`` copies keep a
permuted layout, so a transposed view needs an explicit ``contiguous()``).
Anything else is reported as an exclusion with a reason and left untouched.
"""
from __future__ import annotations

import operator
import struct
from dataclasses import dataclass

from .recipe import BindingParam, Cast, Dequantize, Fill, InlineParam, Pad, Recipe, Reshape, TensorSpec, Transpose
from .symbolic import Const, Symbol, add, dense_strides, product, product_key


@dataclass(frozen=True)
class Exclusion:
    node: str
    reason: str


@dataclass(frozen=True)
class Candidate:
    source: str          # root node (CPU tensor input)
    tail: str            # last member (its uses are redirected)
    members: tuple       # member node names, in order
    recipe: Recipe
    parameters: tuple    # node names of runtime parameter tensors, in recipe order
    device: object       # destination torch.device


@dataclass(frozen=True)
class ImportReport:
    candidates: tuple
    exclusions: tuple


class _Reject(Exception):
    def __init__(self, reason):
        super().__init__(reason)
        self.reason = reason


def _require(cond, reason):
    if not cond:
        raise _Reject(reason)


_DTYPES = {"torch.float32": "float32", "torch.float16": "float16", "torch.bfloat16": "bfloat16",
           "torch.int8": "int8"}
_CASTS = {("float32", "float16"): Cast("float16", "ieee_rne"), ("float32", "bfloat16"): Cast("bfloat16", "ieee_rne"),
          ("float16", "float32"): Cast("float32", "exact"), ("bfloat16", "float32"): Cast("float32", "exact")}
_METHOD_CASTS = {"float": "float32", "half": "float16", "bfloat16": "bfloat16"}
_ONE = InlineParam("float32", (), (0x3F800000,))


def _dtype_name(dtype):
    return _DTYPES.get(str(dtype))


def _dense(shape):
    strides, run = [], 1
    for e in reversed(shape):
        strides.append(run)
        run *= e
    return tuple(reversed(strides))


def _is_dense(shape, strides):
    return all(e == 1 or s == d for e, s, d in zip(shape, strides, _dense(shape)))


_FUNCTION_KINDS = None


def _function_kinds():
    """call_function targets -> op family: Torch functions (Dynamo graphs),
    their ATen overloads (AOT / export graphs) and the decomposed
    dequantize ops of ``torch.ops.quantized_decomposed`` when that library
    is registered (reference reloc_torch/compat.py:538-586)."""
    global _FUNCTION_KINDS
    if _FUNCTION_KINDS is not None:
        return _FUNCTION_KINDS
    import torch
    import torch.nn.functional as F

    aten = torch.ops.aten
    kinds = {torch.permute: "permute", torch.transpose: "transpose", torch.t: "t", torch.reshape: "view",
             torch.movedim: "movedim", torch.moveaxis: "movedim", torch.swapaxes: "transpose",
             torch.swapdims: "transpose", torch.unflatten: "unflatten",
             torch.flatten: "flatten", torch.squeeze: "squeeze", torch.unsqueeze: "unsqueeze", torch.clone: "clone",
             F.pad: "pad", torch._C._nn.pad: "pad", operator.mul: "mul", torch.mul: "mul",
             aten.permute.default: "permute", aten.transpose.int: "transpose", aten.t.default: "t",
             aten.view.default: "view", aten.reshape.default: "view", aten._unsafe_view.default: "view",
             aten.squeeze.default: "squeeze", aten.squeeze.dim: "squeeze", aten.squeeze.dims: "squeeze",
             aten.unsqueeze.default: "unsqueeze", aten.flatten.using_ints: "flatten", aten.clone.default: "clone",
             aten.constant_pad_nd.default: "constant_pad", aten._to_copy.default: "to", aten.to.dtype: "to",
             aten.to.device: "to"}
    try:
        qd = torch.ops.quantized_decomposed
        for op, kind in ((qd.dequantize_per_tensor, "dequantize_tensor"),
                         (qd.dequantize_per_channel, "dequantize_channel"),
                         (qd.quantize_per_tensor, "quantize_decomposed"),
                         (qd.quantize_per_channel, "quantize_decomposed")):
            kinds[op] = kind
            for name in op.overloads():
                kinds[getattr(op, name)] = kind
    except (AttributeError, RuntimeError):
        pass  # the library is not registered: no graph can hold its ops
    _FUNCTION_KINDS = kinds
    return kinds


def _kind(node):
    """The op family of an FX node, or None."""
    if node.op == "call_method":
        t = node.target
        if t in ("permute", "transpose", "t", "reshape", "view", "flatten", "squeeze", "unsqueeze", "contiguous",
                 "clone", "movedim", "unflatten"):
            return "view" if t == "reshape" else t
        if t in ("swapaxes", "swapdims"):
            return "transpose"
        if t == "moveaxis":
            return "movedim"
        if t in ("to", "cuda"):
            return "to"
        if t in _METHOD_CASTS:
            return "cast"
        if t == "mul":
            return "mul"
        return None
    if node.op == "call_function":
        if node.target is getattr and len(node.args) == 2 and node.args[1] in ("T", "mT"):
            return "attr_" + node.args[1]  # x.T (all dims reversed), x.mT (last two swapped)
        kinds = _function_kinds()
        kind = kinds.get(node.target)
        if kind is None and "quantized_decomposed" in str(node.target):
            global _FUNCTION_KINDS
            _FUNCTION_KINDS = None  # the library was registered after the first lookup
            kind = _function_kinds().get(node.target)
        return kind
    return None


def _tensor_arg(node):
    """The chain operand of a member node (first positional tensor node)."""
    if node.args and hasattr(node.args[0], "op"):
        return node.args[0]
    return None


def _mul_operands(node):
    a = node.args[0] if node.args else None
    b = node.args[1] if len(node.args) > 1 else None
    return a, b


def _ints(values, reason):
    out = []
    for v in values:
        _require(type(v) is int, reason)
        out.append(v)
    return tuple(out)


def _varargs(node, reason):
    """Dims/shape given as *args or as one tuple/list."""
    rest = list(node.args[1:])
    if len(rest) == 1 and isinstance(rest[0], (tuple, list)):
        rest = list(rest[0])
    for key in ("dims", "shape", "size"):
        if key in node.kwargs:
            rest = list(node.kwargs[key])
    return _ints(rest, reason)


def _device_of(value):
    import torch

    if isinstance(value, torch.device):
        return value
    if isinstance(value, str):
        return torch.device(value)
    if type(value) is int:
        return torch.device("cuda", value)
    return None


class _Walk:
    """Shape / stride / dtype / device state along a chain."""

    def __init__(self, shape, dtype, inputs, sym=None):
        self.shape = tuple(shape)
        # Symbolic extents (dynamic dims of a Dynamo graph) or all constants;
        # layout decisions use the example's concrete `shape`.
        self.sym = tuple(sym) if sym is not None else tuple(Const(e) for e in self.shape)
        self.strides = _dense(self.shape)
        self.dtype = dtype
        self.device = "cpu"
        self.target_device = None
        self.ops = []
        self.parameters = []  # parameter node names in declaration order
        self.inputs = inputs  # node name -> example tensor
        self.scalars = {}  # SymInt placeholder name -> (example value, Symbol)

    # layout -------------------------------------------------------------
    def permute(self, perm):
        rank = len(self.shape)
        _require(len(perm) == rank and all(-rank <= d < rank for d in perm), "unsupported_permutation")
        perm = tuple(d % rank for d in perm)
        _require(sorted(perm) == list(range(rank)), "unsupported_permutation")
        if perm != tuple(range(rank)):
            self.ops.append(Transpose(perm))
        self.shape = tuple(self.shape[d] for d in perm)
        self.sym = tuple(self.sym[d] for d in perm)
        self.strides = tuple(self.strides[d] for d in perm)

    @property
    def symbolic(self):
        return any(not isinstance(e, Const) for e in self.sym)

    def reshape(self, target, need_dense=True, sym_target=None):
        if self.symbolic and sym_target is None:
            raise _Reject("symbolic_reshape")
        total = 1
        for e in self.shape:
            total *= e
        target = list(target)
        if target.count(-1) == 1:
            known = 1
            for e in target:
                if e != -1:
                    known *= e
            _require(known > 0 and total % known == 0, "unsupported_reshape")
            target[target.index(-1)] = total // known
        _require(all(e >= 0 for e in target), "unsupported_reshape")
        prod = 1
        for e in target:
            prod *= e
        _require(prod == total, "unsupported_reshape")
        if need_dense:
            _require(_is_dense(self.shape, self.strides), "non_dense_reshape")
        target = tuple(target)
        new_sym = tuple(sym_target) if sym_target is not None else tuple(Const(e) for e in target)
        if new_sym != self.sym:
            self.ops.append(Reshape(new_sym))
        self.shape = target
        self.sym = new_sym
        self.strides = _dense(target)

    def squeeze(self, dims):
        rank = len(self.shape)
        dims = range(rank) if dims is None else [d % rank for d in dims]
        keep = [i for i in range(rank) if not (i in dims and self.shape[i] == 1)]
        _require(keep, "rank_zero")
        # a dynamic dim that is 1 in the example need not be 1 later
        _require(all(isinstance(self.sym[i], Const) for i in range(rank) if i not in keep), "symbolic_squeeze")
        shape = tuple(self.shape[i] for i in keep)
        strides = tuple(self.strides[i] for i in keep)
        if shape != self.shape:
            self.sym = tuple(self.sym[i] for i in keep)
            self.ops.append(Reshape(self.sym))
        self.shape, self.strides = shape, strides

    def unsqueeze(self, dim):
        rank = len(self.shape)
        _require(-rank - 1 <= dim <= rank, "unsupported_view_dimension")
        dim %= rank + 1
        inner = self.strides[dim] * self.shape[dim] if dim < rank else 1
        self.shape = self.shape[:dim] + (1,) + self.shape[dim:]
        self.sym = self.sym[:dim] + (Const(1),) + self.sym[dim:]
        self.strides = self.strides[:dim] + (inner,) + self.strides[dim:]
        self.ops.append(Reshape(self.sym))

    def pad(self, widths, value):
        _require(len(widths) % 2 == 0 and len(widths) <= 2 * len(self.shape), "unsupported_padding")
        _require(all(type(w) is int and w >= 0 for w in widths), "unsupported_padding")
        fill = _fill(self.dtype, value)
        for i in range(len(widths) // 2):
            axis = len(self.shape) - 1 - i
            lo, hi = widths[2 * i], widths[2 * i + 1]
            if lo or hi:
                self.ops.append(Pad(axis, Const(lo), Const(hi), fill))
                self.shape = self.shape[:axis] + (self.shape[axis] + lo + hi,) + self.shape[axis + 1:]
                self.sym = self.sym[:axis] + (add(add(self.sym[axis], lo), hi),) + self.sym[axis + 1:]
        self.strides = _dense(self.shape)

    # values ---------------------------------------------------------------
    def cast(self, dtype):
        if dtype == self.dtype:
            return
        if self.dtype == "int8" and dtype in ("float32", "float16", "bfloat16"):
            # int8 -> float is a dequantize by exactly 1.0 (exact in f32), then an
            # exact narrowing (every int8 is representable in f16 and bf16)
            self.ops.append(Dequantize("float32", _ONE, None, None, "affine"))
            self.dtype = "float32"
            if dtype != "float32":
                self.ops.append(_CASTS[("float32", dtype)])
                self.dtype = dtype
            return
        op = _CASTS.get((self.dtype, dtype))
        _require(op is not None, "typed_transform_unavailable")
        self.ops.append(op)
        self.dtype = dtype

    def scale(self, operand, graph_nodes):
        """``x * s`` right after an int8 -> f32 dequantize by 1: fold s in."""
        _require(self.ops and isinstance(self.ops[-1], Dequantize) and self.ops[-1].scale == _ONE
                 and self.dtype == "float32", "typed_transform_unavailable")
        _require(_is_dense(self.shape, self.strides), "non_dense_operand")
        if isinstance(operand, (int, float)) and not isinstance(operand, bool):
            bits = struct.unpack("<I", struct.pack("<f", float(operand)))[0]
            value = struct.unpack("<f", struct.pack("<I", bits))[0]
            _require(value > 0 and value != float("inf"), "unsupported_parameter")
            self.ops[-1] = Dequantize("float32", InlineParam("float32", (), (bits,)), None, None, "affine")
            return
        _require(hasattr(operand, "op"), "unsupported_parameter")
        name, shape = _parameter_source(operand, self.inputs)
        _require(name is not None, "unsupported_parameter")
        tensor = self.inputs[name]
        _require(str(tensor.dtype) == "torch.float32" and tensor.device.type == "cpu", "parameter_dtype_unsupported")
        rank = len(self.shape)
        _require(len(shape) <= rank, "unsupported_parameter")
        shape = (1,) * (rank - len(shape)) + tuple(shape)
        axes = [i for i, e in enumerate(shape) if e != 1]
        if not axes:  # one value for every element
            _require(tensor.numel() == 1, "unsupported_parameter")
            self.ops[-1] = Dequantize("float32", BindingParam(name, "float32", ()), None, None, "affine")
        else:
            _require(len(axes) == 1 and shape[axes[0]] == self.shape[axes[0]], "unsupported_parameter")
            _require(tensor.dim() == 1 or tensor.numel() == self.shape[axes[0]], "unsupported_parameter")
            self.ops[-1] = Dequantize("float32", BindingParam(name, "float32", (self.sym[axes[0]],)),
                                      None, axes[0], "affine")
        _require(name not in self.parameters, "unsupported_parameter")
        self.parameters.append(name)

    def _tensor_parameter(self, operand, dtypes, numel):
        """The name of a runtime parameter tensor (an input of the graph)."""
        _require(hasattr(operand, "op"), "unsupported_parameter")
        name, _ = _parameter_source(operand, self.inputs)
        _require(name is not None and operand.op in ("placeholder", "get_attr"), "unsupported_parameter")
        tensor = self.inputs[name]
        _require(str(tensor.dtype) in dtypes and tensor.device.type == "cpu", "parameter_dtype_unsupported")
        _require(tensor.numel() == numel and tensor.dim() <= 1, "unsupported_parameter")
        _require(name not in self.parameters, "unsupported_parameter")
        self.parameters.append(name)
        return name

    def dequantize(self, node, per_channel):
        """``quantized_decomposed.dequantize_per_tensor`` /
        ``dequantize_per_channel`` of an int8 tensor: ``(q - zp) * scale`` in
        f32 (the decomposition computes exactly this: an exact integer
        difference, then one multiply by the f32 scale), then the optional
        ``out_dtype`` narrowing."""
        import torch

        args = list(node.args) + [None] * 7
        _require(self.dtype == "int8" and args[6 if per_channel else 5] == torch.int8,
                 "typed_transform_unavailable")
        ints = ("torch.int32", "torch.int64", "torch.int16", "torch.int8")
        if per_channel:
            axis = args[3]
            _require(type(axis) is int, "unsupported_parameter")
            rank = len(self.shape)
            _require(-rank <= axis < rank, "unsupported_parameter")
            axis %= rank
            extent = self.shape[axis]
            scale = BindingParam(self._tensor_parameter(args[1], ("torch.float32",), extent), "float32",
                                 (self.sym[axis],))
            zp = None
            if args[2] is not None:
                zp = BindingParam(self._tensor_parameter(args[2], ints, extent), "int32", (self.sym[axis],))
        else:
            axis = None
            value = args[1]
            if isinstance(value, (int, float)) and not isinstance(value, bool):
                bits = struct.unpack("<I", struct.pack("<f", float(value)))[0]
                scale = InlineParam("float32", (), (bits,))
            else:
                scale = BindingParam(self._tensor_parameter(value, ("torch.float32",), 1), "float32", ())
            value = args[2]
            if type(value) is int:
                _require(-(1 << 31) <= value < (1 << 31), "unsupported_parameter")
                zp = InlineParam("int32", (), (value & 0xFFFFFFFF,)) if value else None
            else:
                zp = BindingParam(self._tensor_parameter(value, ints, 1), "int32", ())
        self.ops.append(Dequantize("float32", scale, zp, axis, "affine"))
        self.dtype = "float32"
        out_dtype = node.kwargs.get("out_dtype")
        if out_dtype is not None:
            name = _dtype_name(out_dtype)
            _require(name in ("float32", "float16", "bfloat16"), "typed_transform_unavailable")
            self.cast(name)

    def move(self, device):
        _require(device.type == "cuda" and self.device == "cpu", "unsupported_device")
        self.device = "cuda"
        self.target_device = device


def _fill(dtype, value):
    _require(type(value) in (int, float, bool), "unsupported_padding")
    try:
        if dtype == "int8":
            _require(int(value) == value and -128 <= value <= 127, "unsupported_padding")
            return Fill("int8", int(value) & 0xFF)
        if dtype == "float32":
            return Fill("float32", int.from_bytes(struct.pack("<f", value), "little"))
        if dtype == "float16":
            return Fill("float16", int.from_bytes(struct.pack("<e", value), "little"))
        _require(float(value) == 0.0, "unsupported_padding")
        return Fill("bfloat16", 0)
    except (OverflowError, struct.error):
        raise _Reject("unsupported_padding") from None


def _parameter_source(node, inputs):
    """(input name, broadcast shape) of a scale operand: an input tensor, or a
    view of one by unsqueeze / view / reshape / ``[:, None]`` indexing."""
    if node.op in ("placeholder", "get_attr"):
        t = inputs.get(node.name)
        return (node.name, tuple(t.shape)) if t is not None else (None, None)
    base = node.args[0] if node.args and hasattr(node.args[0], "op") else None
    if base is None or base.op not in ("placeholder", "get_attr") or base.name not in inputs:
        return None, None
    shape = tuple(inputs[base.name].shape)
    k = _kind(node)
    if k == "unsqueeze":
        dim = node.args[1] if len(node.args) > 1 else node.kwargs.get("dim")
        if type(dim) is not int:
            return None, None
        dim %= len(shape) + 1
        return base.name, shape[:dim] + (1,) + shape[dim:]
    if k == "view":
        target = [d for d in (node.args[1:] if len(node.args) > 2 or not isinstance(node.args[1], (tuple, list))
                              else node.args[1])]
        if all(type(d) is int for d in target) and -1 not in target:
            return base.name, tuple(target)
        return None, None
    if node.op == "call_function" and node.target is operator.getitem:
        index = node.args[1]
        index = index if isinstance(index, tuple) else (index,)
        out, dim = [], 0
        for item in index:
            if item is None:
                out.append(1)
            elif isinstance(item, slice) and item == slice(None):
                out.append(shape[dim])
                dim += 1
            else:
                return None, None
        return base.name, tuple(out) + shape[dim:]
    return None, None


def _operand(node):
    """The chain tensor of a member node: for ``mul`` the factor produced by
    an int8 -> float conversion (the only multiply that folds), else the
    first positional argument."""
    if _kind(node) == "mul":
        for x in _mul_operands(node):
            if hasattr(x, "op") and _kind(x) in ("cast", "to"):
                return x
        return None
    return _tensor_arg(node)


def _quotient(total, known):
    """``product(total) / product(known)`` as a product expression when the
    known factors cancel exactly (symbols and the constant), else None."""
    t, k = product_key(total), product_key(known)
    if t is None or k is None or k[0] == 0 or t[0] % k[0]:
        return None
    atoms = list(t[1])
    for a in k[1]:
        if a not in atoms:
            return None
        atoms.remove(a)
    return product([Const(t[0] // k[0]), *atoms])


def _view(walk, node):
    """view / reshape: integer targets, -1, and (dynamic graphs) SymInt
    placeholders as target extents. With dynamic dims the target's extents
    must multiply to the source's symbolically; a -1 is the exact quotient
    of the two products (else the chain keeps the example's sizes)."""
    rest = list(node.args[1:])
    if len(rest) == 1 and isinstance(rest[0], (tuple, list)):
        rest = list(rest[0])
    for key in ("shape", "size"):
        if key in node.kwargs:
            rest = list(node.kwargs[key])
    concrete, sym = [], []
    for v in rest:
        if type(v) is int:
            concrete.append(v)
            sym.append(Const(v) if v >= 0 else None)
        elif hasattr(v, "op") and v.name in walk.scalars:
            concrete.append(walk.scalars[v.name][0])
            sym.append(walk.scalars[v.name][1])
        else:
            raise _Reject("unsupported_symbolic_expr")
    if not walk.symbolic and all(isinstance(e, Const) or e is None for e in sym):
        walk.reshape(concrete)
        return
    _require(concrete.count(-1) <= 1, "unsupported_reshape")
    if -1 in concrete:
        i = concrete.index(-1)
        q = _quotient(walk.sym, [e for e in sym if e is not None])
        _require(q is not None, "symbolic_reshape")
        sym[i] = q
    _require(product_key(sym) == product_key(walk.sym), "symbolic_reshape")
    walk.reshape(concrete, sym_target=tuple(sym))


def _step(walk, node):
    """Apply one member node to the walk state."""
    import torch

    k = _kind(node)
    if k == "permute":
        walk.permute(_varargs(node, "unsupported_permutation"))
    elif k == "transpose":
        d0 = node.args[1] if len(node.args) > 1 else node.kwargs.get("dim0")
        d1 = node.args[2] if len(node.args) > 2 else node.kwargs.get("dim1")
        rank = len(walk.shape)
        _require(type(d0) is int and type(d1) is int, "unsupported_permutation")
        perm = list(range(rank))
        perm[d0 % rank], perm[d1 % rank] = perm[d1 % rank], perm[d0 % rank]
        walk.permute(tuple(perm))
    elif k == "t":
        _require(len(walk.shape) <= 2, "unsupported_permutation")
        walk.permute((1, 0) if len(walk.shape) == 2 else (0,))
    elif k == "attr_T":
        walk.permute(tuple(reversed(range(len(walk.shape)))))
    elif k == "attr_mT":
        rank = len(walk.shape)
        _require(rank >= 2, "unsupported_permutation")
        walk.permute(tuple(range(rank - 2)) + (rank - 1, rank - 2))
    elif k == "movedim":
        src = node.args[1] if len(node.args) > 1 else node.kwargs.get("source")
        dst = node.args[2] if len(node.args) > 2 else node.kwargs.get("destination")
        src = (src,) if type(src) is int else tuple(src) if isinstance(src, (tuple, list)) else None
        dst = (dst,) if type(dst) is int else tuple(dst) if isinstance(dst, (tuple, list)) else None
        _require(src is not None and dst is not None and len(src) == len(dst), "unsupported_permutation")
        rank = len(walk.shape)
        _ints(src + dst, "unsupported_permutation")
        _require(all(-rank <= d < rank for d in src + dst), "unsupported_permutation")
        src, dst = [d % rank for d in src], [d % rank for d in dst]
        _require(len(set(src)) == len(src) and len(set(dst)) == len(dst), "unsupported_permutation")
        # result dim dst[i] is source dim src[i]; the other dims keep their order
        perm = [None] * rank
        for a, b in zip(src, dst):
            perm[b] = a
        rest = iter(d for d in range(rank) if d not in src)
        perm = tuple(p if p is not None else next(rest) for p in perm)
        walk.permute(perm)
    elif k == "unflatten":
        dim = node.args[1] if len(node.args) > 1 else node.kwargs.get("dim")
        sizes = node.args[2] if len(node.args) > 2 else node.kwargs.get("sizes")
        _require(type(dim) is int and isinstance(sizes, (tuple, list)), "unsupported_view_dimension")
        rank = len(walk.shape)
        _require(-rank <= dim < rank, "unsupported_view_dimension")
        dim %= rank
        sizes = _ints(sizes, "unsupported_reshape")
        _require(sizes.count(-1) <= 1 and all(e >= 0 or e == -1 for e in sizes), "unsupported_reshape")
        known = [Const(e) for e in sizes if e != -1]
        if -1 in sizes:
            q = _quotient([walk.sym[dim]], known)
            _require(q is not None, "symbolic_reshape")
            part = [q if e == -1 else Const(e) for e in sizes]
        else:
            part = [Const(e) for e in sizes]
        concrete = list(walk.shape[:dim]) + list(sizes) + list(walk.shape[dim + 1:])
        sym = walk.sym[:dim] + tuple(part) + walk.sym[dim + 1:]
        _require(product_key(sym) == product_key(walk.sym), "symbolic_reshape")
        walk.reshape(concrete, sym_target=sym)
    elif k == "view":
        _view(walk, node)
    elif k == "flatten":
        rank = len(walk.shape)
        start = node.args[1] if len(node.args) > 1 else node.kwargs.get("start_dim", 0)
        end = node.args[2] if len(node.args) > 2 else node.kwargs.get("end_dim", -1)
        _require(type(start) is int and type(end) is int, "unsupported_view_dimension")
        start, end = start % rank, end % rank
        _require(start <= end, "unsupported_view_dimension")
        inner = 1
        for e in walk.shape[start:end + 1]:
            inner *= e
        walk.reshape(walk.shape[:start] + (inner,) + walk.shape[end + 1:],
                     sym_target=walk.sym[:start] + (product(walk.sym[start:end + 1]),) + walk.sym[end + 1:])
    elif k == "squeeze":
        dims = node.args[1] if len(node.args) > 1 else node.kwargs.get("dim")
        dims = None if dims is None else (dims,) if type(dims) is int else tuple(dims)
        if dims is not None:
            _ints(dims, "unsupported_view_dimension")
        walk.squeeze(dims)
    elif k == "unsqueeze":
        dim = node.args[1] if len(node.args) > 1 else node.kwargs.get("dim")
        _require(type(dim) is int, "unsupported_view_dimension")
        walk.unsqueeze(dim)
    elif k == "contiguous":
        fmt = node.kwargs.get("memory_format", torch.contiguous_format)
        _require(fmt == torch.contiguous_format, "unsupported_memory_format")
        walk.strides = _dense(walk.shape)
    elif k == "clone":
        # preserve_format keeps a dense permuted layout's strides; the
        # destination check at the end of the chain still requires a dense result
        fmt = node.kwargs.get("memory_format", torch.preserve_format)
        _require(fmt in (torch.preserve_format, torch.contiguous_format), "unsupported_memory_format")
        if fmt == torch.contiguous_format:
            walk.strides = _dense(walk.shape)
    elif k == "constant_pad":
        widths = node.args[1] if len(node.args) > 1 else node.kwargs.get("pad")
        value = node.args[2] if len(node.args) > 2 else node.kwargs.get("value", 0)
        _require(isinstance(widths, (tuple, list)), "unsupported_padding")
        walk.pad(tuple(widths), 0 if value is None else value)
    elif k in ("dequantize_tensor", "dequantize_channel"):
        walk.dequantize(node, per_channel=k == "dequantize_channel")
    elif k == "quantize_decomposed":
        # the decomposition divides by the scale (a reciprocal rounded in
        # double) and converts NaN as the platform does: not the plan
        # format's quantize, bit for bit (the reference importer excludes it too)
        raise _Reject("quantize_semantics_unproved")
    elif k == "pad":
        widths = node.args[1] if len(node.args) > 1 else node.kwargs.get("pad")
        mode = node.args[2] if len(node.args) > 2 else node.kwargs.get("mode", "constant")
        value = node.args[3] if len(node.args) > 3 else node.kwargs.get("value", 0)
        _require(mode == "constant", "unsupported_padding")
        _require(isinstance(widths, (tuple, list)), "unsupported_padding")
        walk.pad(tuple(widths), 0 if value is None else value)
    elif k == "cast":
        walk.cast(_METHOD_CASTS[node.target])
    elif k == "to":
        device, dtype = None, None
        if node.target == "cuda":
            dev = node.args[1] if len(node.args) > 1 else node.kwargs.get("device")
            if dev is None:
                device = torch.device("cuda")  # the current device at call time
            elif isinstance(dev, (str, torch.device)):
                device = _device_of(dev)
            else:
                _require(type(dev) is int, "unsupported_transfer")
                device = torch.device("cuda", dev)
        for a in list(node.args[1:]) + [node.kwargs.get("device"), node.kwargs.get("dtype")]:
            if a is None:
                continue
            if isinstance(a, torch.dtype):
                dtype = a
            elif _device_of(a) is not None:
                device = _device_of(a)
            elif isinstance(a, bool):  # non_blocking / copy positional flags
                continue
            else:
                raise _Reject("unsupported_transfer")
        _require(node.kwargs.get("memory_format", torch.preserve_format) in (torch.preserve_format,
                                                                            torch.contiguous_format),
                 "unsupported_memory_format")
        if dtype is not None:
            name = _dtype_name(dtype)
            _require(name is not None, "unsupported_dtype")
            walk.cast(name)
        if device is not None and device.type != walk.device:
            walk.move(device)
        if node.kwargs.get("memory_format") == torch.contiguous_format:
            walk.strides = _dense(walk.shape)
    elif k == "mul":
        chain = _operand(node)
        a, b = _mul_operands(node)
        walk.scale(b if a is chain else a, None)
    else:
        raise _Reject("unrecognized_fx_target")


def _member(node):
    return _kind(node) is not None


def _symbolic_shape(root, example):
    """Extents of a Dynamo placeholder: a Symbol for each dynamic dim (a bare
    SymInt symbol in the node's example metadata, at least 2 in the example so
    the captured layout decisions hold for every size), else a Const; None
    when the graph is static or a dim is an expression."""
    import torch

    meta = root.meta.get("example_value")
    if meta is None or not hasattr(meta, "shape"):
        return None
    out, dynamic = [], False
    for d, e in zip(meta.shape, example.shape):
        if isinstance(d, torch.SymInt):
            name = str(d.node.expr)
            if name.isdigit():  # a dim the capture specialized
                out.append(Const(int(name)))
                continue
            if not name.isidentifier() or int(e) < 2:
                return None
            out.append(Symbol(name))
            dynamic = True
        else:
            out.append(Const(int(d)))
    return out if dynamic else None


def _walk(members, src, dtype, inputs, sym, scalars=None):
    walk = _Walk(src.shape, dtype, inputs, sym)
    # SymInt view targets: symbols in a symbolic walk, the example's sizes in a static one
    walk.scalars = {k: (v, e if sym is not None else Const(v)) for k, (v, e) in (scalars or {}).items()}
    moves = 0
    for m in members:
        before = walk.device
        _step(walk, m)
        moves += walk.device != before
    _require(moves == 1 and walk.device == "cuda", "same_device_transfer")
    _require(_is_dense(walk.shape, walk.strides), "destination_layout")
    return walk


def import_graph(gm, example_inputs=None):
    """Discover replaceable regions of ``gm`` (read-only)."""
    import torch

    nodes = list(gm.graph.nodes)
    inputs, scalars = {}, {}
    examples = iter(example_inputs or ())
    for n in nodes:
        if n.op == "placeholder":
            value = next(examples, None)
            if isinstance(value, torch.Tensor):
                inputs[n.name] = value
            meta = n.meta.get("example_value")
            if isinstance(meta, torch.SymInt):
                hint = value.node.hint if isinstance(value, torch.SymInt) else value
                name = str(meta.node.expr)
                if type(hint) is int and name.isidentifier():
                    scalars[n.name] = (hint, Symbol(name))
        elif n.op == "get_attr":
            try:
                value = operator.attrgetter(n.target)(gm)
            except AttributeError:
                value = None
            if isinstance(value, torch.Tensor):
                inputs[n.name] = value
    candidates, exclusions, taken = [], [], set()
    for node in nodes:
        if node in taken or _kind(node) != "to":
            continue
        members = [node]
        # backwards: single-user members down to the root
        root = _operand(node)
        while root is not None and _member(root) and len(root.users) == 1 and root not in taken:
            members.insert(0, root)
            root = _operand(root)
        # forwards: single users that continue the chain
        while len(members[-1].users) == 1:
            user = next(iter(members[-1].users))
            if not _member(user) or _operand(user) is not members[-1] or user in taken:
                break
            members.append(user)
        try:
            _require(not (root is not None and _member(root) and len(root.users) > 1), "escaping_intermediate")
            _require(root is not None and root.op in ("placeholder", "get_attr") and root.name in inputs,
                     "unsupported_root")
            src = inputs[root.name]
            _require(src.device.type == "cpu", "source_not_on_cpu")
            _require(src.layout == torch.strided and not src.is_quantized and src.is_contiguous(), "source_layout")
            _require(all(type(d) is int for d in src.shape) and src.dim() > 0 and src.numel() > 0,
                     "unsupported_symbolic_expr")
            dtype = _dtype_name(src.dtype)
            _require(dtype is not None, "unsupported_dtype")
            sym = _symbolic_shape(root, src)
            try:
                walk = _walk(members, src, dtype, inputs, sym, scalars)
            except _Reject as error:
                if sym is None or not error.reason.startswith("symbolic_"):
                    raise
                sym = None  # dynamic dims the chain cannot keep: capture the example's shape
                walk = _walk(members, src, dtype, inputs, None)
            src_sym = tuple(sym) if sym is not None else tuple(Const(e) for e in src.shape)
            src_spec = TensorSpec(src_sym, dense_strides(src_sym), Const(0), dtype)
            dst_spec = TensorSpec(walk.sym, dense_strides(walk.sym), Const(0), walk.dtype)
            recipe = Recipe(src_spec, tuple(walk.ops), dst_spec, "h2d")
            candidates.append(Candidate(root.name, members[-1].name, tuple(m.name for m in members), recipe,
                                        tuple(walk.parameters), walk.target_device))
            taken.update(members)
        except _Reject as error:
            exclusions.append(Exclusion(node.name, error.reason))
    return ImportReport(tuple(candidates), tuple(exclusions))


__all__ = ("Candidate", "Exclusion", "ImportReport", "import_graph")
