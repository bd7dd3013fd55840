"""Randomized decoder/binder parity with the reference (CPU): seeded random
recipes (rank 1-4, a random permutation, an optional constant pad, an
optional split of one axis, one value stage with inline or runtime
parameters, per tensor or per channel) are encoded by this repository's
encoder; the product decoder/binder must accept exactly what the reference
accepts and produce its bound layout, footprints and stage arithmetic, and
the C restatement must execute them as the reference runtime does."""
import numpy as np
import pytest

from helpers import encode
from test_plan_parity import _compare_typed


def _random_case(seed):
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    rng = np.random.default_rng(seed)
    rank = int(rng.integers(1, 5))
    shape = [int(rng.integers(1, 7)) for _ in range(rank)]
    op = ["f16", "bf16", "quantize", "dequantize", "dequantize_channel", "widen"][int(rng.integers(0, 6))]
    src_dtype = {"dequantize": "int8", "dequantize_channel": "int8", "widen": "float16"}.get(op, "float32")
    src = tuple(S.Const(e) for e in shape)
    ops, cur = [], list(shape)
    if rank > 1 and rng.random() < 0.8:
        perm = tuple(int(p) for p in rng.permutation(rank))
        ops.append(R.Transpose(perm))
        cur = [cur[p] for p in perm]
    if rng.random() < 0.3 and cur[-1] % 2 == 0 and cur[-1] > 2:  # split the last axis
        cur = cur[:-1] + [2, cur[-1] // 2]
        ops.append(R.Reshape(tuple(S.Const(e) for e in cur)))
    params = {}
    if op in ("f16", "bf16"):
        dst_dtype = {"f16": "float16", "bf16": "bfloat16"}[op]
        value_op = R.Cast(dst_dtype, "ieee_rne")
    elif op == "widen":
        dst_dtype, value_op = "float32", R.Cast("float32", "exact")
    elif op == "quantize":
        dst_dtype = "int8"
        value_op = R.Quantize("int8", R.InlineParam("float32", (), (0x3D4CCCCD,)), None, None, "symmetric_rne")
    elif op == "dequantize":
        dst_dtype = "float32"
        zp = int(rng.integers(-5, 6))
        value_op = R.Dequantize("float32", R.InlineParam("float32", (), (0x3C23D70A,)),
                                R.InlineParam("int32", (), (zp & 0xFFFFFFFF,)) if zp else None, None, "affine")
    else:
        dst_dtype = "float32"
        axis = int(rng.integers(0, len(cur)))
        n = cur[axis]
        value_op = R.Dequantize("float32", R.BindingParam("scale", "float32", (S.Const(n),)), None, axis, "affine")
        params["scale"] = ("float32", [n], np.exp(rng.normal(-3, 0.5, n)).astype(np.float32).tobytes())
    ops.append(value_op)
    if rng.random() < 0.4:
        axis = int(rng.integers(0, len(cur)))
        lo, hi = int(rng.integers(0, 3)), int(rng.integers(0, 3))
        if lo or hi:
            ops.append(R.Pad(axis, S.Const(lo), S.Const(hi), R.Fill(dst_dtype, 0)))
            cur[axis] += lo + hi
    dst = tuple(S.Const(e) for e in cur)
    recipe = R.Recipe(R.TensorSpec(src, S.dense_strides(src), S.Const(0), src_dtype), tuple(ops),
                      R.TensorSpec(dst, S.dense_strides(dst), S.Const(0), dst_dtype), "h2d")
    return recipe, shape, src_dtype, params


@pytest.mark.parametrize("seed", range(128))
def test_random_recipes_bind_and_execute_like_the_reference(ref_lib, seed):
    from oracle import oracle
    from sym_b200 import pyreloc

    recipe, shape, src_dtype, params = _random_case(seed)
    try:
        blob = encode(recipe)
    except Exception as error:  # the encoder refuses the recipe: nothing to compare
        pytest.skip(f"encoder: {error}")
    try:
        theirs = ref_lib.TypedProgram(blob, {}, params)
    except ref_lib.RefError:
        with pytest.raises((pyreloc.BindError, pyreloc.DecodeError)):
            pyreloc.bind_typed(pyreloc.load_typed_plan(blob), {}, params)
        return
    _compare_typed(ref_lib, blob, {}, params)
    rng = np.random.default_rng(1000 + seed)
    n = int(np.prod(shape))
    if src_dtype == "int8":
        src = rng.integers(-128, 128, n, dtype=np.int8)
    elif src_dtype == "float16":
        src = rng.integers(0, 1 << 16, n, dtype=np.uint16)
    else:
        src = (rng.standard_normal(n) * 4).astype(np.float32)
    raw = src.view(np.uint8).reshape(-1)
    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), {}, params).describe()
    dts = [bound["stages"][0]["input_dtype"]] + [s["output_dtype"] for s in bound["stages"]]
    mine = oracle.Program.from_description(bound, dts).execute(raw)
    assert np.array_equal(mine, theirs.execute(raw))


def _random_layout(seed):
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    rng = np.random.default_rng(seed)
    rank = int(rng.integers(2, 5))
    shape = [int(rng.integers(1, 7)) for _ in range(rank)]
    dtype = ["float32", "float16", "int8"][int(rng.integers(0, 3))]
    ops, cur = [R.Transpose(tuple(int(p) for p in rng.permutation(rank)))], None
    cur = [shape[p] for p in ops[0].perm]
    if rng.random() < 0.5:
        axis = int(rng.integers(0, rank))
        lo, hi = int(rng.integers(0, 3)), int(rng.integers(1, 3))
        ops.append(R.Pad(axis, S.Const(lo), S.Const(hi), R.Fill(dtype, 0)))
        cur[axis] += lo + hi
    src = tuple(S.Const(e) for e in shape)
    dst = tuple(S.Const(e) for e in cur)
    return (R.Recipe(R.TensorSpec(src, S.dense_strides(src), S.Const(0), dtype), tuple(ops),
                     R.TensorSpec(dst, S.dense_strides(dst), S.Const(0), dtype), "h2d"), shape, dtype)


@pytest.mark.parametrize("seed", range(64))
def test_random_layout_plans_bind_and_execute_like_the_reference(ref_lib, seed):
    """Layout-only (wire v0) random permutations with pads: the product binder
    and the C restatement against the reference."""
    from oracle import oracle
    from sym_b200 import pyreloc
    from test_plan_parity import LAYOUT_KEYS

    recipe, shape, dtype = _random_layout(seed)
    blob = encode(recipe)
    assert pyreloc.wire_version(blob) == 0
    theirs = ref_lib.LayoutPlan(blob, {})
    mine = pyreloc.bind(pyreloc.load_plan(blob), {}).describe()
    for k in LAYOUT_KEYS:
        assert mine[k] == theirs.info[k], k
    width = {"float32": 4, "float16": 2, "int8": 1}[dtype]
    raw = np.random.default_rng(2000 + seed).integers(0, 256, int(np.prod(shape)) * width, dtype=np.uint8)
    desc = {"layout": mine, "result_extents": [mine["total_bytes"] // mine["element_size"]], "stages": [],
            "destination_bytes": mine["total_bytes"]}
    got = oracle.Program.from_description(desc, [dtype]).execute(raw)
    assert np.array_equal(got, theirs.execute(raw))


def _random_symbolic(seed):
    """A typed recipe whose source has one or two symbolic extents, permuted,
    optionally with a pad and a per-channel scale on a symbolic axis."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    rng = np.random.default_rng(seed)
    rank = int(rng.integers(2, 5))
    names = ["a", "b"][:int(rng.integers(1, 3))]
    sym_axes = sorted(int(x) for x in rng.choice(rank, size=len(names), replace=False))
    src = [S.Const(int(rng.integers(1, 6))) for _ in range(rank)]
    for name, ax in zip(names, sym_axes):
        src[ax] = S.Symbol(name)
    perm = tuple(int(p) for p in rng.permutation(rank))
    cur = [src[p] for p in perm]
    ops = [R.Transpose(perm)]
    per_channel = rng.random() < 0.5
    if per_channel:
        axis = int(rng.integers(0, rank))
        ops.append(R.Dequantize("float32", R.BindingParam("scale", "float32", (cur[axis],)), None, axis, "affine"))
        src_dtype, dst_dtype = "int8", "float32"
    else:
        ops.append(R.Cast("float16", "ieee_rne"))
        src_dtype, dst_dtype = "float32", "float16"
    if rng.random() < 0.5:
        axis = int(rng.integers(0, rank))
        if not (per_channel and axis == ops[1].axis):
            lo, hi = int(rng.integers(0, 3)), int(rng.integers(1, 3))
            ops.append(R.Pad(axis, S.Const(lo), S.Const(hi), R.Fill(dst_dtype, 0)))
            cur[axis] = S.add(S.add(cur[axis], lo), hi)
    recipe = R.Recipe(R.TensorSpec(tuple(src), S.dense_strides(tuple(src)), S.Const(0), src_dtype), tuple(ops),
                      R.TensorSpec(tuple(cur), S.dense_strides(tuple(cur)), S.Const(0), dst_dtype), "h2d")
    sizes = {name: int(rng.integers(1, 9)) for name in names}
    return recipe, src, sizes, per_channel, ops


@pytest.mark.parametrize("seed", range(64))
def test_random_symbolic_recipes_bind_like_the_reference(ref_lib, seed):
    """Symbols bound at random sizes: the product binder and the reference
    binder produce the same bound layout, footprints and stage arithmetic,
    and the C restatement executes like the reference runtime."""
    from oracle import oracle
    from sym_b200 import pyreloc

    recipe, src, sizes, per_channel, ops = _random_symbolic(seed)
    blob = encode(recipe)
    shape = [sizes[e.name] if hasattr(e, "name") else e.value for e in src]
    params = {}
    if per_channel:
        n = ops[1].scale.extents[0]
        n = sizes[n.name] if hasattr(n, "name") else n.value
        params["scale"] = ("float32", [n], np.exp(np.random.default_rng(seed).normal(-3, 0.5, n))
                           .astype(np.float32).tobytes())
    _compare_typed(ref_lib, blob, sizes, params)
    count = int(np.prod(shape))
    rng = np.random.default_rng(3000 + seed)
    raw = (rng.integers(-128, 128, count, dtype=np.int8) if per_channel
           else (rng.standard_normal(count) * 4).astype(np.float32)).view(np.uint8).reshape(-1)
    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sizes, params).describe()
    dts = [bound["stages"][0]["input_dtype"]] + [s["output_dtype"] for s in bound["stages"]]
    got = oracle.Program.from_description(bound, dts).execute(raw)
    assert np.array_equal(got, ref_lib.TypedProgram(blob, sizes, params).execute(raw))
