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
