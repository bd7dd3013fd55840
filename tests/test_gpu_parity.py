"""GPU parity: the fused sm_100a path through the drop-in C-ABI must be
bit-identical to the reference typed CPU executor on the same inputs.

The checker is the reference runtime itself (oracle/_ref) when it is built,
else the C restatement (oracle/typed_oracle.c) pinned by test_oracle.py.
Inputs are seeded; the configurations follow the benchmark configs at sizes the
checker finishes in seconds (full-size runs are covered by the bench's
size-independent checks)."""
import numpy as np
import pytest

from helpers import (bits_to_bytes, corpus_params, encode, recipe_c1, recipe_c2, recipe_c3, recipe_c4,
                     run_typed_gpu, typed_corpus)

pytestmark = pytest.mark.gpu

ROUTES = ["dma_ring", "zero_copy", "staged"]


def expected(blob, symbols, params, src):
    from oracle import oracle, ref

    if ref.available():
        return ref.TypedProgram(blob, symbols, params).execute(np.ascontiguousarray(src).view(np.uint8).reshape(-1))
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), symbols, params).describe()
    dts = [bound["stages"][0]["input_dtype"]] + [s["output_dtype"] for s in bound["stages"]]
    return oracle.Program.from_description(bound, dts).execute(np.ascontiguousarray(src).view(np.uint8).reshape(-1))


CASES = [(c, b) for c in typed_corpus() for b in c["bindings"]]


@pytest.mark.parametrize("route", ROUTES)
@pytest.mark.parametrize("case,binding", CASES, ids=[f"{c['name']}-{i}" for i, (c, b) in enumerate(CASES)])
def test_corpus_golden_on_gpu(case, binding, route):
    src = np.frombuffer(bits_to_bytes(binding["source"]["bits"], binding["source"]["dtype"]), np.uint8)
    out, rep = run_typed_gpu(bytes.fromhex(case["blob"]), binding["symbols"], corpus_params(case), src, route=route)
    assert out.tobytes() == bits_to_bytes(binding["expected"]["bits"], binding["expected"]["dtype"])
    assert rep["executed"] and rep["route"] == route


def _specials_f32(rng, n):
    x = rng.standard_normal(n).astype(np.float32)
    special = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 2.5, -2.5, 0.5, -0.5, 1e-45, -1e-45, 65504, 65520,
                        1e5, -1e5, 127.0, 128.0, -129.0, 6.4, -6.4, 6.35, 6.45], np.float32)
    x[: special.size] = special
    x[-special.size:] = special
    return x


@pytest.mark.parametrize("n", [64, 4096, 1 << 16, (1 << 20) + 64 * 7])
@pytest.mark.parametrize("route", ROUTES)
def test_c1_transpose(n, route):
    from sym_b200 import pyreloc

    blob = encode(recipe_c1())
    assert pyreloc.wire_version(blob) == 0
    # A layout-only plan executes through the typed path with an identity
    # stage-free program? No: v0 plans are checked through the layout binder;
    # the GPU path for them is exercised in test_layout_gpu.
    src = np.random.default_rng(0).uniform(-1, 1, n).astype(np.float32)
    from layout_gpu import run_layout_gpu, expected_layout

    out = run_layout_gpu(blob, {"N": n}, src, route=route)
    assert np.array_equal(out, expected_layout(blob, {"N": n}, src))


@pytest.mark.parametrize("shape", [(1, 3, 5, 7), (2, 3, 16, 24), (3, 3, 224, 224)])
@pytest.mark.parametrize("route", ROUTES)
def test_c2_nchw_to_nhwc_pad_f16(shape, route):
    blob = encode(recipe_c2(*shape))
    src = np.random.default_rng(1).uniform(0, 1, int(np.prod(shape))).astype(np.float32)
    src[:5] = [np.nan, np.inf, -np.inf, 65520.0, 1e-8]
    out, rep = run_typed_gpu(blob, {}, {}, src, route=route)
    assert np.array_equal(out, expected(blob, {}, {}, src))
    assert rep["device_kernel"] == "transpose"


def _channels_last(batch, channels, hw, pad, op):
    """NCHW f32 -> NHWC with `pad` fill channels after the value op: the
    narrow-transpose family (C2 and its neighbours)."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    shape = tuple(S.Const(x) for x in (batch, channels, hw, 1))
    src = R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), "float32")
    result_dtype = {"copy": "float32", "f16": "float16", "bf16": "bfloat16", "quantize": "int8"}[op]
    ops = [R.Transpose((0, 2, 3, 1))]
    if op in ("f16", "bf16"):
        ops.append(R.Cast(result_dtype, "ieee_rne"))
    elif op == "quantize":
        ops.append(R.Quantize("int8", R.InlineParam("float32", (), (0x3D4CCCCD,)), None, None, "symmetric_rne"))
    if pad:
        ops.append(R.Pad(3, S.Const(0), S.Const(pad), R.Fill(result_dtype, 0)))
    out = tuple(S.Const(x) for x in (batch, hw, 1, channels + pad))
    return R.Recipe(src, tuple(ops), R.TensorSpec(out, S.dense_strides(out), S.Const(0), result_dtype), "h2d")


@pytest.mark.parametrize("channels,pad", [(3, 1), (2, 0), (3, 0), (4, 0), (2, 2), (1, 1)])
@pytest.mark.parametrize("op", ["copy", "f16", "bf16", "quantize"])
@pytest.mark.parametrize("hw", [4096, 4093])
def test_narrow_channels_last(channels, pad, op, hw):
    """Every narrow variant (2-4 destination channels, with and without pad
    channels, copy / casts / per-tensor quantize) and a pixel count that is
    not a multiple of the vector width (the tiled fallback) stay
    bit-identical to the reference."""
    blob = encode(_channels_last(3, channels, hw, pad, op))
    x = _specials_f32(np.random.default_rng(5), 3 * channels * hw)
    for route in ("dma_ring", "zero_copy"):
        if op == "copy":  # no value stage: the encoder emits a layout-only (wire v0) plan
            from layout_gpu import expected_layout, run_layout_gpu

            out = run_layout_gpu(blob, {}, x, route=route)
            assert np.array_equal(out, expected_layout(blob, {}, x)), route
            continue
        out, rep = run_typed_gpu(blob, {}, {}, x, route=route)
        assert np.array_equal(out, expected(blob, {}, {}, x)), route


def _transpose_2d(rows, cols, op):
    """f32 [rows, cols] -> [cols, rows], optionally narrowed after the transpose."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    shape = (S.Const(rows), S.Const(cols))
    src = R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), "float32")
    result_dtype = {"copy": "float32", "f16": "float16", "bf16": "bfloat16"}[op]
    ops = [R.Transpose((1, 0))]
    if op != "copy":
        ops.append(R.Cast(result_dtype, "ieee_rne"))
    out = (S.Const(cols), S.Const(rows))
    return R.Recipe(src, tuple(ops), R.TensorSpec(out, S.dense_strides(out), S.Const(0), result_dtype), "h2d")


@pytest.mark.parametrize("rows,cols", [(64, 32), (128, 96), (1024, 640), (4096, 4096), (200, 96), (64, 33)])
@pytest.mark.parametrize("op", ["copy", "f16", "bf16"])
def test_f32_transposes(rows, cols, op):
    """32-bit tile transposes (TMA tiles of 32 x 64 cells where the extents
    allow, the SIMT tiles elsewhere, ring chunks of whole rows) against the
    reference."""
    blob = encode(_transpose_2d(rows, cols, op))
    x = _specials_f32(np.random.default_rng(6), rows * cols)
    for route, chunk in (("dma_ring", 0), ("dma_ring", 64 << 10), ("zero_copy", 0)):
        if op == "copy":  # layout-only plan (wire v0)
            from layout_gpu import expected_layout, run_layout_gpu

            out = run_layout_gpu(blob, {}, x, route=route, chunk_size=chunk)
            assert np.array_equal(out, expected_layout(blob, {}, x)), (route, chunk)
            continue
        out, rep = run_typed_gpu(blob, {}, {}, x, route=route, chunk_size=chunk)
        assert np.array_equal(out, expected(blob, {}, {}, x)), (route, chunk)
        assert rep["device_kernel"] == "transpose"


def _runs_recipe(shape, perm, op, pad=None, src_dtype="float32"):
    """A permutation of the outer axes that keeps the last axis last (whole
    unit-stride rows move: the runs family), then one value op, then an
    optional pad (axis, lo, hi) of an outer result axis."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    src_shape = tuple(S.Const(x) for x in shape)
    src = R.TensorSpec(src_shape, S.dense_strides(src_shape), S.Const(0), src_dtype)
    out = [shape[d] for d in perm]
    ops = [R.Transpose(tuple(perm))]
    result_dtype = src_dtype
    if op in ("f16", "bf16"):
        result_dtype = {"f16": "float16", "bf16": "bfloat16"}[op]
        ops.append(R.Cast(result_dtype, "ieee_rne"))
    elif op == "widen":
        result_dtype = "float32"
        ops.append(R.Cast("float32", "exact"))
    elif op == "quantize":
        result_dtype = "int8"
        ops.append(R.Quantize("int8", R.InlineParam("float32", (), (0x3D4CCCCD,)), None, None, "symmetric_rne"))
    elif op == "dequantize_axis1":  # one scale per result axis-1 index (an outer axis)
        result_dtype = "float32"
        ops.append(R.Dequantize("float32", R.BindingParam("scale", "float32", (S.Const(out[1]),)), None, 1,
                                "affine"))
    elif op == "dequantize_f16":
        result_dtype = "float16"
        ops.append(R.Dequantize("float32", R.InlineParam("float32", (), (0x3C23D70A,)), None, None, "affine"))
        ops.append(R.Cast("float16", "ieee_rne"))
    if pad is not None:
        axis, lo, hi = pad
        ops.append(R.Pad(axis, S.Const(lo), S.Const(hi), R.Fill(result_dtype, 0)))
        out[axis] += lo + hi
    out = tuple(S.Const(x) for x in out)
    return R.Recipe(src, tuple(ops), R.TensorSpec(out, S.dense_strides(out), S.Const(0), result_dtype), "h2d")


@pytest.mark.parametrize("shape,perm,op,pad", [
    ((2, 3, 4, 64), (0, 2, 1, 3), "copy", None),
    ((2, 3, 4, 64), (0, 2, 1, 3), "f16", None),
    ((2, 3, 4, 64), (2, 0, 1, 3), "bf16", None),
    ((2, 3, 4, 64), (0, 2, 1, 3), "quantize", None),
    ((4, 8, 2, 32), (1, 0, 2, 3), "widen", None),
    ((2, 16, 8, 128), (0, 2, 1, 3), "dequantize_axis1", None),
    ((3, 5, 96), (1, 0, 2), "dequantize_f16", None),
    ((2, 3, 4, 64), (1, 0, 2, 3), "f16", (0, 1, 2)),
    ((2, 3, 4, 64), (0, 2, 1, 3), "quantize", (2, 2, 0)),
    ((2, 3, 30), (1, 0, 2), "f16", None),          # rows not a whole number of vectors: generic kernel
    ((128, 128, 1024), (1, 0, 2), "f16", None),    # the transpose + cast latency case (warp spans of 4)
    ((4, 6, 256), (1, 0, 2), "f16", None),         # warp spans of 2 units per lane
    ((2, 3, 512), (1, 0, 2), "bf16", (0, 1, 1)),   # spans over an outer pad
    ((2, 16, 8, 512), (0, 2, 1, 3), "dequantize_axis1", None),  # a per-run scale with spans
    ((6, 4, 128), (1, 0, 2), "quantize", None),
])
def test_outer_permutation_runs(shape, perm, op, pad):
    """Permutations that move whole unit-stride rows (attention-style
    [B,S,H,D] -> [B,H,S,D], swaps of leading axes) with every value op the
    runs kernel specializes, outer pads, a per-run channel, ring chunks that
    cut the source rows, against the reference."""
    src_dtype = {"widen": "float16", "dequantize_axis1": "int8", "dequantize_f16": "int8"}.get(op, "float32")
    blob = encode(_runs_recipe(shape, perm, op, pad, src_dtype))
    rng = np.random.default_rng(11)
    n = int(np.prod(shape))
    if src_dtype == "float32":
        x = _specials_f32(rng, n)
    elif src_dtype == "float16":
        x = rng.integers(0, 1 << 16, n, dtype=np.uint16)  # every f16 pattern, NaN payloads included
    else:
        x = rng.integers(-128, 128, n, dtype=np.int8)
    params = {}
    if op == "dequantize_axis1":
        scale = np.exp(rng.normal(-3, 0.5, shape[perm[1]])).astype(np.float32)
        params = {"scale": ("float32", [shape[perm[1]]], scale.tobytes())}
    chunk_small = max(16 << 10, (n * x.itemsize) // 5)
    for route, chunk in (("dma_ring", 0), ("dma_ring", chunk_small), ("zero_copy", 0), ("staged", 0)):
        if op == "copy":  # layout-only plan (wire v0)
            from layout_gpu import expected_layout, run_layout_gpu

            out = run_layout_gpu(blob, {}, x, route=route, chunk_size=chunk)
            assert np.array_equal(out, expected_layout(blob, {}, x)), (route, chunk)
            continue
        out, rep = run_typed_gpu(blob, {}, params, x, route=route, chunk_size=chunk)
        assert np.array_equal(out, expected(blob, {}, params, x)), (route, chunk)
        assert rep["device_kernel"] == "runs"


@pytest.mark.parametrize("seq", [1, 3, 128])
@pytest.mark.parametrize("route", ROUTES)
def test_c3_quantize_dequantize(seq, route):
    rng = np.random.default_rng(2)
    n = 8 * seq * 4096
    x = _specials_f32(rng, n)
    qblob = encode(recipe_c3("quantize"))
    q, rep = run_typed_gpu(qblob, {"B": 8, "S": seq}, {}, x, route=route)
    assert np.array_equal(q, expected(qblob, {"B": 8, "S": seq}, {}, x))
    assert rep["device_kernel"] == "contiguous"
    dblob = encode(recipe_c3("dequantize"))
    y, _ = run_typed_gpu(dblob, {"B": 8, "S": seq}, {}, q, route=route)
    assert np.array_equal(y, expected(dblob, {"B": 8, "S": seq}, {}, q))


def _c4_inputs(out_f, in_f, seed=3):
    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, size=(out_f, in_f), dtype=np.int8)
    q.reshape(-1)[:4] = [-128, 127, 0, -1]
    scale = np.exp(rng.normal(-5, 0.5, out_f)).astype(np.float32)
    return q, scale


@pytest.mark.parametrize("out_f,in_f", [(3, 5), (96, 200), (257, 131), (100, 272), (72, 400), (1024, 4096),
                                         (4096, 11008)])
@pytest.mark.parametrize("route", ROUTES)
def test_c4_dequant_f16_transpose(out_f, in_f, route):
    blob = encode(recipe_c4())
    q, scale = _c4_inputs(out_f, in_f)
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    out, rep = run_typed_gpu(blob, sym, params, q, route=route, chunk_size=1 << 20)
    assert np.array_equal(out, expected(blob, sym, params, q))
    assert rep["device_kernel"] == "transpose"


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_c4_other_result_types(dtype):
    blob = encode(recipe_c4(dtype))
    q, scale = _c4_inputs(300, 520)
    sym = {"out_features": 300, "in_features": 520}
    params = {"scale": ("float32", [300], scale.tobytes())}
    out, _ = run_typed_gpu(blob, sym, params, q)
    assert np.array_equal(out, expected(blob, sym, params, q))


def test_route_auto_learns_and_stays_exact():
    from helpers import resources

    blob = encode(recipe_c4())
    q, scale = _c4_inputs(512, 1024)
    sym = {"out_features": 512, "in_features": 1024}
    params = {"scale": ("float32", [512], scale.tobytes())}
    want = expected(blob, sym, params, q)
    resources().clear()  # nothing learned for this class yet
    routes = set()
    for _ in range(6):
        out, rep = run_typed_gpu(blob, sym, params, q, route="auto")
        assert np.array_equal(out, want)
        routes.add(rep["route"])
    assert routes == {"dma_ring", "zero_copy"}


def test_route_auto_reprobes_the_slower_route():
    """Each route is measured twice (the first sample may include one-time
    allocation); after that the slower route is measured again after 4, 16
    and every 128 executions, so a stale measurement cannot decide for good."""
    from helpers import resources

    blob = encode(recipe_c4())
    q, scale = _c4_inputs(64, 256, seed=9)
    sym = {"out_features": 64, "in_features": 256}
    params = {"scale": ("float32", [64], scale.tobytes())}
    want = expected(blob, sym, params, q)
    resources().clear()  # a fresh context: nothing learned for this class yet
    routes = []
    for _ in range(4 + 128):
        out, rep = run_typed_gpu(blob, sym, params, q, route="auto")
        assert np.array_equal(out, want)
        routes.append(rep["route"])
    assert routes[:4] == ["zero_copy", "zero_copy", "dma_ring", "dma_ring"]
    assert set(routes[4:]) == {"dma_ring", "zero_copy"}  # the faster route, and the probe of the other


def expected_rows(blob, symbols, params, src, begin, end):
    from oracle import oracle, ref

    flat = np.ascontiguousarray(src).view(np.uint8).reshape(-1)
    if ref.available():
        return ref.TypedProgram(blob, symbols, params).execute_rows(flat, begin, end)
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), symbols, params).describe()
    dts = [bound["stages"][0]["input_dtype"]] + [s["output_dtype"] for s in bound["stages"]]
    return oracle.Program.from_description(bound, dts).execute_rows(flat, begin, end)


@pytest.mark.parametrize("shards", [1, 2, 3, 8])
@pytest.mark.parametrize("host_source", [True, False])
@pytest.mark.parametrize("out_f,in_f", [(320, 1000), (192, 2048)])
def test_c4_row_windows(shards, host_source, out_f, in_f):
    """Each shard produces result rows [k*in/N, (k+1)*in/N) -- the per-GPU
    window of the sharded weight fetch -- bit-identical to the reference's
    executeHostChunk of the same window."""
    import torch
    from helpers import resources
    from sym_b200 import pyreloc

    blob = encode(recipe_c4())
    q, scale = _c4_inputs(out_f, in_f, seed=11)
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    tmpl = pyreloc.prepare_dispatch_template(pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params))
    host = torch.from_numpy(q.copy()).pin_memory()
    dev_src = host.cuda()
    bounds = [in_f * k // shards for k in range(shards + 1)]
    for k in range(shards):
        b, e = bounds[k], bounds[k + 1]
        out = torch.empty((e - b) * out_f * 2, dtype=torch.uint8, device="cuda")
        src_ptr = host.data_ptr() if host_source else dev_src.data_ptr()
        pyreloc.execute_rows(tmpl, src_ptr, out.data_ptr(), b, e, device=0, host_source=host_source,
                             resources=resources(), chunk_size=64 << 10)
        assert np.array_equal(out.cpu().numpy(), expected_rows(blob, sym, params, q, b, e)), (k, b, e)


def test_pageable_source_runs_on_the_gpu():
    blob = encode(recipe_c3("quantize"))
    x = _specials_f32(np.random.default_rng(4), 8 * 5 * 4096)
    out, rep = run_typed_gpu(blob, {"B": 8, "S": 5}, {}, x, route="auto", pinned=False)
    assert np.array_equal(out, expected(blob, {"B": 8, "S": 5}, {}, x))
    assert rep["route"] in ("dma_ring", "staged")


@pytest.mark.parametrize("route,chunk", [("dma_ring", 0), ("dma_ring", 3 << 20), ("dma_ring", 11 << 20),
                                         ("staged", 0), ("auto", 0)])
def test_pageable_sources_bounce_through_pinned_buffers(route, chunk):
    """Pageable sources of 1 MiB or more are copied by host threads into
    pinned bounce buffers of 8 MiB and DMA'd from there: ring chunks that
    are not whole buffers, a tail piece and a reuse of a buffer."""
    blob = encode(recipe_c4())
    q, scale = _c4_inputs(4608, 6000, seed=12)  # 27.6 MB of int8: three buffers, one reused
    sym = {"out_features": 4608, "in_features": 6000}
    params = {"scale": ("float32", [4608], scale.tobytes())}
    out, rep = run_typed_gpu(blob, sym, params, q, route=route, pinned=False, chunk_size=chunk)
    assert np.array_equal(out, expected(blob, sym, params, q))
    assert rep["route"] in ("dma_ring", "staged")


@pytest.mark.parametrize("out_f,in_f,cuts", [(512, 1024, [0, 64, 320, 512]), (300, 256, [0, 100, 300]),
                                             (28672 // 8, 512, [0, 1792, 3584])])
def test_source_row_windows_assemble_the_result(out_f, in_f, cuts):
    """Source-row windows held in separate device buffers (as the shards of a
    multi-GPU fetch are) assemble the exact result, each launch writing only
    the cells its rows produce (the rest of the destination stays as set)."""
    import torch
    from helpers import resources
    from sym_b200 import pyreloc

    blob = encode(recipe_c4())
    q, scale = _c4_inputs(out_f, in_f, seed=21)
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    tmpl = pyreloc.prepare_dispatch_template(pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params))
    out = torch.full((in_f * out_f,), 0x7FFF, dtype=torch.int16, device="cuda")
    shards = [torch.from_numpy(q[b:e].copy()).cuda() for b, e in zip(cuts, cuts[1:])]
    for (b, e), shard in zip(zip(cuts, cuts[1:]), shards):
        rep = pyreloc.execute_source_rows(tmpl, shard.data_ptr(), b, e, out.data_ptr(), device=0,
                                          resources=resources())
        assert rep["executed"] and rep["route"] == "device"
    got = out.view(torch.uint8).cpu().numpy()
    assert np.array_equal(got, expected(blob, sym, params, q))
    with pytest.raises(pyreloc.TransferError):
        pyreloc.execute_source_rows(tmpl, shards[0].data_ptr(), 0, out_f + 1, out.data_ptr(), device=0)


@pytest.mark.parametrize("out_f,in_f,cuts,launches", [
    (512, 1024, [0, 64, 320, 512], 1),          # TMA tiles: one launch over all blocks
    (3584 * 2, 512, [0, 2816, 5696, 7168], 1),  # uneven 64-row blocks
    (300, 256, [0, 100, 300], 2),                # not 64-row blocks: one launch per block
    (256, 512, [0, 128, 128, 256], 1),           # an empty block
])
def test_source_shards_one_launch(out_f, in_f, cuts, launches):
    """All source rows as separately stored blocks (a multi-GPU fetch's
    shards) produce the exact result through one call."""
    import torch
    from helpers import resources
    from sym_b200 import pyreloc

    blob = encode(recipe_c4())
    q, scale = _c4_inputs(out_f, in_f, seed=23)
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    tmpl = pyreloc.prepare_dispatch_template(pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params))
    out = torch.empty(in_f * out_f * 2, dtype=torch.uint8, device="cuda")
    shards = [torch.from_numpy(q[b:e].copy()).cuda() if e > b else torch.empty(16, dtype=torch.int8, device="cuda")
              for b, e in zip(cuts, cuts[1:])]
    rep = pyreloc.execute_source_shards(tmpl, [s.data_ptr() for s in shards], cuts, out.data_ptr(), device=0,
                                        resources=resources())
    assert rep["kernel_launches"] == launches
    assert np.array_equal(out.cpu().numpy(), expected(blob, sym, params, q))
    with pytest.raises(pyreloc.TransferError):
        pyreloc.execute_source_shards(tmpl, [shards[0].data_ptr()], [0, out_f - 1], out.data_ptr(), device=0)
