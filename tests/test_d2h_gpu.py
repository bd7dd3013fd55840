"""Device-to-host typed transfers on the GPU (the reference's D2H rows,
Dispatch.cpp:1072-1105, here b200_fused_d2h): a device source is transformed
by the fused kernels into ring chunks (or straight into mapped pinned host
memory) and drained to the host, bit-identical to the reference executor on
the same bytes."""
import numpy as np
import pytest

from helpers import dense, encode, recipe_c2, recipe_c3, recipe_c4, resources

pytestmark = pytest.mark.gpu

ROUTES = ["auto", "dma_ring", "zero_copy", "staged"]


def _expected(blob, sym, params, src):
    from oracle import ref

    if not ref.available():
        pytest.skip("reference runtime (oracle/_ref) not built")
    return ref.TypedProgram(blob, sym, params).execute(np.ascontiguousarray(src).view(np.uint8).reshape(-1))


def _run_d2h(blob, sym, params, src, route, pinned=True, chunk=0):
    import torch
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params)
    info = bound.describe()
    tmpl = pyreloc.prepare_dispatch_template(bound, "d2h", "cuda")
    dev = torch.from_numpy(np.ascontiguousarray(src).view(np.uint8).reshape(-1).copy()).cuda()
    out = torch.empty(info["destination_bytes"], dtype=torch.uint8)
    if pinned:
        out = out.pin_memory()
    w = {"float32": 4, "float16": 2, "bfloat16": 2, "int8": 1}
    sv = pyreloc.BufferView(dev.data_ptr(), dev.numel(), 0, info["source_extents"], dense(info["source_extents"]),
                            w[info["source_dtype"]], "cuda", 0)
    dv = pyreloc.BufferView(out.data_ptr(), out.numel(), 0, info["result_extents"], dense(info["result_extents"]),
                            w[info["result_dtype"]], "host", -1)
    req = pyreloc.prepare_dispatch_from_template(tmpl, sv, dv)
    rep = pyreloc.execute_dispatch(req, resources=resources(), route=route, chunk_size=chunk)
    return out.numpy(), dict(rep)


@pytest.mark.parametrize("route", ROUTES)
@pytest.mark.parametrize("seq", [1, 64, 257])
def test_quantize_kv_block_to_host(route, seq):
    """f32 [8, S, 4096] on the GPU -> int8 on the host: a quarter of the
    bytes cross PCIe (the KV-cache eviction shape)."""
    x = np.random.default_rng(seq).standard_normal(8 * seq * 4096).astype(np.float32)
    x[:6] = [np.nan, np.inf, -np.inf, 2.5, -2.5, 6.35]
    blob, sym = encode(recipe_c3("quantize")), {"B": 8, "S": seq}
    got, rep = _run_d2h(blob, sym, {}, x, route, chunk=256 << 10)
    assert np.array_equal(got, _expected(blob, sym, {}, x))
    assert rep["implementation"].startswith("b200_fused_d2h") and rep["executed"]
    if route in ("dma_ring", "zero_copy", "staged"):
        assert rep["route"] == route


@pytest.mark.parametrize("route", ROUTES)
@pytest.mark.parametrize("out_f,in_f", [(96, 200), (1024, 4096), (257, 131)])
def test_dequant_transpose_to_host(route, out_f, in_f):
    rng = np.random.default_rng(out_f)
    q = rng.integers(-128, 128, size=(out_f, in_f), dtype=np.int8)
    scale = np.exp(rng.normal(-5, 0.5, out_f)).astype(np.float32)
    blob = encode(recipe_c4())
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    got, _ = _run_d2h(blob, sym, params, q, route, chunk=64 << 10)
    assert np.array_equal(got, _expected(blob, sym, params, q))


def test_padded_layout_and_pageable_destination():
    x = np.random.default_rng(5).uniform(0, 1, 2 * 3 * 40 * 24).astype(np.float32)
    blob = encode(recipe_c2(2, 3, 40, 24))
    for route in ("auto", "dma_ring", "staged"):
        got, _ = _run_d2h(blob, {}, {}, x, route, pinned=False)
        assert np.array_equal(got, _expected(blob, {}, {}, x)), route


def test_torch_bridge_d2h():
    """reloc_torch.dispatch with a d2h recipe: CUDA tensor in, pinned CPU
    tensor out, ordered after the caller's current stream."""
    import torch
    from sym_b200.reloc_torch import dispatch
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S
    from sym_b200.reloc_torch.compiler import CompilerClient

    shape = (S.Symbol("B"), S.Symbol("S"), S.Const(128))
    spec = lambda dt: R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), dt)  # noqa: E731
    recipe = R.Recipe(spec("float16"), (R.Cast("float32", "exact"),), spec("float32"), "d2h")
    compiled = CompilerClient.from_environment().compile(recipe)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        src = torch.randn(4, 33, 128, device="cuda").half()  # produced on the side stream
        req = dispatch.prepare_typed_transfer(compiled, src, "cpu")
        res = dispatch.execute_typed_transfer(req)
    out = res.tensor
    assert out.device.type == "cpu" and out.is_pinned() and out.dtype == torch.float32
    assert torch.equal(out, src.float().cpu())
    assert res.report["implementation"].startswith("b200_fused_d2h")
