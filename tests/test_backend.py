"""RelocBackend on the host: the FX importer (reference fx_import.import_graph)
accepts the supported CPU -> GPU chains with the recipe their ops mean,
rejects the rest with a reason, and the backend rewrites accepted regions
into one region call. Graphs come from torch.fx.symbolic_trace; nothing here
executes on a device."""
import pytest


def _trace(fn):
    import torch.fx as fx

    return fx.symbolic_trace(fn)


def _ops(c):
    return [type(op).__name__ for op in c.recipe.operations]


def test_weight_dequant_chain():
    import torch
    from sym_b200.reloc_torch.fx_import import import_graph
    from sym_b200.reloc_torch.recipe import BindingParam

    def f(q, s):
        w = (q.float() * s[:, None]).half().t().contiguous().cuda()
        return w @ w.t()

    r = import_graph(_trace(f), (torch.zeros(16, 32, dtype=torch.int8), torch.ones(16)))
    (c,) = r.candidates
    assert _ops(c) == ["Dequantize", "Cast", "Transpose"] and c.parameters == ("s",)
    dq = c.recipe.operations[0]
    assert dq.axis == 0 and dq.scale == BindingParam("s", "float32", dq.scale.extents)
    assert [e.value for e in c.recipe.destination.shape] == [32, 16] and c.recipe.destination.dtype == "float16"
    assert c.device == torch.device("cuda")


def test_channels_last_pad_cast_chain():
    import torch
    import torch.nn.functional as F
    from sym_b200.reloc_torch.fx_import import import_graph

    def f(x):
        return F.pad(x.permute(0, 2, 3, 1), (0, 1)).half().to("cuda")

    (c,) = import_graph(_trace(f), (torch.zeros(2, 3, 5, 7),)).candidates
    assert _ops(c) == ["Transpose", "Pad", "Cast"]
    assert [e.value for e in c.recipe.destination.shape] == [2, 5, 7, 4]


def test_scalar_scale_and_plain_int8_cast():
    import torch
    from sym_b200.reloc_torch.fx_import import import_graph
    from sym_b200.reloc_torch.recipe import InlineParam

    def f(q):
        return (q.float() * 0.05).cuda(), q.half().cuda()

    # q has two users: neither chain may swallow the other's member
    r = import_graph(_trace(f), (torch.zeros(4, 8, dtype=torch.int8),))
    assert len(r.candidates) == 2
    a, b = r.candidates
    assert a.recipe.operations[0].scale == InlineParam("float32", (), (0x3D4CCCCD,))
    assert _ops(b) == ["Dequantize", "Cast"] and b.recipe.operations[0].scale.bits == (0x3F800000,)


@pytest.mark.parametrize("case,reason", [
    ("transposed_view", "destination_layout"),
    ("escaping", "escaping_intermediate"),
    ("float_to_int", "typed_transform_unavailable"),
    ("gpu_source", "source_not_on_cpu"),
    ("reflect_pad", "unsupported_padding"),
    ("two_axis_scale", "unsupported_parameter"),
])
def test_rejections_carry_reasons(case, reason):
    import torch
    import torch.nn.functional as F
    from sym_b200.reloc_torch.fx_import import import_graph

    x = torch.zeros(8, 4)
    fns = {
        "transposed_view": (lambda x: x.t().cuda(), (x,)),
        "escaping": (lambda x: (x.t().cuda(), x.t().sum()), (x,)),
        "float_to_int": (lambda x: x.to(torch.int8).cuda(), (x,)),
        "gpu_source": (lambda x: x.t().contiguous().cuda(), (torch.zeros(8, 4, device="meta"),)),
        "reflect_pad": (lambda x: F.pad(x, (1, 1), mode="reflect").cuda(), (x,)),
        "two_axis_scale": (lambda q, s: (q.float() * s).cuda(),
                           (torch.zeros(8, 4, dtype=torch.int8), torch.ones(8, 4))),
    }
    fn, ex = fns[case]
    if case == "escaping":
        def fn(x):
            y = x.t()
            return y.cuda(), y.sum()
    r = import_graph(_trace(fn), ex)
    assert not r.candidates
    assert reason in [e.reason for e in r.exclusions]


def test_backend_rewrites_accepted_regions_only():
    import torch
    from sym_b200.reloc_torch.backend import RelocBackend

    def f(q, s, x):
        w = (q.float() * s[:, None]).half().t().contiguous().cuda()
        y = x.t().cuda()  # rejected: non-dense destination
        return w, y

    backend = RelocBackend()
    fn = backend(_trace(f), (torch.zeros(16, 32, dtype=torch.int8), torch.ones(16), torch.zeros(8, 4)))
    code = fn.rewritten.__self__.code
    assert "reloc_region_" in code and ".cuda()" in code  # the rejected region keeps its nodes
    assert len(fn.regions) == 1
    st = backend.stats()
    assert st["regions"] == 1 and st["plan_compiles"] == 1
    assert ("cuda_1", "destination_layout") in st["exclusions"]
    backend.close()
    with pytest.raises(RuntimeError):
        fn(torch.zeros(16, 32, dtype=torch.int8), torch.ones(16), torch.zeros(8, 4))


def _dynamo_graphs(fn, *args):
    """The graphs Dynamo captures for ``fn`` with dynamic shapes (recorded by
    a backend; the calls themselves fail on a host without a GPU)."""
    import torch

    graphs = []

    def record(gm, example_inputs):
        graphs.append((gm, list(example_inputs)))
        return gm.forward

    torch._dynamo.reset()
    try:
        torch.compile(fn, backend=record, dynamic=True)(*args)
    except (RuntimeError, AssertionError):
        pass
    torch._dynamo.reset()
    return graphs


def test_dynamic_dims_become_plan_symbols():
    import torch
    from sym_b200.reloc_torch.compiler import CompilerClient
    from sym_b200.reloc_torch.fx_import import import_graph
    from sym_b200.reloc_torch.symbolic import Symbol

    def f(q, s):
        return (q.float() * s[:, None]).half().t().contiguous().cuda()

    ((gm, ex),) = _dynamo_graphs(f, torch.zeros(16, 32, dtype=torch.int8), torch.ones(16))
    (c,) = import_graph(gm, ex).candidates
    rows, cols = c.recipe.source.shape
    assert isinstance(rows, Symbol) and isinstance(cols, Symbol)
    assert c.recipe.destination.shape == (cols, rows)
    assert c.recipe.operations[0].scale.extents == (rows,)  # the scale's length is the row symbol
    compiled = CompilerClient.from_environment().compile(c.recipe)
    assert sorted(compiled.symbols) == sorted([rows.name, cols.name])
    bindings = compiled.source_symbols((40, 24))
    assert list(compiled.parameter_extents(bindings).values()) == [("float32", [40])]


def test_dynamic_pad_and_flatten_keep_symbols():
    import torch
    import torch.nn.functional as F
    from sym_b200.reloc_torch.fx_import import import_graph
    from sym_b200.reloc_torch.symbolic import Add, Const, Mul, Symbol

    ((gm, ex),) = _dynamo_graphs(lambda x: F.pad(x.permute(0, 2, 3, 1), (0, 1)).half().to("cuda"),
                                 torch.zeros(2, 3, 5, 7))
    (c,) = import_graph(gm, ex).candidates
    n, ch, h, w = c.recipe.source.shape
    assert all(isinstance(e, Symbol) for e in (n, ch, h, w))
    assert c.recipe.destination.shape[:3] == (n, h, w) and c.recipe.destination.shape[3] == Add(ch, Const(1))

    ((gm, ex),) = _dynamo_graphs(lambda x: x.flatten(1).t().contiguous().cuda(), torch.zeros(6, 4, 5))
    (c,) = import_graph(gm, ex).candidates
    a, b, d = c.recipe.source.shape
    assert c.recipe.destination.shape == (Mul(b, d), a)


def test_dynamic_reshape_captures_the_example_shape():
    """A reshape whose target cannot follow the dynamic dims keeps the
    example's sizes; the region then takes only that shape."""
    import torch
    from sym_b200.reloc_torch.backend import RelocBackend
    from sym_b200.reloc_torch.fx_import import import_graph
    from sym_b200.reloc_torch.symbolic import Const

    ((gm, ex),) = _dynamo_graphs(lambda x: x.reshape(-1, 64).t().contiguous().cuda(), torch.zeros(1 << 12))
    (c,) = import_graph(gm, ex).candidates
    assert c.recipe.source.shape == (Const(4096),)
    fn = RelocBackend()(gm, ex)
    (region,) = fn.regions
    assert region._eligible(torch.zeros(4096), ())
    assert not region._eligible(torch.zeros(8192), ())


def test_dynamic_region_checks_each_call():
    import torch
    from sym_b200.reloc_torch.backend import RelocBackend

    def f(q, s):
        return (q.float() * s[:, None]).half().t().contiguous().cuda()

    ((gm, ex),) = _dynamo_graphs(f, torch.zeros(16, 32, dtype=torch.int8), torch.ones(16))
    fn = RelocBackend()(gm, ex)
    (region,) = fn.regions
    assert region.shape == (None, None)
    q = torch.zeros(40, 24, dtype=torch.int8)
    assert region._eligible(q, (torch.ones(40),))
    assert not region._eligible(q, (torch.ones(24),))          # scale length != rows
    assert not region._eligible(q.float(), (torch.ones(40),))  # dtype
    assert not region._eligible(q[:, :8], (torch.ones(40),))   # not dense
    assert not region._eligible(torch.zeros(0, 24, dtype=torch.int8), (torch.ones(0),))

    ((gm, ex),) = _dynamo_graphs(lambda x: x.t().contiguous().cuda(), torch.zeros(16, 16))
    (region,) = RelocBackend()(gm, ex).regions
    assert region._eligible(torch.zeros(24, 24), ())
    assert not region._eligible(torch.zeros(24, 8), ())  # one symbol, two sizes


def test_decomposed_dequantize_ops_become_typed_recipes():
    """``quantized_decomposed.dequantize_per_channel`` / ``_per_tensor`` (the
    reference importer's audited dequantize operators): tensor scales and
    zero points become runtime parameters, Python scalars exact inline bits,
    ``out_dtype`` a narrowing cast."""
    import torch
    import torch.ao.quantization.fx._decomposed  # noqa: F401  (registers the ops)
    from sym_b200.reloc_torch.fx_import import import_graph
    from sym_b200.reloc_torch.recipe import BindingParam, InlineParam

    qd = torch.ops.quantized_decomposed

    def per_channel(q, s, z):
        return qd.dequantize_per_channel(q, s, z, 0, -128, 127, torch.int8).half().t().contiguous().cuda()

    ((gm, ex),) = _dynamo_graphs(per_channel, torch.zeros(16, 32, dtype=torch.int8), torch.ones(16),
                                 torch.zeros(16, dtype=torch.int64))
    (c,) = import_graph(gm, ex).candidates
    dq = c.recipe.operations[0]
    assert _ops(c) == ["Dequantize", "Cast", "Transpose"] and dq.axis == 0 and len(c.parameters) == 2
    assert isinstance(dq.scale, BindingParam) and dq.zero_point.dtype == "int32"

    ((gm, ex),) = _dynamo_graphs(lambda q: qd.dequantize_per_tensor(q, 0.05, -3, -128, 127, torch.int8).cuda(),
                                 torch.zeros(8, 4, dtype=torch.int8))
    (c,) = import_graph(gm, ex).candidates
    dq = c.recipe.operations[0]
    assert dq.scale == InlineParam("float32", (), (0x3D4CCCCD,))
    assert dq.zero_point == InlineParam("int32", (), (0xFFFFFFFD,)) and not c.parameters

    ((gm, ex),) = _dynamo_graphs(
        lambda q, s: qd.dequantize_per_channel(q, s, None, 1, -128, 127, torch.int8, out_dtype=torch.bfloat16).cuda(),
        torch.zeros(8, 4, dtype=torch.int8), torch.ones(4))
    (c,) = import_graph(gm, ex).candidates
    assert _ops(c) == ["Dequantize", "Cast"] and c.recipe.operations[0].zero_point is None
    assert c.recipe.destination.dtype == "bfloat16"


def test_aten_level_graphs_are_imported():
    """Graphs of ATen overloads (AOT / export level) map to the same recipes."""
    import torch
    import torch.fx as fx
    from sym_b200.reloc_torch.fx_import import import_graph

    aten = torch.ops.aten
    g = fx.Graph()
    x = g.placeholder("x")
    p = g.call_function(aten.permute.default, (x, [1, 0]))
    c = g.call_function(aten.clone.default, (p,), {"memory_format": torch.contiguous_format})
    pad = g.call_function(aten.constant_pad_nd.default, (c, [0, 2], 0.0))
    out = g.call_function(aten._to_copy.default, (pad,), {"dtype": torch.float16, "device": torch.device("cuda")})
    g.output(out)
    (cand,) = import_graph(fx.GraphModule(torch.nn.Module(), g), (torch.zeros(8, 4),)).candidates
    assert _ops(cand) == ["Transpose", "Pad", "Cast"]
    assert [e.value for e in cand.recipe.destination.shape] == [4, 10]

    # a preserved-format clone of a transposed view is not dense: rejected
    g = fx.Graph()
    x = g.placeholder("x")
    t = g.call_function(aten.t.default, (x,))
    c = g.call_function(aten.clone.default, (t,))
    g.output(g.call_function(aten._to_copy.default, (c,), {"device": torch.device("cuda")}))
    r = import_graph(fx.GraphModule(torch.nn.Module(), g), (torch.zeros(8, 4),))
    assert not r.candidates and [e.reason for e in r.exclusions] == ["destination_layout"]


def test_dynamic_view_targets_follow_the_symbols():
    """``x.view(x.shape[0], x.shape[1], 16, 64)`` and ``x.view(-1)`` in a
    dynamic capture: SymInt targets and exact -1 quotients keep the plan
    symbolic; ``reshape(-1, 64)`` (a quotient that is not exact) keeps the
    example's sizes."""
    import torch
    from sym_b200.reloc_torch.fx_import import import_graph
    from sym_b200.reloc_torch.symbolic import Const, Mul, Symbol

    ((gm, ex),) = _dynamo_graphs(lambda x: x.view(x.shape[0], x.shape[1], 16, 64).transpose(1, 2).contiguous().cuda(),
                                 torch.zeros(4, 8, 1024))
    (c,) = import_graph(gm, ex).candidates
    b, s, h = c.recipe.source.shape
    assert isinstance(b, Symbol) and isinstance(s, Symbol) and h == Const(1024)
    assert c.recipe.destination.shape == (b, Const(16), s, Const(64))

    ((gm, ex),) = _dynamo_graphs(lambda x: x.view(-1).cuda(), torch.zeros(4, 8))
    (c,) = import_graph(gm, ex).candidates
    a, b = c.recipe.source.shape
    assert c.recipe.destination.shape in ((Mul(a, b),), (Mul(b, a),))

    ((gm, ex),) = _dynamo_graphs(lambda x: x.reshape(-1, 64).t().contiguous().cuda(), torch.zeros(4, 8, 1024))
    (c,) = import_graph(gm, ex).candidates
    assert all(isinstance(e, Const) for e in c.recipe.source.shape)


def test_bind_shape_caches_without_sharing_state():
    """The per-shape binding cache of a compiled recipe returns the same
    bindings and parameter extents as binding afresh, as copies."""
    from sym_b200.workloads import weight_recipe
    from sym_b200.reloc_torch.compiler import CompilerClient

    compiled = CompilerClient.from_environment().compile(weight_recipe("out_in_f16"))
    for shape in ((64, 96), (96, 64), (64, 96)):
        bindings, declared = compiled.bind_shape(shape)
        assert bindings == compiled.source_symbols(shape)
        assert declared == compiled.parameter_extents(bindings)
        bindings["s0"] = -1
        declared["scale"][1].append(7)
    assert compiled.bind_shape((64, 96)) == ({"s0": 64, "s1": 96}, {"scale": ("float32", [64])})


def test_decomposed_quantize_is_excluded_with_the_reference_reason():
    import torch
    import torch.ao.quantization.fx._decomposed  # noqa: F401
    from sym_b200.reloc_torch.fx_import import import_graph

    qd = torch.ops.quantized_decomposed
    ((gm, ex),) = _dynamo_graphs(lambda x: qd.quantize_per_tensor(x, 0.05, 0, -128, 127, torch.int8).cuda(),
                                 torch.zeros(8, 4))
    r = import_graph(gm, ex)
    assert not r.candidates and "quantize_semantics_unproved" in [e.reason for e in r.exclusions]


def test_inexact_dynamic_unflatten_keeps_the_example_shape():
    """``unflatten(d, (4, -1))`` of a dynamic dim (a quotient the plan cannot
    prove exact) captures the example's sizes; the region takes only that
    shape."""
    import torch
    from sym_b200.reloc_torch.backend import RelocBackend
    from sym_b200.reloc_torch.symbolic import Const

    fn = lambda x: x.unflatten(2, (4, -1)).transpose(1, 2).contiguous().half().cuda()  # noqa: E731
    ((gm, ex),) = _dynamo_graphs(fn, torch.zeros(4, 6, 8))
    (region,) = RelocBackend()(gm, ex).regions
    assert all(isinstance(e, Const) for e in region.candidate.recipe.source.shape)
    assert region._eligible(torch.zeros(4, 6, 8), ()) and not region._eligible(torch.zeros(3, 6, 8), ())
