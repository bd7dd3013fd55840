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
