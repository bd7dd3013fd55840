"""The importer's recipes mean what the Torch ops mean: each accepted region's
recipe, encoded and executed by the reference runtime on the host (the
checker, not the product), gives bit for bit the result of the same ops run
eagerly by PyTorch on the CPU. This pins the importer's translation (axes,
scales, zero points, pads, casts, symbols) without a GPU; the GPU tests then
pin the kernels against the same reference runtime."""
import numpy as np
import pytest

from test_backend import _dynamo_graphs

pytestmark = pytest.mark.skipif("not __import__('oracle.ref', fromlist=['ref']).available()",
                                reason="reference runtime not built")


def _param_entry(tensor, declared_dtype):
    import torch

    if declared_dtype == "int32":
        tensor = tensor.to(torch.int32)
    arr = tensor.detach().contiguous().numpy()
    return (declared_dtype, list(arr.shape), arr.tobytes())


def _reference_result(gm, ex, src, params):
    """The single candidate's recipe executed by the reference runtime."""
    from oracle import ref
    from sym_b200.reloc_torch.compiler import CompilerClient
    from sym_b200.reloc_torch.fx_import import import_graph

    (c,) = import_graph(gm, ex).candidates
    compiled = CompilerClient.from_environment().compile(c.recipe)
    bindings = compiled.source_symbols(tuple(src.shape))
    declared = {p.name: p.dtype for p in compiled.recipe.parameter_bindings}
    named = dict(zip(c.parameters, params))
    raw = _bits(src)
    if compiled.typed:
        prog = ref.TypedProgram(compiled.plan_bytes, bindings,
                                {n: _param_entry(named[n], d) for n, d in declared.items()})
        return prog.execute(raw), c
    return ref.LayoutPlan(compiled.plan_bytes, bindings).execute(raw), c


def _bits(t):
    import torch

    t = t.contiguous()
    if t.dtype in (torch.float16, torch.bfloat16):
        t = t.view(torch.int16)  # numpy has no bfloat16
    return np.ascontiguousarray(t.numpy()).view(np.uint8).reshape(-1)


def test_decomposed_dequantize_per_channel_zero_points_f16_transpose():
    import torch
    import torch.ao.quantization.fx._decomposed  # noqa: F401

    qd = torch.ops.quantized_decomposed
    g = torch.Generator().manual_seed(3)
    q = torch.randint(-128, 128, (48, 40), dtype=torch.int8, generator=g)
    s = torch.exp(torch.randn(48, generator=g) - 4)
    z = torch.randint(-9, 9, (48,), dtype=torch.int64, generator=g)

    def body(q, s, z):
        return qd.dequantize_per_channel(q, s, z, 0, -128, 127, torch.int8).half().t().contiguous()

    ((gm, ex),) = _dynamo_graphs(lambda q, s, z: body(q, s, z).cuda(), q, s, z)
    got, _ = _reference_result(gm, ex, q, (s, z))
    assert np.array_equal(got, _bits(body(q, s, z)))


def test_decomposed_dequantize_per_tensor_inline_and_out_dtype():
    import torch
    import torch.ao.quantization.fx._decomposed  # noqa: F401

    qd = torch.ops.quantized_decomposed
    q = torch.randint(-128, 128, (33, 17), dtype=torch.int8, generator=torch.Generator().manual_seed(4))

    def body(q):
        return qd.dequantize_per_tensor(q, 0.0123, -7, -128, 127, torch.int8)

    ((gm, ex),) = _dynamo_graphs(lambda q: body(q).cuda(), q)
    got, _ = _reference_result(gm, ex, q, ())
    assert np.array_equal(got, _bits(body(q)))

    s = torch.exp(torch.randn(17, generator=torch.Generator().manual_seed(5)) - 3)

    def body2(q, s):
        return qd.dequantize_per_channel(q, s, None, 1, -128, 127, torch.int8, out_dtype=torch.bfloat16)

    ((gm, ex),) = _dynamo_graphs(lambda q, s: body2(q, s).cuda(), q, s)
    got, _ = _reference_result(gm, ex, q, (s,))
    assert np.array_equal(got, _bits(body2(q, s)))


def test_int8_scale_multiply_and_channels_last_pad_cast():
    import torch
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(6)
    q = torch.randint(-128, 128, (24, 40), dtype=torch.int8, generator=g)
    s = torch.exp(torch.randn(24, generator=g) - 4)

    def body(q, s):
        return (q.float() * s[:, None]).half().t().contiguous()

    ((gm, ex),) = _dynamo_graphs(lambda q, s: body(q, s).cuda(), q, s)
    got, _ = _reference_result(gm, ex, q, (s,))
    assert np.array_equal(got, _bits(body(q, s)))

    x = torch.randn(2, 3, 7, 5, generator=g)
    x.view(-1)[:3] = torch.tensor([float("inf"), -0.0, 65520.0])

    def body2(x):
        return F.pad(x.permute(0, 2, 3, 1), (0, 1)).half()

    ((gm, ex),) = _dynamo_graphs(lambda x: body2(x).cuda(), x)
    got, _ = _reference_result(gm, ex, x, ())
    assert np.array_equal(got, _bits(body2(x)))


@pytest.mark.parametrize("shape", [(2, 8, 1024), (3, 5, 1024)])
def test_dynamic_head_split_binds_for_other_sizes(shape):
    """A dynamic capture (traced at one size) run by the reference at another."""
    import torch

    def body(x):
        return x.view(x.shape[0], x.shape[1], 16, 64).transpose(1, 2).contiguous().half()

    ((gm, ex),) = _dynamo_graphs(lambda x: body(x).cuda(), torch.zeros(4, 6, 1024))
    x = torch.randn(shape, generator=torch.Generator().manual_seed(7))
    got, c = _reference_result(gm, ex, x, ())
    assert any(type(e).__name__ == "Symbol" for e in c.recipe.source.shape)
    assert np.array_equal(got, _bits(body(x)))


@pytest.mark.parametrize("name", ["T", "mT", "movedim", "movedim_tuple", "swapaxes", "unflatten", "unflatten_dyn"])
def test_more_view_ops_match_eager(name):
    """``x.T``, ``x.mT``, ``movedim``, ``swapaxes`` and ``unflatten`` (with a
    -1, also in a dynamic capture) become the same permutation or reshape
    the eager ops compute, with a cast so the plan is a typed one."""
    import torch

    bodies = {
        "T": lambda x: x.T.contiguous().half(),
        "mT": lambda x: x.mT.contiguous().half(),
        "movedim": lambda x: x.movedim(0, 2).contiguous().half(),
        "movedim_tuple": lambda x: torch.movedim(x, (0, 1), (2, 0)).contiguous().half(),
        "swapaxes": lambda x: x.swapaxes(0, 2).contiguous().half(),
        "unflatten": lambda x: x.unflatten(2, (2, -1)).transpose(1, 2).contiguous().half(),
        "unflatten_dyn": lambda x: x.unflatten(1, (-1, 1)).transpose(0, 2).contiguous().half(),
    }
    body = bodies[name]
    x = torch.randn(3, 5, 8, generator=torch.Generator().manual_seed(8))
    if name == "unflatten_dyn":  # traced at one size, run at another: the -1 is an exact quotient
        ((gm, ex),) = _dynamo_graphs(lambda x: body(x).cuda(), torch.zeros(4, 6, 8))
    else:
        ((gm, ex),) = _dynamo_graphs(lambda x: body(x).cuda(), x)
    got, c = _reference_result(gm, ex, x, ())
    if name == "unflatten_dyn":
        assert any(type(e).__name__ == "Symbol" for e in c.recipe.source.shape)
    assert np.array_equal(got, _bits(body(x)))


@pytest.mark.parametrize("name", ["int8_half", "int8_bf16_t", "f16_float_t", "bf16_float", "f32_bf16_pad"])
def test_casts_match_eager(name):
    """int8 -> f16/bf16 (exact: every int8 is representable), f16/bf16 -> f32
    widening and f32 -> bf16 narrowing with a pad, as eager PyTorch computes
    them on finite inputs."""
    import torch
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(9)
    cases = {
        "int8_half": (lambda x: x.half(), torch.randint(-128, 128, (7, 33), dtype=torch.int8, generator=g)),
        "int8_bf16_t": (lambda x: x.to(torch.bfloat16).t().contiguous(),
                        torch.randint(-128, 128, (7, 33), dtype=torch.int8, generator=g)),
        "f16_float_t": (lambda x: x.float().t().contiguous(), (torch.randn(9, 20, generator=g) * 1000).half()),
        "bf16_float": (lambda x: x.float(), (torch.randn(9, 20, generator=g) * 1e30).bfloat16()),
        "f32_bf16_pad": (lambda x: F.pad(x.to(torch.bfloat16), (1, 2)), torch.randn(6, 10, generator=g) * 3e38),
    }
    body, x = cases[name]
    ((gm, ex),) = _dynamo_graphs(lambda x: body(x).cuda(), x)
    got, _ = _reference_result(gm, ex, x, ())
    assert np.array_equal(got, _bits(body(x)))


def _random_chain(seed):
    """A random chain of layout ops, at most one narrowing cast and an
    optional constant pad on the last axis, as eager callables."""
    import torch
    import torch.nn.functional as F

    rng = np.random.default_rng(seed)
    rank = int(rng.integers(2, 5))
    shape = tuple(int(rng.integers(2, 6)) for _ in range(rank))
    steps, cur = [], list(shape)
    for _ in range(int(rng.integers(1, 5))):
        kind = ["permute", "transpose", "flatten", "unsqueeze", "mT", "movedim"][int(rng.integers(0, 6))]
        r = len(cur)
        if kind == "permute":
            p = tuple(int(i) for i in rng.permutation(r))
            steps.append(lambda x, p=p: x.permute(*p))
            cur = [cur[i] for i in p]
        elif kind == "transpose" and r >= 2:
            a, b = (int(i) for i in rng.choice(r, 2, replace=False))
            steps.append(lambda x, a=a, b=b: x.transpose(a, b))
            cur[a], cur[b] = cur[b], cur[a]
        elif kind == "flatten" and r >= 3:
            a = int(rng.integers(0, r - 1))
            steps.append(lambda x, a=a: x.contiguous().flatten(a, a + 1))
            cur = cur[:a] + [cur[a] * cur[a + 1]] + cur[a + 2:]
        elif kind == "unsqueeze" and r < 5:
            a = int(rng.integers(0, r + 1))
            steps.append(lambda x, a=a: x.unsqueeze(a))
            cur = cur[:a] + [1] + cur[a:]
        elif kind == "mT" and r >= 2:
            steps.append(lambda x: x.mT)
            cur[-1], cur[-2] = cur[-2], cur[-1]
        elif kind == "movedim" and r >= 2:
            a, b = (int(i) for i in rng.choice(r, 2, replace=False))
            steps.append(lambda x, a=a, b=b: x.movedim(a, b))
            d = cur.pop(a)
            cur.insert(b, d)
    cast = [None, torch.float16, torch.bfloat16][int(rng.integers(0, 3))]
    pad = rng.random() < 0.4

    def body(x):
        for f in steps:
            x = f(x)
        x = x.contiguous()
        if cast is not None:
            x = x.to(cast)
        if pad:
            x = F.pad(x, (0, 1))
        return x

    return body, shape


@pytest.mark.parametrize("seed", range(40))
def test_random_chains_import_to_their_eager_meaning(seed):
    """Random chains of supported layout ops, casts and pads: the imported
    recipe, executed by the reference runtime, equals the eager result."""
    import torch

    from sym_b200.reloc_torch.backend import RelocBackend
    from sym_b200.reloc_torch.compiler import UnsupportedRecipe

    body, shape = _random_chain(seed)
    x = torch.randn(shape, generator=torch.Generator().manual_seed(seed))
    ((gm, ex),) = _dynamo_graphs(lambda x: body(x).cuda(), x)
    try:
        got, _ = _reference_result(gm, ex, x, ())
    except UnsupportedRecipe as error:
        # a layout the plan format cannot state (e.g. merging axes a transpose
        # made non-adjacent): the backend keeps the region's original ops
        backend = RelocBackend()
        assert not backend(gm, ex).regions
        assert (error.reason if hasattr(error, "reason") else str(error)) in str(backend.stats()["exclusions"])
        return
    assert np.array_equal(got, _bits(body(x)))
