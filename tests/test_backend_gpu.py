"""RelocBackend end to end on the GPU: ``torch.compile(fn, backend=RelocBackend())``
returns exactly what eager ``fn`` returns (bit for bit), the accepted regions
run on the B200 kernels (kernel launches counted), graphs captured with
dynamic shapes run one region over every size (the plan's symbols bound per
call), and calls the replacement cannot take (inputs that need autograd) run
the original ops."""
import pytest

pytestmark = pytest.mark.gpu


def _compile(fn, dynamic=False):
    import torch
    from sym_b200.reloc_torch.backend import RelocBackend

    torch._dynamo.reset()
    backend = RelocBackend()
    return torch.compile(fn, backend=backend, dynamic=dynamic), backend


def _bits_equal(a, b):
    import torch

    if a.dtype in (torch.float16, torch.bfloat16):
        return torch.equal(a.view(torch.int16), b.view(torch.int16))
    if a.dtype == torch.float32:
        return torch.equal(a.view(torch.int32), b.view(torch.int32))
    return torch.equal(a, b)


def test_weight_dequant_region_matches_eager():
    import torch
    from sym_b200 import pyreloc

    def f(q, s):
        w = (q.float() * s[:, None]).half().t().contiguous().cuda()
        return w, w.float().sum()

    g = torch.Generator().manual_seed(0)
    q = torch.randint(-128, 128, (1024, 4096), dtype=torch.int8, generator=g)
    s = torch.exp(torch.randn(1024, generator=g) * 0.5 - 5)
    fn, backend = _compile(f)
    l0 = pyreloc.kernel_launches()
    w, total = fn(q, s)
    torch.cuda.synchronize()
    assert pyreloc.kernel_launches() > l0
    want, want_total = f(q, s)
    assert w.is_contiguous() and w.shape == want.shape and _bits_equal(w, want)
    assert torch.equal(total, want_total)
    assert backend.stats()["executions"] >= 1


@pytest.mark.parametrize("shape", [(4, 3, 64, 64), (2, 3, 31, 17)])
def test_channels_last_pad_region_matches_eager(shape):
    import torch
    import torch.nn.functional as F

    def f(x):
        return F.pad(x.permute(0, 2, 3, 1), (0, 1)).half().to("cuda")

    x = torch.rand(shape)
    x.view(-1)[:3] = torch.tensor([float("nan"), float("inf"), 65520.0])
    fn, backend = _compile(f)
    got = fn(x)
    assert _bits_equal(got, f(x)) and backend.stats()["executions"] >= 1


def test_layout_only_region_matches_eager():
    import torch

    def f(x):
        return x.reshape(-1, 64).t().contiguous().cuda() + 0  # a consumer after the region

    x = torch.randn(1 << 16)
    fn, backend = _compile(f)
    assert _bits_equal(fn(x), f(x)) and backend.stats()["executions"] >= 1


def test_autograd_inputs_take_the_original_ops():
    import torch

    def f(x):
        return x.t().contiguous().cuda().float()

    x = torch.randn(64, 32, requires_grad=True)
    fn, backend = _compile(f)
    got = fn(x)
    got.sum().backward()
    assert torch.equal(got.detach(), f(x).detach())
    assert x.grad is not None and torch.equal(x.grad, torch.ones_like(x))


def test_repeat_calls_and_new_values_stay_exact():
    import torch

    def f(q):
        return (q.float() * 0.05).cuda()

    fn, backend = _compile(f)
    for seed in range(3):
        q = torch.randint(-128, 128, (256, 512), dtype=torch.int8, generator=torch.Generator().manual_seed(seed))
        assert _bits_equal(fn(q), f(q))
    assert backend.stats()["executions"] >= 3


def test_dynamic_shapes_bind_per_call():
    """One dynamic capture serves every size: no recompile, each call exact."""
    import torch
    from sym_b200 import pyreloc

    def f(q, s):
        return (q.float() * s[:, None]).half().t().contiguous().cuda()

    fn, backend = _compile(f, dynamic=True)
    g = torch.Generator().manual_seed(1)
    for rows, cols in ((256, 512), (96, 200), (1024, 4096), (33, 7)):
        q = torch.randint(-128, 128, (rows, cols), dtype=torch.int8, generator=g)
        s = torch.exp(torch.randn(rows, generator=g) * 0.5 - 5)
        l0 = pyreloc.kernel_launches()
        got = fn(q, s)
        torch.cuda.synchronize()
        assert pyreloc.kernel_launches() > l0
        assert got.shape == (cols, rows) and _bits_equal(got, f(q, s))
    st = backend.stats()
    assert st["graphs"] == 1 and st["executions"] == 4 and st.get("fallbacks", 0) == 0


@pytest.mark.parametrize("fn_name", ["pad", "flatten"])
def test_dynamic_layout_and_pad_regions(fn_name):
    import torch
    import torch.nn.functional as F

    fns = {
        "pad": (lambda x: F.pad(x.permute(0, 2, 3, 1), (0, 1)).half().to("cuda"),
                [(2, 3, 64, 64), (4, 3, 31, 17), (1, 5, 8, 9)]),
        "flatten": (lambda x: x.flatten(1).t().contiguous().cuda(), [(6, 4, 5), (64, 32, 48), (3, 2, 1000)]),
    }
    f, shapes = fns[fn_name]
    fn, backend = _compile(f, dynamic=True)
    for shape in shapes:
        x = torch.rand(shape)
        assert _bits_equal(fn(x), f(x))
    assert backend.stats()["executions"] >= 2


@pytest.mark.parametrize("case", ["per_channel_zp_f16_t", "per_tensor_inline", "per_channel_bf16_out",
                                  "per_tensor_tensor_params"])
def test_decomposed_dequantize_regions_match_eager(case):
    """Weight-dequant graphs written with ``quantized_decomposed`` ops run as
    one fused transfer each, bit for bit the eager result."""
    import torch
    import torch.ao.quantization.fx._decomposed  # noqa: F401
    from sym_b200 import pyreloc

    qd = torch.ops.quantized_decomposed
    g = torch.Generator().manual_seed(7)
    q = torch.randint(-128, 128, (512, 768), dtype=torch.int8, generator=g)
    s0 = torch.exp(torch.randn(512, generator=g) * 0.5 - 5)
    s1 = torch.exp(torch.randn(768, generator=g) * 0.5 - 5)
    z0 = torch.randint(-20, 20, (512,), dtype=torch.int64, generator=g)
    fns = {
        "per_channel_zp_f16_t": (lambda q, s, z: qd.dequantize_per_channel(q, s, z, 0, -128, 127, torch.int8)
                                 .half().t().contiguous().cuda(), (q, s0, z0)),
        "per_tensor_inline": (lambda q: qd.dequantize_per_tensor(q, 0.0123, -7, -128, 127, torch.int8).cuda(), (q,)),
        "per_channel_bf16_out": (lambda q, s: qd.dequantize_per_channel(q, s, None, 1, -128, 127, torch.int8,
                                                                        out_dtype=torch.bfloat16).cuda(), (q, s1)),
        "per_tensor_tensor_params": (lambda q, s, z: qd.dequantize_per_tensor.tensor(q, s, z, -128, 127,
                                                                                     torch.int8).cuda(),
                                     (q, torch.tensor(0.031), torch.tensor(5))),
    }
    f, args = fns[case]
    fn, backend = _compile(f)
    l0 = pyreloc.kernel_launches()
    got = fn(*args)
    torch.cuda.synchronize()
    assert pyreloc.kernel_launches() > l0 and backend.stats()["executions"] >= 1, backend.stats()
    assert _bits_equal(got, f(*args))


@pytest.mark.parametrize("fn_name", ["heads", "flatten_rest"])
def test_dynamic_view_targets_run_for_every_size(fn_name):
    """Symbolic view targets (SymInt extents, exact -1 quotients) keep one
    plan for every size."""
    import torch

    fns = {
        "heads": (lambda x: x.view(x.shape[0], x.shape[1], 16, 64).transpose(1, 2).contiguous().half().cuda(),
                  [(2, 8, 1024), (3, 40, 1024), (5, 7, 1024)]),
        "flatten_rest": (lambda x: x.view(x.shape[0], -1).t().contiguous().cuda(),
                         [(4, 8, 6), (9, 5, 7), (16, 32, 3)]),
    }
    f, shapes = fns[fn_name]
    fn, backend = _compile(f, dynamic=True)
    for shape in shapes:
        x = torch.randn(shape)
        assert _bits_equal(fn(x), f(x))
    st = backend.stats()
    assert st["executions"] >= 2 and st.get("fallbacks", 0) == 0, st
