"""RelocBackend end to end on the GPU: ``torch.compile(fn, backend=RelocBackend())``
returns exactly what eager ``fn`` returns (bit for bit), the accepted regions
run on the B200 kernels (kernel launches counted), and calls the replacement
cannot take (inputs that need autograd, shapes captured symbolically) run the
original ops."""
import pytest

pytestmark = pytest.mark.gpu


def _compile(fn):
    import torch
    from sym_b200.reloc_torch.backend import RelocBackend

    torch._dynamo.reset()
    backend = RelocBackend()
    return torch.compile(fn, backend=backend, dynamic=False), backend


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
