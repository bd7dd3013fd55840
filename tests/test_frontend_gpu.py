"""The Torch-facing surfaces on the GPU: reloc_torch.dispatch (the typed bridge
of reloc_torch, libreloc/python/reloc_torch/dispatch.py) and WeightFetcher
(examples/workloads/common.py) produce the checker's bits and, for these
recipes, the same bits as the PyTorch reference computation."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _weights(rows, cols, seed):
    import torch

    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.integers(-128, 128, size=(rows, cols), dtype=np.int8))
    return q, rng


@pytest.mark.parametrize("shape", [(48, 200), (1024, 3072)])
def test_weight_fetcher_reference_recipe(shape):
    """int8 [in, out] + per-output scale (axis 1) -> f32 [out, in]."""
    import torch
    from sym_b200.workloads import WeightFetcher

    q, rng = _weights(*shape, seed=1)
    scale = torch.from_numpy(np.exp(rng.normal(-5, 0.5, shape[1])).astype(np.float32))
    with WeightFetcher() as wf:
        got = wf.fetch(q, scale, "cuda")
        again = wf.fetch(q, scale, "cuda")
        stats = wf.resource_stats()
    want = WeightFetcher.reference(q, scale, "cuda")
    assert got.dtype == torch.float32 and list(got.shape) == [shape[1], shape[0]]
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    assert torch.equal(again, got)
    assert wf.report.data["dispatches"] and all(k.startswith("b200_fused_h2d") for k in wf.report.data["dispatches"])
    assert list(stats.values())[0]["requests"] >= 2


@pytest.mark.parametrize("shape", [(4096, 4096), (1000, 2304)])
def test_weight_fetcher_f16_recipe(shape):
    """int8 [out, in] + per-row scale -> f16 [in, out] (the weight-streaming configs)."""
    import torch
    from sym_b200.workloads import WeightFetcher

    q, rng = _weights(*shape, seed=2)
    scale = torch.from_numpy(np.exp(rng.normal(-5, 0.5, shape[0])).astype(np.float32))
    with WeightFetcher(layout="out_in_f16") as wf:
        got = wf.fetch(q, scale, "cuda")
    want = WeightFetcher.reference(q, scale, "cuda", layout="out_in_f16")
    assert got.dtype == torch.float16 and list(got.shape) == [shape[1], shape[0]]
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_weight_fetcher_matches_pytorch_for_every_shape_with_one_artifact():
    """One compiled recipe serves every matrix shape (reference
    test_workload_common.py:186-203); the raw int8 crosses the wire."""
    import torch
    from sym_b200.workloads import Report, WeightFetcher, quantize_per_channel

    report = Report()
    generator = torch.Generator().manual_seed(1)
    with WeightFetcher(report) as fetcher:
        for rows, cols in ((64, 96), (96, 64), (128, 128)):
            q, scale = quantize_per_channel(torch.randn(rows, cols, generator=generator))
            got = fetcher.fetch(q, scale, "cuda:0")
            want = WeightFetcher.reference(q, scale, "cuda:0")
            assert got.shape == (cols, rows) and got.dtype == torch.float32
            assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    assert fetcher.compiles == 1 and fetcher.shapes == {(64, 96), (96, 64), (128, 128)}
    assert report.data["plan_compiles"] == 1
    weights = report.data["bytes"]["weights"]
    assert weights["transfers"] == 3 and weights["wire"] == weights["source"]
    assert weights["destination"] == 4 * weights["source"]
    assert sum(report.data["dispatches"].values()) == 3
    assert all(k.startswith("b200_fused_h2d") for k in report.data["dispatches"])


@pytest.mark.skipif("__import__('torch').cuda.device_count() < 2", reason="needs two GPUs")
def test_weight_fetcher_reaches_a_device_that_is_not_current():
    """Alternating destination devices keeps one warm owner per device and
    leaves the current device alone (reference test_workload_common.py:206-225)."""
    import torch
    from sym_b200.workloads import Report, WeightFetcher, quantize_per_channel

    report = Report()
    fetcher = WeightFetcher(report, kind="expert_weights", layout="out_in_f16")
    q, scale = quantize_per_channel(torch.randn(512, 256, generator=torch.Generator().manual_seed(2)),
                                    "out_in_f16")
    with torch.cuda.device(0), fetcher:
        for device in ("cuda:0", "cuda:1", "cuda:0", "cuda:1"):
            got = fetcher.fetch(q, scale, device)
            assert torch.cuda.current_device() == 0 and got.device == torch.device(device)
            want = WeightFetcher.reference(q, scale, device, layout="out_in_f16")
            assert torch.equal(got.view(torch.int16), want.view(torch.int16))
        stats = fetcher.resource_stats()
        assert len(stats) == 2 and all(s["requests"] == 2 and s["contexts"] == 1 for s in stats.values())
    assert report.data["bytes"]["expert_weights"]["transfers"] == 4


def test_fetch_many_and_stream_ordering():
    """Outputs follow the caller's current stream: work queued on a side
    stream before the fetch is ordered before it."""
    import torch
    from sym_b200.workloads import WeightFetcher

    side = torch.cuda.Stream()
    pairs = []
    for seed, shape in enumerate([(256, 512), (512, 256), (64, 1024)]):
        q, rng = _weights(*shape, seed=10 + seed)
        pairs.append((q, torch.from_numpy(np.exp(rng.normal(-5, 0.5, shape[0])).astype(np.float32))))
    with WeightFetcher(layout="out_in_f16") as wf, torch.cuda.stream(side):
        outs = wf.fetch_many(pairs, "cuda")
        sums = [o.float().sum() for o in outs]  # consumed on the same (side) stream
    torch.cuda.synchronize()
    for (q, s), o, total in zip(pairs, outs, sums):
        want = WeightFetcher.reference(q, s, "cuda", layout="out_in_f16")
        assert torch.equal(o.view(torch.int16), want.view(torch.int16))
        assert torch.allclose(total, want.float().sum())


def test_typed_bridge_rejections():
    import torch
    from sym_b200.reloc_torch import dispatch
    from sym_b200.reloc_torch.compiler import CompilerClient, UnsupportedRecipe
    from sym_b200.workloads import weight_recipe

    compiled = CompilerClient().compile(weight_recipe("out_in_f16"))
    q = torch.zeros((8, 16), dtype=torch.int8)
    with pytest.raises(UnsupportedRecipe):
        dispatch.prepare_typed_transfer(compiled, q, "cuda", parameters={})  # missing scale
    with pytest.raises(UnsupportedRecipe):
        dispatch.prepare_typed_transfer(compiled, q.t(), "cuda", parameters={"scale": torch.ones(16)})
    with pytest.raises(UnsupportedRecipe):
        dispatch.prepare_typed_transfer(compiled, q, "cuda", parameters={"scale": torch.ones(8, dtype=torch.float64)})
    req = dispatch.prepare_typed_transfer(compiled, q, "cuda", parameters={"scale": torch.ones(8)})
    dispatch.execute_typed_transfer(req)
    with pytest.raises(RuntimeError):
        dispatch.execute_typed_transfer(req)  # single-use
