"""Host-side pieces of the weight-streaming workload: the offline int8
preparation ``quantize_per_channel`` (reference
examples/workloads/common.py:368-378, test_workload_common.py:146-154) and the
fetcher's argument checks. Nothing here touches a GPU."""
import pytest


@pytest.mark.parametrize("layout", ["reference", "out_in_f16"])
def test_quantize_per_channel_is_symmetric_int8_per_output_channel(layout):
    import torch
    from sym_b200.workloads import quantize_per_channel

    weight = torch.randn(64, 48, generator=torch.Generator().manual_seed(0))
    if layout == "out_in_f16":
        weight = weight.t().contiguous()  # [out, in]
        weight[5, :] = 0.0
    else:
        weight[:, 5] = 0.0  # an all-zero channel still gets a positive scale
    q, scale = quantize_per_channel(weight, layout)
    per_channel = weight if layout == "reference" else weight.t()  # [in, out] view
    qc = q if layout == "reference" else q.t()
    assert q.dtype == torch.int8 and q.shape == weight.shape and q.is_contiguous()
    assert scale.dtype == torch.float32 and scale.shape == (48,) and bool((scale > 0).all())
    assert int(q.abs().max()) <= 127 and bool((qc[:, 5] == 0).all())
    assert torch.allclose(scale[:5], per_channel[:, :5].abs().amax(dim=0) / 127)
    assert bool(((qc.float() * scale - per_channel).abs() <= scale / 2 + 1e-6).all())


def test_weight_fetcher_argument_checks():
    from sym_b200.workloads import WeightFetcher, quantize_per_channel

    with pytest.raises(ValueError):
        WeightFetcher(resource_policy="sometimes")
    with pytest.raises(ValueError):
        quantize_per_channel(None, layout="in_out_f8")
    wf = WeightFetcher()
    wf.close()
    with pytest.raises(RuntimeError):
        wf.fetch(None, None, "cuda")
    with pytest.raises(RuntimeError):
        with wf:
            pass
