"""Groups, asynchronous submission and prefetch on the GPU: every member of
a group (pyreloc.execute_dispatch_group / submit_dispatch_group) and every
output of the Torch queue (reloc_torch.TransferQueue, PrefetchWindow,
WeightFetcher.fetch_many / prefetch) is bit-identical to the checker, with
one caller-stream wait per group."""
import numpy as np
import pytest

from helpers import dense, encode, recipe_c2, recipe_c3, recipe_c4, resources

pytestmark = pytest.mark.gpu


def _c4_member(out_f, in_f, seed):
    import torch
    from sym_b200 import pyreloc

    rng = np.random.default_rng(seed)
    q = rng.integers(-128, 128, size=(out_f, in_f), dtype=np.int8)
    scale = np.exp(rng.normal(-5, 0.5, out_f)).astype(np.float32)
    blob = encode(recipe_c4())
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    tmpl = pyreloc.prepare_dispatch_template(pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params))
    host = torch.from_numpy(q.copy()).pin_memory()
    out = torch.empty((in_f, out_f), dtype=torch.float16, device="cuda")
    sv = pyreloc.BufferView(host.data_ptr(), host.numel(), 0, [out_f, in_f], dense([out_f, in_f]), 1, "host", -1)
    dv = pyreloc.BufferView(out.data_ptr(), out.numel() * 2, 0, [in_f, out_f], dense([in_f, out_f]), 2, "cuda", 0)
    return (tmpl, sv, dv, "h2d"), host, out, (blob, sym, params, q)


def _c3_member(seq, seed):
    import torch
    from sym_b200 import pyreloc

    x = np.random.default_rng(seed).standard_normal(8 * seq * 4096).astype(np.float32)
    blob = encode(recipe_c3("quantize"))
    sym = {"B": 8, "S": seq}
    tmpl = pyreloc.prepare_dispatch_template(pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, {}))
    host = torch.from_numpy(x.copy()).pin_memory()
    out = torch.empty(x.size, dtype=torch.int8, device="cuda")
    ext = [8, seq, 4096]
    sv = pyreloc.BufferView(host.data_ptr(), x.nbytes, 0, ext, dense(ext), 4, "host", -1)
    dv = pyreloc.BufferView(out.data_ptr(), x.size, 0, ext, dense(ext), 1, "cuda", 0)
    return (tmpl, sv, dv, "h2d"), host, out, (blob, sym, {}, x)


def _expected(blob, sym, params, src):
    from oracle import ref

    if not ref.available():
        pytest.skip("reference runtime (oracle/_ref) not built")
    return ref.TypedProgram(blob, sym, params).execute(np.ascontiguousarray(src).view(np.uint8).reshape(-1))


def _members():
    return [_c4_member(96, 200, 1), _c4_member(1024, 4096, 2), _c3_member(3, 3), _c4_member(257, 131, 4)]


@pytest.mark.parametrize("route", ["auto", "dma_ring", "zero_copy"])
def test_group_executes_every_member_exactly(route):
    import torch
    from sym_b200 import pyreloc

    members = _members()
    g = pyreloc.prepare_dispatch_group([m[0] for m in members])
    stream = torch.cuda.current_stream()
    rep = pyreloc.execute_dispatch_group(g, caller_stream=stream.cuda_stream, resources=resources(), route=route)
    assert rep["logical_transfers"] == len(members) and rep["caller_waits"] == 1
    assert len(rep["items"]) == len(members) and all(i["executed"] for i in rep["items"])
    assert rep["kernel_launches"] >= len(members)
    for _, _, out, (blob, sym, params, src) in members:
        got = out.view(torch.uint8).cpu().numpy().reshape(-1)
        assert np.array_equal(got, _expected(blob, sym, params, src))
    with pytest.raises(pyreloc.TransferError):
        pyreloc.execute_dispatch_group(g, resources=resources())


def test_submitted_group_completes_through_a_consumer_stream():
    """submit returns before the host waits; a consumer stream ordered by
    wait_stream() reads finished outputs; wait()/query() then agree."""
    import torch
    from sym_b200 import pyreloc

    members = _members()
    g = pyreloc.prepare_dispatch_group([m[0] for m in members])
    c = pyreloc.submit_dispatch_group(g, resources=resources(), owners=[m[1:3] for m in members])
    consumer = torch.cuda.Stream()
    c.wait_stream(consumer.cuda_stream)
    with torch.cuda.stream(consumer):
        copies = [m[2].clone() for m in members]  # read on the consumer stream only
    consumer.synchronize()
    c.wait()
    assert c.query() is True
    for copy, (_, _, _, (blob, sym, params, src)) in zip(copies, members):
        assert np.array_equal(copy.view(torch.uint8).cpu().numpy().reshape(-1), _expected(blob, sym, params, src))


def test_submit_without_resources_and_drop_without_wait():
    """A private context lives as long as the completion; dropping the
    handle waits for the group."""
    import torch
    from sym_b200 import pyreloc

    members = [_c4_member(128, 256, 7), _c3_member(1, 8)]
    g = pyreloc.prepare_dispatch_group([m[0] for m in members])
    c = pyreloc.submit_dispatch_group(g)
    del c
    torch.cuda.synchronize()
    for _, _, out, (blob, sym, params, src) in members:
        assert np.array_equal(out.view(torch.uint8).cpu().numpy().reshape(-1), _expected(blob, sym, params, src))


def _layers(n, shapes, seed=20):
    import torch

    rng = np.random.default_rng(seed)
    layers = []
    for _ in range(n):
        pairs = []
        for out_f, in_f in shapes:
            q = torch.from_numpy(rng.integers(-128, 128, size=(out_f, in_f), dtype=np.int8))
            s = torch.from_numpy(np.exp(rng.normal(-5, 0.5, out_f)).astype(np.float32))
            pairs.append((q, s))
        layers.append(pairs)
    return layers


def test_weight_fetcher_fetch_many_is_one_group():
    import torch
    from sym_b200.workloads import WeightFetcher

    (pairs,) = _layers(1, [(256, 512), (512, 256), (64, 1024), (1024, 4096)])
    with WeightFetcher(layout="out_in_f16") as wf:
        outs = wf.fetch_many(pairs, "cuda")
        groups = wf.report.data["transfer_groups"]
    assert groups["groups"] == 1 and groups["logical_transfers"] == 4 and groups["caller_waits"] == 1
    for (q, s), o in zip(pairs, outs):
        want = WeightFetcher.reference(q, s, "cuda", layout="out_in_f16")
        assert torch.equal(o.view(torch.int16), want.view(torch.int16))


def test_prefetch_window_streams_layers_in_order():
    """Layer i+1 is in flight while layer i is consumed on the current
    stream; every consumed output equals the PyTorch reference."""
    import torch
    from sym_b200.workloads import WeightFetcher

    layers = _layers(5, [(512, 1024), (1024, 512), (256, 2048)], seed=30)
    sums = []
    with WeightFetcher(layout="out_in_f16") as wf:
        with wf.prefetch(layers, "cuda", max_output_bytes=64 << 20) as window:
            for outs in window:
                sums.append(torch.stack([o.float().sum() for o in outs]))  # consumer kernels, current stream
        stats = wf.report.data["weight_prefetch"]
    torch.cuda.synchronize()
    (only,) = stats.values()
    assert only["submitted"] == 5 and only["held"] == 0 and only["peak_in_flight"] <= 2
    assert only["totals"]["logical_transfers"] == 15
    for pairs, got in zip(layers, sums):
        want = torch.stack([WeightFetcher.reference(q, s, "cuda", layout="out_in_f16").float().sum()
                            for q, s in pairs])
        assert torch.equal(got, want)


def test_transfer_queue_budget_and_completion_lifecycle():
    import torch
    from sym_b200.reloc_torch import TransferQueue
    from sym_b200.workloads import WeightFetcher

    layers = _layers(3, [(256, 256)], seed=40)
    with WeightFetcher(layout="out_in_f16") as wf, TransferQueue("cuda:0", max_in_flight=2) as queue:
        h0 = queue.submit(wf.prepare_many(layers[0], "cuda"))
        h1 = queue.submit(wf.prepare_many(layers[1], "cuda"))
        g2 = wf.prepare_many(layers[2], "cuda")
        assert not queue.can_submit(g2)
        with pytest.raises(BufferError):
            queue.submit(g2)
        (t0,) = h0.wait_stream()
        want = WeightFetcher.reference(*layers[0][0], "cuda", layout="out_in_f16")
        assert torch.equal(t0.view(torch.int16), want.view(torch.int16))
        h0.release()
        h0.close()
        assert queue.can_submit(g2)
        h2 = queue.submit(g2)
        res = h2.wait()
        assert h2.done()
        want2 = WeightFetcher.reference(*layers[2][0], "cuda", layout="out_in_f16")
        assert torch.equal(res.tensors[0].view(torch.int16), want2.view(torch.int16))
        assert res.report["logical_transfers"] == 1
        h1.close()
        h2.close()
        stats = queue.stats()
    assert stats["held"] == 0 and stats["submitted"] == 3 and stats["totals"]["groups"] == 3
