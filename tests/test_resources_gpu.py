"""Typed-context scratch budgets on the GPU (reference docs/typed-contexts.md,
"Budgets and admission"): the owner's retained and live limits are divided
into per-context quotas; a nonzero live limit caps the scratch one execution
may hold (chunks shrink to fit, insufficient_capacity when not even one row
fits); scratch beyond the retained quota is released when a blocking lease
ends; at the context limit the least recently used context is retired."""
import numpy as np
import pytest

from helpers import WIDTH, dense, encode, recipe_c4
from test_gpu_parity import _c4_inputs, expected

pytestmark = pytest.mark.gpu


def _run(res, blob, sym, params, q, route="dma_ring", device=0):
    import torch
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params)
    tmpl = pyreloc.prepare_dispatch_template(bound, "h2d", "cuda")
    info = bound.describe()
    host = torch.from_numpy(np.ascontiguousarray(q).view(np.uint8).reshape(-1).copy()).pin_memory()
    out = torch.empty(bound.destination_bytes, dtype=torch.uint8, device=f"cuda:{device}")
    sv = pyreloc.BufferView(host.data_ptr(), host.numel(), 0, info["source_extents"],
                            dense(info["source_extents"]), WIDTH[info["source_dtype"]], "host", -1)
    dv = pyreloc.BufferView(out.data_ptr(), out.numel(), 0, info["result_extents"],
                            dense(info["result_extents"]), WIDTH[info["result_dtype"]], "cuda", device)
    rep = pyreloc.execute_dispatch(pyreloc.prepare_dispatch_from_template(tmpl, sv, dv), resources=res, route=route)
    return out.cpu().numpy(), dict(rep)


def _case(out_f=2048, in_f=4096, seed=31):
    q, scale = _c4_inputs(out_f, in_f, seed=seed)
    return (encode(recipe_c4()), {"out_features": out_f, "in_features": in_f},
            {"scale": ("float32", [out_f], scale.tobytes())}, q)


def test_live_limit_shrinks_the_ring_and_stays_exact():
    from sym_b200 import pyreloc

    blob, sym, params, q = _case()  # 8 MiB of int8 rows of 4 KiB
    live = 3 << 20
    res = pyreloc.DispatchResources(max_live_bytes=live)
    out, rep = _run(res, blob, sym, params, q)
    assert np.array_equal(out, expected(blob, sym, params, q))
    st = res.stats()
    assert st["peak_live_bytes"] <= live and rep["host_chunk_bytes"] * 4 <= live
    assert rep["host_chunks"] > 1
    res.close()


def test_live_limit_too_small_for_one_row_is_insufficient_capacity():
    from sym_b200 import pyreloc

    blob, sym, params, q = _case(256, 65536)  # rows of 64 KiB; 4 ring slots cannot fit in 128 KiB
    res = pyreloc.DispatchResources(max_live_bytes=128 << 10)
    with pytest.raises(pyreloc.TransferError) as info:
        _run(res, blob, sym, params, q)
    assert info.value.code == "insufficient_capacity"
    # the context is not poisoned: a plan that fits still runs exactly
    blob2, sym2, params2, q2 = _case(64, 256)
    out, _ = _run(res, blob2, sym2, params2, q2)
    assert np.array_equal(out, expected(blob2, sym2, params2, q2))
    res.close()


def test_retained_quota_releases_scratch_after_blocking_calls():
    from sym_b200 import pyreloc

    blob, sym, params, q = _case()
    res = pyreloc.DispatchResources(max_retained_bytes=1 << 20)
    for _ in range(2):
        out, _ = _run(res, blob, sym, params, q)
        assert np.array_equal(out, expected(blob, sym, params, q))
    st = res.stats()
    assert st["retained_bytes"] <= 1 << 20 and st["releases"] >= 2
    assert st["peak_live_bytes"] > 1 << 20  # the ring existed while the call ran
    keep = pyreloc.DispatchResources(max_retained_bytes=256 << 20)
    _run(keep, blob, sym, params, q)
    _run(keep, blob, sym, params, q)
    assert keep.stats()["releases"] == 0 and keep.stats()["retained_bytes"] > 1 << 20
    res.close()
    keep.close()


@pytest.mark.skipif("__import__('torch').cuda.device_count() < 2", reason="needs two GPUs")
def test_context_limit_retires_the_least_recently_used_context():
    import torch
    from sym_b200 import pyreloc

    blob, sym, params, q = _case(256, 512)
    want = expected(blob, sym, params, q)
    res = pyreloc.DispatchResources(max_contexts=1)
    with torch.cuda.device(0):
        for device in (0, 1, 0):
            out, _ = _run(res, blob, sym, params, q, device=device)
            assert np.array_equal(out, want) and torch.cuda.current_device() == 0
    st = res.stats()
    assert st["contexts"] == 1 and st["evictions"] == 2
    res.close()


def test_acquire_timeout_bounds_the_wait_for_a_busy_context():
    """A call that finds its context leased by another call fails with
    acquire_timeout after ``acquire_timeout_ms`` (0: at once), and a call
    that may wait long enough runs once the lease ends (reference
    DispatchResources acquireTimeoutMs)."""
    import threading
    import time

    import torch
    from sym_b200 import pyreloc

    blob, sym, params, q = _case(64, 256)
    want = expected(blob, sym, params, q)
    busy = pyreloc.DispatchResources(acquire_timeout_ms=0)
    # a long blocking call holds the context: 1.5 GiB from pageable memory
    big_blob, big_sym, big_params, big = _case(49152, 32768, seed=5)
    started, done = threading.Event(), threading.Event()

    def hold():
        from sym_b200 import pyreloc as p

        bound = p.bind_typed(p.load_typed_plan(big_blob), big_sym, big_params)
        tmpl = p.prepare_dispatch_template(bound, "h2d", "cuda")
        info = bound.describe()
        out = torch.empty(bound.destination_bytes, dtype=torch.uint8, device="cuda:0")
        sv = p.BufferView(big.ctypes.data, big.nbytes, 0, info["source_extents"], dense(info["source_extents"]),
                          1, "host", -1)
        dv = p.BufferView(out.data_ptr(), out.numel(), 0, info["result_extents"], dense(info["result_extents"]),
                          2, "cuda", 0)
        req = p.prepare_dispatch_from_template(tmpl, sv, dv)
        started.set()
        p.execute_dispatch(req, resources=busy, route="dma_ring")
        done.set()

    t = threading.Thread(target=hold)
    t.start()
    started.wait()
    time.sleep(0.005)
    raised = None
    if not done.is_set():
        with pytest.raises(pyreloc.TransferError) as info:
            _run(busy, blob, sym, params, q)
        raised = info.value.code
    t.join()
    assert raised in ("acquire_timeout", None)
    assert raised == "acquire_timeout" or done.is_set()
    patient = pyreloc.DispatchResources(acquire_timeout_ms=60_000)
    out, _ = _run(patient, blob, sym, params, q)
    assert np.array_equal(out, want)
    out, _ = _run(busy, blob, sym, params, q)  # idle now: the zero timeout admits at once
    assert np.array_equal(out, want)
    busy.close()
    patient.close()
