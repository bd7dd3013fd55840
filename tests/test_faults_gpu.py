"""Failure paths on the GPU, made without faulting the GPU.

Two kinds of failure are injected, both through test hooks of the thin CUDA
layer (libsb_cuda.so) that the library itself never arms:

* Host-side CUDA errors (``sbc_test_fault_mode``): event records, copies,
  event or stream synchronizations report ``cudaErrorUnknown`` on the host
  without being issued, after real work was enqueued. The contract checked is
  the reference's typed-context one (libreloc README "quarantine" section;
  python/tests/DispatchFaultShim.cpp with torch_frontend/test_dispatch.py:330,
  test_group.py:225, test_async_transfers.py:193): a failure whose completion
  can be proven retires the context (``backend_failure``; the next call gets a
  fresh context and is bit-exact); one whose completion cannot be proven is
  ``completion_unknown``, quarantines the owners for the life of the process,
  and the resources refuse all further work, while fresh resources still run
  bit-exact.
* A bounded device wait that runs out (``sbc_test_withhold_tile``): the TMA
  tile kernel withholds one tile's copy and arrival, so the warps waiting for
  it give up after a short time limit, set the context's fault word and leave.
  The call reports ``backend_failure``; the GPU context stays usable.
"""
import gc
import weakref

import numpy as np
import pytest

from helpers import WIDTH, dense, encode, recipe_c4

pytestmark = pytest.mark.gpu

OUT_F, IN_F = 512, 1024  # a TMA-tiled shape: 4 x 16 tiles of 128 x 64


def _plan(out_f=OUT_F, in_f=IN_F, seed=0):
    from sym_b200 import pyreloc

    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, size=(out_f, in_f), dtype=np.int8)
    scale = np.exp(rng.normal(-5, 0.5, out_f)).astype(np.float32)
    blob = encode(recipe_c4())
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params)
    return blob, sym, params, bound, q


def _want(ref_lib, blob, sym, params, q):
    return ref_lib.TypedProgram(blob, sym, params).execute(q.view(np.uint8).reshape(-1))


class _Call:
    """A prepared request over pinned host source and device destination."""

    def __init__(self, bound, q, route="dma_ring"):
        import torch
        from sym_b200 import pyreloc

        self.tmpl = pyreloc.prepare_dispatch_template(bound, "h2d", "cuda",
                                                      implementation=f"b200_fused_h2d@{route}")
        info = bound.describe()
        self.host = torch.from_numpy(q.view(np.uint8).reshape(-1).copy()).pin_memory()
        self.out = torch.full((bound.destination_bytes,), 0xA5, dtype=torch.uint8, device="cuda")
        self.sv = pyreloc.BufferView(self.host.data_ptr(), self.host.numel(), 0, info["source_extents"],
                                     dense(info["source_extents"]), WIDTH[info["source_dtype"]], "host", -1)
        self.dv = pyreloc.BufferView(self.out.data_ptr(), self.out.numel(), 0, info["result_extents"],
                                     dense(info["result_extents"]), WIDTH[info["result_dtype"]], "cuda", 0)

    def request(self):
        from sym_b200 import pyreloc

        return pyreloc.prepare_dispatch_from_template(self.tmpl, self.sv, self.dv)

    def result(self):
        import torch

        torch.cuda.synchronize()
        return self.out.cpu().numpy()


class _Owner:
    """A stand-in buffer owner whose lifetime the test observes."""


def _error_code(fn):
    """The TransferError code `fn` raises. The exception (and with it the
    traceback's frames, which hold the call's arguments) is dropped before
    returning, so only the library can keep an owner alive afterwards."""
    from sym_b200 import pyreloc

    try:
        fn()
    except pyreloc.TransferError as e:
        return e.code
    raise AssertionError("the call did not fail")


def _armed(mode, fn):
    from sym_b200 import _native

    hooks = _native.cuda_layer()
    assert hooks.sbc_test_fault_mode(mode) == 0
    try:
        return fn()
    finally:
        hooks.sbc_test_fault_mode(0)


@pytest.mark.parametrize("mode,code", [(1, "backend_failure"), (2, "completion_unknown"),
                                       (3, "backend_failure"), (4, "completion_unknown"),
                                       (5, "backend_failure"), (6, "completion_unknown")])
def test_host_side_cuda_errors_retire_or_quarantine(ref_lib, mode, code):
    import torch
    from sym_b200 import pyreloc

    blob, sym, params, bound, q = _plan(seed=mode)
    want = _want(ref_lib, blob, sym, params, q)
    res = pyreloc.DispatchResources()
    call = _Call(bound, q)
    # a healthy call first, so the failing one reuses a warm context
    pyreloc.execute_dispatch(call.request(), resources=res, chunk_size=64 * IN_F)
    assert np.array_equal(call.result(), want)
    owner = _Owner()
    ref = weakref.ref(owner)
    req = call.request()
    # small chunks: several copies and events, so mode 3/4's third copy exists
    seen = _error_code(lambda: _armed(mode, lambda: pyreloc.execute_dispatch(
        req, resources=res, chunk_size=64 * IN_F, owners=(owner,))))
    assert seen == code
    assert req.consumed
    del owner
    gc.collect()
    torch.cuda.synchronize()  # the injected errors never reached the GPU: drain it
    stats = res.stats()
    if code == "completion_unknown":
        assert stats["quarantined"]
        assert ref() is not None, "a quarantined owner was released"
        with pytest.raises(pyreloc.TransferError) as again:
            pyreloc.execute_dispatch(call.request(), resources=res)
        assert again.value.code == "completion_unknown"
        with pytest.raises(pyreloc.TransferError):
            res.close()
        # fresh resources are unaffected
        fresh = pyreloc.DispatchResources()
        call2 = _Call(bound, q)
        pyreloc.execute_dispatch(call2.request(), resources=fresh)
        assert np.array_equal(call2.result(), want)
        fresh.close()
    else:
        assert not stats["quarantined"]
        assert stats["retirements"] == 1 and stats["contexts"] == 0, stats
        assert ref() is None, "an owner was kept although completion was proven"
        call.out.fill_(0x5A)
        pyreloc.execute_dispatch(call.request(), resources=res)  # a fresh context
        assert np.array_equal(call.result(), want)
        assert res.stats()["contexts"] == 1
        res.close()


def test_submitted_group_whose_completion_cannot_be_proven_quarantines_its_owners(ref_lib):
    import torch
    from sym_b200 import pyreloc

    blob, sym, params, bound, q = _plan(seed=11)
    want = _want(ref_lib, blob, sym, params, q)
    res = pyreloc.DispatchResources(max_retained_bytes=256 << 20)
    call = _Call(bound, q)
    group = pyreloc.prepare_dispatch_group([(call.tmpl, call.sv, call.dv, "h2d")])
    owner = _Owner()
    ref = weakref.ref(owner)
    completion = pyreloc.submit_dispatch_group(group, resources=res, owners=(owner,))
    del owner
    assert _error_code(lambda: _armed(6, completion.wait)) == "completion_unknown"  # event wait and drain fail
    del completion
    gc.collect()
    assert ref() is not None
    torch.cuda.synchronize()
    assert np.array_equal(call.result(), want)  # the real work did run


def _withheld(fn, job=0, limit_ns=20_000_000):
    from sym_b200 import _native

    hooks = _native.cuda_layer()
    before = hooks.sbc_wait_launch_count()
    hooks.sbc_test_withhold_tile(job, limit_ns)
    try:
        return fn()
    finally:
        hooks.sbc_test_withhold_tile(0xFFFFFFFF, 0)
        assert hooks.sbc_wait_launch_count() > before, "no TMA tile kernel ran"


def test_bounded_wait_runs_out_blocking_call(ref_lib):
    from sym_b200 import pyreloc

    blob, sym, params, bound, q = _plan(seed=21)
    want = _want(ref_lib, blob, sym, params, q)
    res = pyreloc.DispatchResources()
    call = _Call(bound, q)
    req = call.request()
    with pytest.raises(pyreloc.TransferError) as info:
        _withheld(lambda: pyreloc.execute_dispatch(req, resources=res))
    assert info.value.code == "backend_failure"
    assert "bounded wait" in info.value.detail
    assert not np.array_equal(call.result(), want)  # the withheld tile was never written
    stats = res.stats()
    assert stats["retirements"] == 1 and not stats["quarantined"]
    call.out.fill_(0x5A)
    pyreloc.execute_dispatch(call.request(), resources=res)
    assert np.array_equal(call.result(), want)
    res.close()


def test_bounded_wait_runs_out_async_call_reported_by_the_next_call(ref_lib):
    """With asynchronous completion the call returns once enqueued; the fault
    word (host memory) is read by the next call on the same context."""
    import torch
    from sym_b200 import pyreloc

    blob, sym, params, bound, q = _plan(seed=22)
    want = _want(ref_lib, blob, sym, params, q)
    res = pyreloc.DispatchResources()
    call = _Call(bound, q)
    dsrc = call.host.to("cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def rows(async_completion):
        return pyreloc.execute_rows(call.tmpl, dsrc.data_ptr(), call.out.data_ptr(), 0, IN_F, device=0,
                                    host_source=False, resources=res, caller_stream=stream,
                                    async_completion=async_completion)

    _withheld(lambda: rows(True))
    torch.cuda.synchronize()
    with pytest.raises(pyreloc.TransferError) as info:
        rows(True)
    assert info.value.code == "backend_failure" and "bounded wait" in info.value.detail
    rows(False)
    assert np.array_equal(call.result(), want)
    res.close()


def test_bounded_wait_runs_out_in_a_submitted_group(ref_lib):
    from sym_b200 import pyreloc

    blob, sym, params, bound, q = _plan(seed=23)
    want = _want(ref_lib, blob, sym, params, q)
    res = pyreloc.DispatchResources(max_retained_bytes=256 << 20)
    call = _Call(bound, q)
    group = pyreloc.prepare_dispatch_group([(call.tmpl, call.sv, call.dv, "h2d")])
    completion = _withheld(lambda: pyreloc.submit_dispatch_group(group, resources=res))
    with pytest.raises(pyreloc.TransferError) as info:
        completion.wait()
    assert info.value.code == "backend_failure" and "bounded wait" in info.value.detail
    # the context stays usable: the fault was this group's, its streams are healthy
    call.out.fill_(0x5A)
    pyreloc.execute_dispatch(call.request(), resources=res)
    assert np.array_equal(call.result(), want)
    res.close()


def test_bounded_wait_runs_out_in_the_allocation_free_entry_point(ref_lib):
    import torch
    from sym_b200 import pyreloc

    blob, sym, params, bound, q = _plan(seed=24)
    want = _want(ref_lib, blob, sym, params, q)
    tmpl = pyreloc.prepare_dispatch_template(bound)
    host = torch.from_numpy(q.view(np.uint8).reshape(-1).copy()).pin_memory()
    out = torch.full((bound.destination_bytes,), 0xA5, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    with pytest.raises(pyreloc.TransferError) as info:
        _withheld(lambda: pyreloc.execute_h2d_static(tmpl, host.data_ptr(), out.data_ptr(), stream))
    assert info.value.code == "backend_failure" and "bounded wait" in info.value.detail
    out.fill_(0x5A)
    pyreloc.execute_h2d_static(tmpl, host.data_ptr(), out.data_ptr(), stream)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), want)

