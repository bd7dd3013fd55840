"""The allocation-free entry point (sb_execute_h2d_static).

Some callers cannot allocate device memory -- a caching allocator owns the
heap, the process has a fixed device budget, or allocation is forbidden
between graph captures. For them the library stages through a statically
allocated device array instead of a context's HBM ring. These tests call that
entry point through the C-ABI and require its output to equal, bit for bit,
what the allocating entry point (execute_dispatch) produces for the same plan
and input, on two calls in a row (the array keeps the previous call's
contents, so the second call checks that nothing stale leaks through).

Kept in a file collected last, so a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

from helpers import encode, recipe_c3, recipe_c4, run_typed_gpu

pytestmark = pytest.mark.gpu


def _static_twice(blob, symbols, params, src):
    import torch
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), symbols, params)
    tmpl = pyreloc.prepare_dispatch_template(bound)
    host = torch.from_numpy(np.ascontiguousarray(src).view(np.uint8).reshape(-1).copy()).pin_memory()
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):
        out = torch.full((bound.destination_bytes,), 0xA5, dtype=torch.uint8, device="cuda")
        pyreloc.execute_h2d_static(tmpl, host.data_ptr(), out.data_ptr(), stream)
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
    return outs


def _reference(blob, symbols, params, src):
    """The reference CPU executor's bytes, when its build is present."""
    from oracle import ref

    if not ref.available():
        return None
    return ref.TypedProgram(blob, symbols, params).execute(np.ascontiguousarray(src).view(np.uint8).reshape(-1))


def test_static_entry_point_matches_execute_dispatch_weights():
    """int8 [out, in] -> dequantize (per-row scale) -> f16 -> transpose, with
    more source rows than one staging slot holds (several chunks per call)."""
    rng = np.random.default_rng(5)
    out_f, in_f = 2600, 16384  # 42.6 MB of int8: two chunks through the 31 MiB slot
    q = rng.integers(-128, 128, size=(out_f, in_f), dtype=np.int8)
    scale = np.exp(rng.normal(-5, 0.5, out_f)).astype(np.float32)
    blob = encode(recipe_c4())
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    want, _ = run_typed_gpu(blob, sym, params, q, route="dma_ring")
    first, second = _static_twice(blob, sym, params, q)
    assert np.array_equal(first, want)
    assert np.array_equal(second, want)
    reference = _reference(blob, sym, params, q)
    assert reference is None or np.array_equal(first, reference)


def test_static_entry_point_matches_execute_dispatch_quantize():
    """f32 -> s8 per-tensor quantize (contiguous kernel), specials included."""
    rng = np.random.default_rng(6)
    x = rng.standard_normal(8 * 7 * 4096).astype(np.float32)
    x[:6] = [np.nan, np.inf, -np.inf, 2.5, -2.5, 1e-40]
    blob = encode(recipe_c3("quantize"))
    want, _ = run_typed_gpu(blob, {"B": 8, "S": 7}, {}, x, route="dma_ring")
    first, second = _static_twice(blob, {"B": 8, "S": 7}, {}, x)
    assert np.array_equal(first, want)
    assert np.array_equal(second, want)
    reference = _reference(blob, {"B": 8, "S": 7}, {}, x)
    assert reference is None or np.array_equal(first, reference)


def test_static_entry_point_rejects_rows_beyond_the_scratch():
    """A single source row larger than the staging slot is refused up front."""
    import torch
    from sym_b200 import pyreloc

    out_f, in_f = 2, 40 << 20  # one 40 MiB source row
    blob = encode(recipe_c4())
    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), {"out_features": out_f, "in_features": in_f},
                               {"scale": ("float32", [out_f], np.ones(out_f, np.float32).tobytes())})
    tmpl = pyreloc.prepare_dispatch_template(bound)
    host = torch.zeros(out_f * in_f, dtype=torch.int8)
    out = torch.empty(bound.destination_bytes, dtype=torch.uint8, device="cuda")
    with pytest.raises(pyreloc.TransferError) as info:
        pyreloc.execute_h2d_static(tmpl, host.data_ptr(), out.data_ptr(), None)
    assert info.value.code == "invalid_options"
