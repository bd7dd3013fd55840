"""Parity at the benchmark configurations' full sizes.

Every configuration of the benchmark is run at the sizes the benchmark names
and compared byte for byte with the reference's own CPU executor
(oracle/_ref: decodeTypedPlan + bindTyped + typed::executeHost, or the layout
executor for the wire-v0 plan), the checker the reference's conformance suite
uses (libreloc/python/tests/test_typed_conformance.py:83,
CudaDispatch.EveryEligibleHostToDeviceRowMatchesTheReference). Seeded
synthetic inputs with the configurations' distributions stand in for data.

The multi-GPU fetch's assembly (one tile launch reading N source-row shards,
picked per 64-row tile) is checked here on one GPU with all shards in local
memory, at the full Llama-70B matrix sizes and with the uneven 64-row
aligned shard bounds the bench derives from per-GPU bandwidth weights.
"""
import hashlib
import os

import numpy as np
import pytest

from helpers import WIDTH, dense, encode, recipe_c1, recipe_c2, recipe_c3, recipe_c4

pytestmark = pytest.mark.gpu

LLAMA70B = {"q": (8192, 8192), "k": (1024, 8192), "v": (1024, 8192), "o": (8192, 8192),
            "gate": (28672, 8192), "up": (28672, 8192), "down": (8192, 28672)}
LLAMA7B = {"q": (4096, 4096), "k": (4096, 4096), "v": (4096, 4096), "o": (4096, 4096),
           "gate": (11008, 4096), "up": (11008, 4096), "down": (4096, 11008)}


@pytest.fixture(scope="module")
def pool(ref_lib):
    return ref_lib.GatherPool(len(os.sched_getaffinity(0)))


@pytest.fixture(scope="module")
def res():
    from sym_b200 import pyreloc

    r = pyreloc.DispatchResources(max_retained_bytes=1 << 30)
    yield r
    r.close()


def _weights(out_f, in_f, seed):
    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, size=(out_f, in_f), dtype=np.int8)
    scale = np.exp(rng.normal(-5.0, 0.5, out_f)).astype(np.float32)
    return q, scale


def _typed_gpu(res, blob, sym, params, src, route="dma_ring"):
    import torch
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params)
    tmpl = pyreloc.prepare_dispatch_template(bound, "h2d", "cuda", implementation=f"b200_fused_h2d@{route}")
    info = bound.describe()
    host = torch.from_numpy(np.ascontiguousarray(src).reshape(-1).view(np.uint8)).pin_memory()
    out = torch.empty(bound.destination_bytes, dtype=torch.uint8, device="cuda")
    sv = pyreloc.BufferView(host.data_ptr(), host.numel(), 0, info["source_extents"], dense(info["source_extents"]),
                            WIDTH[info["source_dtype"]], "host", -1)
    dv = pyreloc.BufferView(out.data_ptr(), out.numel(), 0, info["result_extents"], dense(info["result_extents"]),
                            WIDTH[info["result_dtype"]], "cuda", 0)
    rep = pyreloc.execute_dispatch(pyreloc.prepare_dispatch_from_template(tmpl, sv, dv), resources=res)
    return out, tmpl, dict(rep)


def _ref_typed(ref_lib, pool, blob, sym, params, src):
    p = ref_lib.TypedProgram(blob, sym, params)
    dst = np.empty(p.info["destination_bytes"], np.uint8)
    p.execute_into(np.ascontiguousarray(src).reshape(-1).view(np.uint8), dst, pool=pool)
    return dst


def _same(gpu_tensor, want):
    got = gpu_tensor.cpu().numpy()
    if not np.array_equal(got, want):
        bad = np.flatnonzero(got != want)
        raise AssertionError(f"{bad.size} bytes differ, first at {bad[:8].tolist()}")


@pytest.mark.parametrize("name", ["gate", "down"])
def test_llama70b_matrix_full_size_matches_reference(ref_lib, pool, res, name):
    """The headline workload's largest matrices, [28672, 8192] and
    [8192, 28672] int8 -> per-row dequantize -> f16 -> transpose, through the
    host-pinned DMA ring (the bench's host path) and from device memory (the
    bench's device-resident path)."""
    import torch
    from sym_b200 import pyreloc

    out_f, in_f = LLAMA70B[name]
    q, scale = _weights(out_f, in_f, seed=4)
    blob = encode(recipe_c4())
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    want = _ref_typed(ref_lib, pool, blob, sym, params, q)
    out, tmpl, rep = _typed_gpu(res, blob, sym, params, q)
    assert rep["device_kernel"] == "transpose"
    _same(out, want)
    dsrc = torch.from_numpy(q.reshape(-1).view(np.uint8)).to("cuda")
    out.fill_(0)
    pyreloc.execute_rows(tmpl, dsrc.data_ptr(), out.data_ptr(), 0, in_f, device=0, host_source=False, resources=res)
    _same(out, want)


@pytest.mark.parametrize("weights", [(1.0,) * 8, (23.3, 23.4, 23.6, 23.4, 35.8, 36.0, 35.9, 36.0), (1.0, 3.0)])
def test_llama70b_sharded_assembly_full_size_matches_reference(ref_lib, pool, res, weights):
    """The multi-GPU fetch's kernel: all N source-row shards of a full gate
    matrix (bounds from per-GPU weights, 64-row aligned) read by one tile
    launch, each shard a separate buffer, against the reference result."""
    import torch
    from sym_b200 import pyreloc
    from sym_b200.workloads import weighted_row_bounds

    out_f, in_f = LLAMA70B["gate"]
    q, scale = _weights(out_f, in_f, seed=7)
    blob = encode(recipe_c4())
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    want = _ref_typed(ref_lib, pool, blob, sym, params, q)
    bounds = weighted_row_bounds(out_f, list(weights))
    assert all((b1 - b0) % 64 == 0 for b0, b1 in zip(bounds, bounds[1:]))
    shards = [torch.from_numpy(np.ascontiguousarray(q[b0:b1]).reshape(-1).view(np.uint8)).to("cuda")
              for b0, b1 in zip(bounds, bounds[1:])]
    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params)
    tmpl = pyreloc.prepare_dispatch_template(bound)
    out = torch.zeros(bound.destination_bytes, dtype=torch.uint8, device="cuda")
    rep = pyreloc.execute_source_shards(tmpl, [s.data_ptr() for s in shards], bounds, out.data_ptr(), device=0,
                                        resources=res)
    assert rep["kernel_launches"] == 1  # one launch over all shards
    _same(out, want)
    # and shard by shard (the per-window path)
    out.fill_(0)
    for s, b0, b1 in zip(shards, bounds, bounds[1:]):
        pyreloc.execute_source_rows(tmpl, s.data_ptr(), b0, b1, out.data_ptr(), device=0, resources=res)
    _same(out, want)


def test_llama7b_full_layer_matches_reference(ref_lib, pool, res):
    """C4: one whole Llama-7B layer (7 matrices) through the DMA ring."""
    blob = encode(recipe_c4())
    for k, (name, (out_f, in_f)) in enumerate(LLAMA7B.items()):
        q, scale = _weights(out_f, in_f, seed=k)
        sym = {"out_features": out_f, "in_features": in_f}
        params = {"scale": ("float32", [out_f], scale.tobytes())}
        out, _, _ = _typed_gpu(res, blob, sym, params, q)
        _same(out, _ref_typed(ref_lib, pool, blob, sym, params, q))


@pytest.mark.parametrize("n", [1 << 20, 1 << 22, 1 << 24])
def test_c1_transpose_at_baseline_sizes(ref_lib, res, n):
    """C1: f32 [N] -> [N/64, 64] -> transpose -> [64, N/64] (wire v0), the
    symbol rebound per size without re-encoding."""
    import torch
    from sym_b200 import pyreloc

    blob = encode(recipe_c1())
    x = np.random.default_rng(0).uniform(-1.0, 1.0, n).astype(np.float32)
    want = ref_lib.LayoutPlan(blob, {"N": n}).execute(x.view(np.uint8), threads=len(os.sched_getaffinity(0)))
    bound = pyreloc.bind(pyreloc.load_plan(blob), {"N": n})
    host = torch.from_numpy(x.view(np.uint8)).pin_memory()
    out = torch.empty(4 * n, dtype=torch.uint8, device="cuda")
    sv = pyreloc.BufferView(host.data_ptr(), host.numel(), 0, [n], [1], 4, "host", -1)
    dv = pyreloc.BufferView(out.data_ptr(), out.numel(), 0, [n], [1], 4, "cuda", 0)
    pyreloc.execute_dispatch(pyreloc.make_transfer(bound, sv, dv), resources=res)
    _same(out, want)


def test_c2_full_batch_matches_reference(ref_lib, pool, res):
    """C2: f32 NCHW [64, 3, 224, 224] -> NHWC -> pad C 3 -> 4 -> f16."""
    blob = encode(recipe_c2())
    x = np.random.default_rng(0).uniform(0.0, 1.0, (64, 3, 224, 224)).astype(np.float32)
    out, _, _ = _typed_gpu(res, blob, {}, {}, x)
    _same(out, _ref_typed(ref_lib, pool, blob, {}, {}, x))


@pytest.mark.parametrize("s", [128, 1024, 8192])
def test_c3_quantize_and_dequantize_at_baseline_sizes(ref_lib, pool, res, s):
    """C3q / C3d: f32 [8, S, 4096] normal(0, 1) -> s8 (scale 0.05, zp 0) and
    the same int8 back to f32, S in {128, 1024, 8192} (S = 8192 is 1 GiB of
    f32)."""
    x = np.random.default_rng(0).standard_normal(8 * s * 4096, dtype=np.float32)
    sym = {"B": 8, "S": s}
    qblob, dblob = encode(recipe_c3("quantize")), encode(recipe_c3("dequantize"))
    out, _, _ = _typed_gpu(res, qblob, sym, {}, x)
    q = _ref_typed(ref_lib, pool, qblob, sym, {}, x)
    _same(out, q)
    del x, out
    out, _, _ = _typed_gpu(res, dblob, sym, {}, q.view(np.int8))
    _same(out, _ref_typed(ref_lib, pool, dblob, sym, {}, q.view(np.int8)))


def test_layer_digest_is_the_reference_digest(ref_lib, pool, res):
    """The bench's output check hashes assembled matrices (SHA-256 of each
    matrix's f16 bytes); the digest of the product's result equals the
    digest of the reference's for a full Llama-70B q projection."""
    out_f, in_f = LLAMA70B["q"]
    q, scale = _weights(out_f, in_f, seed=0)
    blob = encode(recipe_c4())
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    out, _, _ = _typed_gpu(res, blob, sym, params, q)
    assert hashlib.sha256(out.cpu().numpy().tobytes()).hexdigest() == \
        hashlib.sha256(_ref_typed(ref_lib, pool, blob, sym, params, q).tobytes()).hexdigest()
