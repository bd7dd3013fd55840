"""Decoder and binder parity with the reference (CPU).

The product decoder/binder (sym_b200 C++ runtime, via its C-ABI) must produce
the reference's bound layouts, footprints and checked stage arithmetic for
every corpus plan and every benchmark-configuration plan, and the reference's
exact diagnostics (byte offset + message) for hostile blobs."""
import json

import numpy as np
import pytest

from helpers import corpus_params, encode, layout_corpus, recipe_c1, recipe_c2, recipe_c3, recipe_c4, typed_corpus

LAYOUT_KEYS = ["extents", "src_strides", "dst_strides", "element_size", "total_bytes", "L", "pads"]
STAGE_KEYS = ["per_channel", "channel_is_dim", "channel_dim", "channel_length", "scale_bits", "inv_scale_bits",
              "zero_point"]
LLAMA7B = [(4096, 4096), (11008, 4096), (4096, 11008)]
LLAMA70B = [(8192, 8192), (1024, 8192), (28672, 8192), (8192, 28672)]


def _compare_typed(ref_lib, blob, symbols, params):
    from sym_b200 import pyreloc

    mine = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), symbols, params).describe()
    theirs = ref_lib.TypedProgram(blob, symbols, params).info
    for k in ["source_extents", "result_extents", "source_bytes", "destination_bytes", "parameter_bytes"]:
        assert mine[k] == theirs[k], k
    for k in LAYOUT_KEYS:
        assert mine["layout"][k] == theirs["layout"][k], k
    assert [(c["boundary"], c["elements"], c["bytes"]) for c in mine["cuts"]] == \
        [(c["boundary"], c["elements"], c["bytes"]) for c in theirs["cuts"]]
    for a, b in zip(mine["stages"], theirs["stages"]):
        for k in STAGE_KEYS:
            assert a[k] == b[k], k


@pytest.mark.parametrize("case", typed_corpus(), ids=[c["name"] for c in typed_corpus()])
def test_typed_corpus_bind_parity(ref_lib, case):
    for b in case["bindings"]:
        _compare_typed(ref_lib, bytes.fromhex(case["blob"]), b["symbols"], corpus_params(case))


@pytest.mark.parametrize("case", layout_corpus(), ids=[c["name"] for c in layout_corpus()])
def test_layout_corpus_bind_parity(ref_lib, case):
    from sym_b200 import pyreloc

    blob = bytes.fromhex(case["blob"])
    mine = pyreloc.bind(pyreloc.load_plan(blob), case["symbols"]).describe()
    theirs = ref_lib.LayoutPlan(blob, case["symbols"]).info
    for k in LAYOUT_KEYS:
        assert mine[k] == theirs[k], k


def test_config_plans_bind_parity(ref_lib):
    from sym_b200 import pyreloc

    c1 = encode(recipe_c1())
    for n in (1 << 20, 1 << 22, 1 << 24):
        mine = pyreloc.bind(pyreloc.load_plan(c1), {"N": n}).describe()
        theirs = ref_lib.LayoutPlan(c1, {"N": n}).info
        for k in LAYOUT_KEYS:
            assert mine[k] == theirs[k]
        assert mine["extents"] == [64, n // 64] and mine["src_strides"] == [1, 64]
    _compare_typed(ref_lib, encode(recipe_c2()), {}, {})
    for s in (128, 1024, 8192):
        _compare_typed(ref_lib, encode(recipe_c3("quantize")), {"B": 8, "S": s}, {})
        _compare_typed(ref_lib, encode(recipe_c3("dequantize")), {"B": 8, "S": s}, {})
    blob = encode(recipe_c4())
    for out_f, in_f in LLAMA7B + LLAMA70B:
        scale = np.exp(np.random.default_rng(out_f).normal(-5, 0.5, out_f)).astype(np.float32)
        _compare_typed(ref_lib, blob, {"out_features": out_f, "in_features": in_f},
                       {"scale": ("float32", [out_f], scale.tobytes())})


def test_c2_bound_layout_is_the_survey_layout():
    """C2 binds to extents [64, 50176, 3] with the channel pad 3 -> 4 and fill 0x0000."""
    from sym_b200 import pyreloc

    b = pyreloc.bind_typed(pyreloc.load_typed_plan(encode(recipe_c2())), {}, {}).describe()
    assert b["layout"]["extents"] == [64, 50176, 3]
    assert b["layout"]["src_strides"] == [150528, 1, 50176]
    assert b["layout"]["dst_strides"] == [200704, 4, 1]
    assert b["layout"]["pads"] == [{"axis": 2, "lo": 0, "hi": 1, "fill": 0}]
    assert b["stages"][0]["inv_scale_bits"] == []


def _mutations(blob, rng, count):
    yield from (blob[:n] for n in range(0, len(blob), max(1, len(blob) // 40)))
    for _ in range(count):
        b = bytearray(blob)
        for _ in range(int(rng.integers(1, 4))):
            i = int(rng.integers(0, len(b)))
            b[i] = int(rng.integers(0, 256))
        yield bytes(b)
    yield blob + b"\x00"


@pytest.mark.parametrize("typed", [True, False])
def test_decode_error_parity_on_hostile_blobs(ref_lib, typed):
    """Truncations and random byte mutations: same accept/reject decision,
    same byte offset, same message as the reference decoder."""
    from sym_b200 import pyreloc

    rng = np.random.default_rng(20260710)
    blobs = [bytes.fromhex(c["blob"]) for c in (typed_corpus() if typed else layout_corpus())]
    blobs.append(encode(recipe_c4()) if typed else encode(recipe_c1()))
    load = pyreloc.load_typed_plan if typed else pyreloc.load_plan
    checked = 0
    for blob in blobs:
        for m in _mutations(blob, rng, 60):
            theirs = ref_lib.decode_error(m, typed)
            try:
                load(m)
                mine = None
            except pyreloc.DecodeError as e:
                mine = (e.offset, str(e).split(": ", 1)[1])
            assert mine == theirs, (m.hex(), mine, theirs)
            checked += 1
    assert checked > 500


def test_bind_error_parity(ref_lib):
    """Rejected bindings carry the reference's message."""
    from oracle.ref import RefError
    from sym_b200 import pyreloc

    blob = encode(recipe_c4())
    plan = pyreloc.load_typed_plan(blob)
    good = {"scale": ("float32", [4], np.ones(4, np.float32).tobytes())}
    sym = {"out_features": 4, "in_features": 8}
    bad_cases = [
        ({"out_features": 4}, good),
        ({**sym, "extra": 1}, good),
        (sym, {}),
        (sym, {"scale": ("float32", [3], np.ones(3, np.float32).tobytes())}),
        (sym, {"scale": ("float32", [4], np.array([1, 0, 1, 1], np.float32).tobytes())}),
        (sym, {"scale": ("float32", [4], np.array([1, np.nan, 1, 1], np.float32).tobytes())}),
        (sym, {"scale": ("float32", [4], np.array([1, -2, 1, 1], np.float32).tobytes())}),
        (sym, {"scale": ("int32", [4], np.ones(4, np.int32).tobytes())}),
        (sym, {"scale": ("float32", [], np.ones(1, np.float32).tobytes())}),
        (sym, {**good, "zp": ("int32", [], b"\0\0\0\0")}),
        ({"out_features": 0, "in_features": 8}, good),
    ]
    for symbols, params in bad_cases:
        with pytest.raises(RefError) as theirs:
            ref_lib.TypedProgram(blob, symbols, params)
        with pytest.raises(pyreloc.BindError) as mine:
            pyreloc.bind_typed(plan, symbols, params)
        assert str(theirs.value) == "bind: " + str(mine.value), (symbols, list(params))
    c1 = encode(recipe_c1())
    with pytest.raises(RefError) as theirs:
        ref_lib.LayoutPlan(c1, {"N": 100})
    with pytest.raises(pyreloc.BindError) as mine:
        pyreloc.bind(pyreloc.load_plan(c1), {"N": 100})
    assert str(theirs.value) == "bind: " + str(mine.value)


def test_capability_table():
    """Every supported plan is eligible for the B200 rows; CPU rows excluded."""
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(encode(recipe_c3("quantize"))), {"B": 1, "S": 2}, {})
    cap = pyreloc.query_capability(bound, "h2d", "cuda")
    assert [r["implementation"] for r in cap["eligible"]] == \
        ["b200_fused_h2d", "b200_fused_h2d@dma_ring", "b200_fused_h2d@zero_copy"]
    excluded = {r["implementation"] for r in cap["excluded"]}
    assert {"cpu_reference", "cpu_stages_cuda_stages@0", "cpu_stages_cuda_stages@1"} <= excluded
    d2h = pyreloc.query_capability(bound, "d2h", "cuda")
    assert [r["implementation"] for r in d2h["eligible"]] == \
        ["b200_fused_d2h", "b200_fused_d2h@dma_ring", "b200_fused_d2h@zero_copy"]
    # the finished result crosses the link device -> host
    assert d2h["eligible"][0]["wire_boundary"] == 1 and d2h["eligible"][0]["wire_bytes"] == 2 * 4096
    assert "b200_fused_h2d" in {r["implementation"] for r in d2h["excluded"]}
    assert pyreloc.query_capability(bound, "d2h", "host")["eligible"] == []
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.prepare_dispatch_template(bound, policy="original_cpu")
    assert e.value.code == "implementation_unavailable"
    tmpl = pyreloc.prepare_dispatch_template(bound, implementation="b200_fused_h2d@zero_copy")
    assert tmpl.selection["implementation"] == "b200_fused_h2d@zero_copy"


def test_view_validation_errors():
    """Views that do not match the bound plan are rejected before any launch."""
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(encode(recipe_c3("quantize"))), {"B": 1, "S": 2}, {})
    tmpl = pyreloc.prepare_dispatch_template(bound)
    src = pyreloc.BufferView(0x1000, 4 * 8192, 0, [1, 2, 4096], [8192, 4096, 1], 4, "host", -1)
    dst = pyreloc.BufferView(0x2000, 8192, 0, [1, 2, 4096], [8192, 4096, 1], 1, "cuda", 0)
    cases = [
        (pyreloc.BufferView(0x1000, 4 * 8192, 0, [1, 2, 4096], [8192, 4096, 1], 2, "host", -1), dst,
         "plan_mismatch"),
        (pyreloc.BufferView(0x1000, 100, 0, [1, 2, 4096], [8192, 4096, 1], 4, "host", -1), dst,
         "insufficient_capacity"),
        (pyreloc.BufferView(0x1000, 4 * 8192, 0, [1, 2, 4096], [8192, 1, 2], 4, "host", -1), dst,
         "unsupported_layout"),
        (src, pyreloc.BufferView(0x2000, 8192, 0, [1, 2, 4096], [8192, 4096, 1], 1, "host", -1),
         "direction_mismatch"),
        (src, pyreloc.BufferView(0x2000, 8192, 0, [2, 1, 4096], [4096, 4096, 1], 1, "cuda", 0), "plan_mismatch"),
    ]
    for s, d, code in cases:
        with pytest.raises(pyreloc.TransferError) as e:
            pyreloc.prepare_dispatch_from_template(tmpl, s, d)
        assert e.value.code == code
    req = pyreloc.prepare_dispatch_from_template(tmpl, src, dst)
    assert req.report["implementation"] == "b200_fused_h2d"
