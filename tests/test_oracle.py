"""The checkers are pinned before they are trusted: the reference runtime build
(oracle/_ref) and the C restatement (oracle/typed_oracle.c) must reproduce the
reference's committed golden vectors and the normative witness table of
docs/reloc-typed-semantics.md §6."""
import hashlib
import struct

import numpy as np
import pytest

from helpers import bits_to_bytes, corpus_params, dtypes_of, layout_corpus, typed_corpus
from oracle import oracle

CASES = [(c, b) for c in typed_corpus() for b in c["bindings"]]
IDS = [f"{c['name']}-{i}" for i, (c, b) in enumerate(CASES)]


@pytest.mark.parametrize("case,binding", CASES, ids=IDS)
def test_reference_runtime_reproduces_golden(ref_lib, case, binding):
    prog = ref_lib.TypedProgram(bytes.fromhex(case["blob"]), binding["symbols"], corpus_params(case))
    src = np.frombuffer(bits_to_bytes(binding["source"]["bits"], binding["source"]["dtype"]), np.uint8)
    out = prog.execute(src)
    assert out.tobytes() == bits_to_bytes(binding["expected"]["bits"], binding["expected"]["dtype"])


@pytest.mark.parametrize("case,binding", CASES, ids=IDS)
def test_c_oracle_reproduces_golden(case, binding):
    """The C restatement, driven by this repository's binder description."""
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(bytes.fromhex(case["blob"])), binding["symbols"],
                               corpus_params(case))
    prog = oracle.Program.from_description(bound.describe(), dtypes_of(case["stages"]))
    src = np.frombuffer(bits_to_bytes(binding["source"]["bits"], binding["source"]["dtype"]), np.uint8)
    assert prog.execute(src).tobytes() == bits_to_bytes(binding["expected"]["bits"], binding["expected"]["dtype"])


@pytest.mark.parametrize("case", layout_corpus(), ids=[c["name"] for c in layout_corpus()])
def test_c_oracle_layout_corpus(case):
    """Layout-only plans: the C restatement against the reference runtime's output hash."""
    from sym_b200 import pyreloc

    if case["source_hex"] is None:
        pytest.skip("large fixture")
    bound = pyreloc.bind(pyreloc.load_plan(bytes.fromhex(case["blob"])), case["symbols"]).describe()
    desc = {"layout": bound, "result_extents": [e + sum(p["lo"] + p["hi"] for p in bound["pads"] if p["axis"] == k)
                                                for k, e in enumerate(bound["extents"])],
            "stages": [], "destination_bytes": bound["total_bytes"]}
    # result coordinates are never read without per-channel stages
    width = case["element_size"]
    dt = {1: "int8", 2: "float16", 4: "float32"}[width]
    prog = oracle.Program.from_description(desc, [dt])
    src = np.frombuffer(bytes.fromhex(case["source_hex"]), np.uint8)
    out = prog.execute(src)
    assert out.size == case["expected_bytes"]
    assert hashlib.sha256(out.tobytes()).hexdigest() == case["expected_sha256"]


def _f32bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def test_witness_vectors():
    """docs/reloc-typed-semantics.md §6, row by row."""
    L = oracle.lib()
    inv1 = L.orc_reciprocal(1.0)
    ties = [-2.5, -1.5, -0.5, 0.5, 1.5, 2.5]
    assert [L.orc_quantize(_f32bits(x), inv1) for x in ties] == [-2, -2, 0, 0, 2, 2]
    lim = [-129.0, -128.0, -127.0, 126.0, 127.0, 128.0]
    assert [L.orc_quantize(_f32bits(x), inv1) for x in lim] == [-128, -128, -127, 126, 127, 127]
    assert [L.orc_quantize(b, inv1) for b in (0x7FC00000, 0x7F800000, 0xFF800000)] == [-128, 127, -128]
    f16 = [(0.0, 0x0000), (-0.0, 0x8000), (2.0 ** -24, 0x0001), (2.0 ** -25, 0x0000), (1.5 * 2.0 ** -25, 0x0001),
           (2.0 ** -14, 0x0400), (65504.0, 0x7BFF), (65519.99, 0x7BFF), (65520.0, 0x7C00), (1e5, 0x7C00),
           (1 + 2.0 ** -11, 0x3C00), (1 + 3 * 2.0 ** -12, 0x3C01)]
    for x, want in f16:
        assert L.orc_narrow_f16(_f32bits(x)) == want, x
    assert [L.orc_widen_f16(h) for h in (0x0001, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x8000)] == \
        [0x33800000, 0x38800000, 0x477FE000, 0x7F800000, 0xFF800000, 0x80000000]
    bf = [(0.0, 0x0000), (-0.0, 0x8000), (1 + 2.0 ** -8, 0x3F80), (1 + 3 * 2.0 ** -9, 0x3F81),
          (2.0 ** -133, 0x0001), (2.0 ** -134, 0x0000), (1.5 * 2.0 ** -134, 0x0001), (2.0 ** -126, 0x0080),
          (3.3895314e38, 0x7F7F), (3.3961775e38, 0x7F80), (3.4e38, 0x7F80)]
    for x, want in bf:
        assert L.orc_narrow_bf16(_f32bits(x)) == want, x
    assert [L.orc_widen_bf16(b) for b in (0x0001, 0x0080, 0x7F7F, 0x7F80, 0xFF80, 0x8000)] == \
        [0x00010000, 0x00800000, 0x7F7F0000, 0x7F800000, 0xFF800000, 0x80000000]
    # reciprocal formation: x * fl32(1/0.3) differs from x / 0.3 in 3 of 8
    inv = L.orc_reciprocal(np.float32(0.3))
    xs = np.array([0.1, 0.3, 0.7, 1.1, 2.9, 10.1, 100.3, 1000.7], np.float32)
    a = xs * np.float32(inv)
    b = xs / np.float32(0.3)
    assert int(np.sum(a.view(np.uint32) != b.view(np.uint32))) == 3
    scale = np.float32(0.3)
    assert [L.orc_dequantize(q, 0, scale) for q in (-128, -1, 0, 1, 127)] == \
        [0xC219999A, 0xBE99999A, 0x00000000, 0x3E99999A, 0x42186667]
    assert L.orc_dequantize(-128, 127, scale) == 0xC2990000


def test_narrowing_random_bits_agree_with_numpy():
    """f32 -> f16 RNE over random non-NaN bit patterns vs numpy's IEEE conversion."""
    L = oracle.lib()
    rng = np.random.default_rng(7)
    bits = rng.integers(0, 2 ** 32, size=20000, dtype=np.uint64).astype(np.uint32)
    f = bits.view(np.float32)
    keep = ~np.isnan(f)
    want = f[keep].astype(np.float16).view(np.uint16)
    got = np.array([L.orc_narrow_f16(int(b)) for b in bits[keep]], dtype=np.uint16)
    assert np.array_equal(got, want)
