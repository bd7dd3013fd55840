"""The in-process plan encoder (replacement for the MLIR exporter) produces
plans the reference decoder and binder accept and the reference executor runs
to the reference's committed golden bits, and for every reference corpus
recipe it reproduces the exporter's committed blob byte for byte (the
exporter's canonical form: merged adjacent axes, positional axis names,
simplified expressions)."""
import numpy as np
import pytest

from helpers import bits_to_bytes, corpus_params, encode, recipe_c1, recipe_c2, recipe_c3, recipe_c4, typed_corpus

CASES = typed_corpus()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_corpus_recipes_execute_to_the_golden_bits(ref_lib, case):
    from sym_b200.reloc_torch import recipe as R

    blob = encode(R.from_json(case["recipe"]))
    assert blob.hex() == case["blob"]
    for b in case["bindings"]:
        prog = ref_lib.TypedProgram(blob, b["symbols"], corpus_params(case))
        src = np.frombuffer(bits_to_bytes(b["source"]["bits"], b["source"]["dtype"]), np.uint8)
        assert prog.execute(src).tobytes() == bits_to_bytes(b["expected"]["bits"], b["expected"]["dtype"])


def test_config_plans_are_accepted_by_the_reference(ref_lib):
    assert ref_lib.wire_version(encode(recipe_c1())) == 0
    assert ref_lib.decode_error(encode(recipe_c1()), False) is None
    for r in (recipe_c2(), recipe_c3("quantize"), recipe_c3("dequantize"), recipe_c4(), recipe_c4("float32"),
              recipe_c4("bfloat16")):
        blob = encode(r)
        assert ref_lib.wire_version(blob) == 1
        assert ref_lib.decode_error(blob, True) is None


def test_unsupported_recipes_are_rejected():
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S
    from sym_b200.reloc_torch.compiler import UnsupportedRecipe, encode as enc

    shape = (S.Const(4), S.Const(6))
    src = R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), "float32")
    scale = R.BindingParam("s", "float32", (S.Const(4),))
    # pad on the per-channel axis before its quantize
    bad = R.Recipe(src, (R.Quantize("int8", scale, None, 0, "symmetric_rne"),
                         R.Pad(0, S.Const(1), S.Const(0), R.Fill("int8", 0))), src, "h2d")
    with pytest.raises(UnsupportedRecipe):
        enc(bad)
    # reshape across a per-channel axis
    bad = R.Recipe(src, (R.Quantize("int8", scale, None, 0, "symmetric_rne"), R.Reshape((S.Const(24),))), src, "h2d")
    with pytest.raises(UnsupportedRecipe):
        enc(bad)
    # a fill through a runtime-parameter stage cannot fold
    bad = R.Recipe(src, (R.Pad(1, S.Const(1), S.Const(0), R.Fill("float32", 0)),
                         R.Quantize("int8", R.BindingParam("t", "float32", ()), None, None, "symmetric_rne")),
                   src, "h2d")
    with pytest.raises(UnsupportedRecipe):
        enc(bad)


def test_divisibility_guard_is_emitted():
    from sym_b200 import pyreloc

    plan = pyreloc.load_plan(encode(recipe_c1()))
    with pytest.raises(pyreloc.BindError, match="divisibility violated"):
        pyreloc.bind(plan, {"N": 100})
    assert pyreloc.bind(plan, {"N": 128}).extents == [64, 2]
