"""Bit-pattern coverage of every kernel family's value conversions against the
reference executor (reference CudaKernelsTest.cpp: NarrowingRneWitnessesAndRandomBits,
ExactWideningWitnessBits, CudaConvertBF16.NarrowingAndWideningMatchTheHostBits).

Each family has its own conversion code (packed f32x2 -> f16x2 narrowing in
the runs, narrow and tile kernels, scalar narrowing in the others), so each
sees the same inputs: uniformly random 32-bit patterns (NaNs with every
payload and sign, infinities, subnormals, huge values), the f16 and bf16
rounding boundaries, and for widening every one of the 65,536 16-bit
patterns."""
import numpy as np
import pytest

from helpers import encode, run_typed_gpu
from test_gpu_parity import _channels_last, _runs_recipe, _transpose_2d, expected

pytestmark = pytest.mark.gpu

# f32 patterns at the f16 / bf16 rounding boundaries: largest finite, the
# overflow tie, min normal and subnormal, half of the min subnormal (a tie to
# zero), ties to even above 1.0, NaNs with payloads in the kept and the
# dropped mantissa bits.
_WITNESSES = np.array([
    0x477FEFFF, 0x477FF000, 0x477FF001, 0x477FE000, 0x38800000, 0x387FC000, 0x33800000, 0x33000000, 0x33000001,
    0x3F801000, 0x3F803000, 0x3F800FFF, 0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00000, 0x7F800001, 0x7FA00000,
    0xFF801234, 0x7F802000, 0x00000001, 0x80000001, 0x007FFFFF, 0x3F808000, 0x3F818000, 0x3F7FFFFF, 0x7F7FFFFF,
    0xFF7FFFFF, 0x00000000, 0x80000000,
], dtype=np.uint32)


def _f32_bits(n, seed):
    rng = np.random.default_rng(seed)
    x = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    k = _WITNESSES.size
    x[:k] = _WITNESSES
    x[k:2 * k] = _WITNESSES[::-1]  # each witness in both halves of a packed pair
    x[-k:] = _WITNESSES
    return x.view(np.float32)


def _cast_1d(n, op):
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    src_dtype = {"f16": "float32", "bf16": "float32", "widen": "float16", "widen_bf16": "bfloat16"}[op]
    dst_dtype = {"f16": "float16", "bf16": "bfloat16", "widen": "float32", "widen_bf16": "float32"}[op]
    policy = "ieee_rne" if op in ("f16", "bf16") else "exact"
    shape = (S.Const(n),)
    return R.Recipe(R.TensorSpec(shape, (S.Const(1),), S.Const(0), src_dtype), (R.Cast(dst_dtype, policy),),
                    R.TensorSpec(shape, (S.Const(1),), S.Const(0), dst_dtype), "h2d")


@pytest.mark.parametrize("op", ["f16", "bf16"])
@pytest.mark.parametrize("family", ["contiguous", "transpose", "narrow", "runs", "generic"])
def test_narrowing_bits_in_every_family(family, op):
    if family == "contiguous":
        n = (1 << 20) + 12
        recipe, shape = _cast_1d(n, op), (n,)
    elif family == "transpose":  # TMA tiles of 32-bit cells
        recipe, shape = _transpose_2d(1024, 1024, op), (1024, 1024)
    elif family == "narrow":  # three channels padded to four
        recipe, shape = _channels_last(4, 3, 4096, 1, op), (4, 3, 4096, 1)
    elif family == "runs":  # whole rows of 256 cells, warp spans
        recipe, shape = _runs_recipe((16, 32, 512), (1, 0, 2), op), (16, 32, 512)
    else:  # rows of 30 cells: not a whole number of vectors
        recipe, shape = _runs_recipe((8, 32, 30), (1, 0, 2), op), (8, 32, 30)
    blob = encode(recipe)
    x = _f32_bits(int(np.prod(shape)), seed=21)
    out, rep = run_typed_gpu(blob, {}, {}, x)
    assert out.tobytes() == expected(blob, {}, {}, x).tobytes()
    if family != "generic":  # k_narrow is a member of the transpose family
        assert rep["device_kernel"] == {"narrow": "transpose"}.get(family, family)


@pytest.mark.parametrize("op", ["widen", "widen_bf16"])
@pytest.mark.parametrize("family", ["contiguous", "runs"])
def test_every_16_bit_pattern_widens_like_the_reference(family, op):
    patterns = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    if family == "contiguous":
        blob = encode(_cast_1d(patterns.size, op))
    else:
        from sym_b200.reloc_torch import recipe as R
        from sym_b200.reloc_torch import symbolic as S

        src_dtype = "float16" if op == "widen" else "bfloat16"
        shape = (S.Const(16), S.Const(16), S.Const(256))
        out = (S.Const(16), S.Const(16), S.Const(256))
        blob = encode(R.Recipe(R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), src_dtype),
                               (R.Transpose((1, 0, 2)), R.Cast("float32", "exact")),
                               R.TensorSpec(out, S.dense_strides(out), S.Const(0), "float32"), "h2d"))
    got, rep = run_typed_gpu(blob, {}, {}, patterns)
    assert got.tobytes() == expected(blob, {}, {}, patterns).tobytes()
    assert rep["device_kernel"] == family


def _quantize_2d(rows, cols):
    """f32 [rows, cols] -> transpose -> s8 with scale 0.05 (the SIMT tile family)."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    shape = (S.Const(rows), S.Const(cols))
    out = (S.Const(cols), S.Const(rows))
    q = R.Quantize("int8", R.InlineParam("float32", (), (0x3D4CCCCD,)), None, None, "symmetric_rne")
    return R.Recipe(R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), "float32"), (R.Transpose((1, 0)), q),
                    R.TensorSpec(out, S.dense_strides(out), S.Const(0), "int8"), "h2d")


@pytest.mark.parametrize("family", ["contiguous", "tile", "narrow", "runs", "generic"])
def test_quantize_bits_in_every_family(family):
    """Symmetric RNE quantize (scale 0.05: multiply by the host-formed
    reciprocal 20.0f, clamp, round half to even; NaN -> -128) of random 32-bit
    patterns and the boundaries (ties at +-2.5 / 20, the clamp limits,
    infinities, NaNs) in each family."""
    from helpers import recipe_c3

    if family == "contiguous":
        recipe, shape, symbols = recipe_c3("quantize"), (2, 129, 4096), {"B": 2, "S": 129}
    elif family == "tile":
        recipe, shape, symbols = _quantize_2d(512, 768), (512, 768), {}
    elif family == "narrow":
        recipe, shape, symbols = _channels_last(4, 3, 4096, 1, "quantize"), (4, 3, 4096, 1), {}
    elif family == "runs":
        recipe, shape, symbols = _runs_recipe((16, 32, 512), (1, 0, 2), "quantize"), (16, 32, 512), {}
    else:
        recipe, shape, symbols = _runs_recipe((8, 32, 30), (1, 0, 2), "quantize"), (8, 32, 30), {}
    blob = encode(recipe)
    n = int(np.prod(shape))
    x = _f32_bits(n, seed=22)
    edges = (np.array([-2.5, -1.5, -0.5, 0.5, 1.5, 2.5, -6.4, 6.4, 6.35, 6.45, -6.45, 6.425, -6.425],
                      np.float32) / np.float32(20.0))
    edges = np.concatenate([edges, np.array([127.0, 128.0, -128.0, -129.0, 6.4, -6.4], np.float32),
                            np.array([0x7FC00000, 0xFFC00001, 0x7F800000, 0xFF800000], np.uint32).view(np.float32)])
    x[100:100 + edges.size] = edges
    x[1000:1000 + edges.size] = edges[::-1]
    # half of the elements in a human range, where rounding decides the result
    rng = np.random.default_rng(23)
    x[n // 2:] = (rng.standard_normal(n - n // 2) * 3.0).astype(np.float32)
    out, rep = run_typed_gpu(blob, symbols, {}, x)
    assert out.tobytes() == expected(blob, symbols, {}, x).tobytes()
