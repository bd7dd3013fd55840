"""Shared helpers for the parity tests: fixtures, config-shaped recipes, and
running a plan through the product (C-ABI via sym_b200.pyreloc) on the GPU."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
WIDTH = {"float32": 4, "int8": 1, "float16": 2, "bfloat16": 2, "uint16": 2, "uint8": 1, "uint32": 4}


def typed_corpus():
    return json.loads((GOLDEN / "typed_corpus.json").read_text())


def layout_corpus():
    return json.loads((GOLDEN / "layout_corpus.json").read_text())


def bits_to_bytes(bits, dtype):
    w = WIDTH[dtype]
    return b"".join(int(x, 16).to_bytes(w, "little") for x in bits)


def corpus_params(case):
    return {k: (v["dtype"], v["shape"], bytes.fromhex(v["hex"])) for k, v in case["parameters"].items()}


def dtypes_of(stages_or_desc):
    """Boundary dtypes: source, then each stage's output."""
    st = stages_or_desc
    return [st[0]["input_dtype"]] + [s["output_dtype"] for s in st]


# ---- config-shaped recipes (the benchmark configurations, parameterized sizes) ----

def recipe_c1():
    """C1: f32 [N] -> reshape [N floordiv 64, 64] -> transpose -> [64, N floordiv 64] (wire v0)."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    n = S.Symbol("N")
    src = R.TensorSpec((n,), (S.Const(1),), S.Const(0), "float32")
    q = S.FloorDiv(n, 64)
    dst = R.TensorSpec((S.Const(64), q), S.dense_strides((S.Const(64), q)), S.Const(0), "float32")
    return R.Recipe(src, (R.Reshape((q, S.Const(64))), R.Transpose((1, 0))), dst, "h2d")


def recipe_c2(batch=64, channels=3, h=224, w=224):
    """C2: f32 NCHW -> NHWC -> pad C to C+1 with 0.0 -> f16 (wire v1)."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    shape = tuple(S.Const(x) for x in (batch, channels, h, w))
    src = R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), "float32")
    out = tuple(S.Const(x) for x in (batch, h, w, channels + 1))
    dst = R.TensorSpec(out, S.dense_strides(out), S.Const(0), "float16")
    ops = (R.Transpose((0, 2, 3, 1)), R.Pad(3, S.Const(0), S.Const(1), R.Fill("float32", 0)),
           R.Cast("float16", "ieee_rne"))
    return R.Recipe(src, ops, dst, "h2d")


def recipe_c3(direction="quantize", scale_bits=0x3D4CCCCD, hidden=4096):
    """C3q / C3d: f32 [B, S, H] <-> s8 with a per-tensor inline scale (zp 0);
    B and S symbolic."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    shape = (S.Symbol("B"), S.Symbol("S"), S.Const(hidden))
    scale = R.InlineParam("float32", (), (scale_bits,))
    if direction == "quantize":
        src = R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), "float32")
        dst = R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), "int8")
        ops = (R.Quantize("int8", scale, None, None, "symmetric_rne"),)
    else:
        src = R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), "int8")
        dst = R.TensorSpec(shape, S.dense_strides(shape), S.Const(0), "float32")
        ops = (R.Dequantize("float32", scale, None, None, "affine"),)
    return R.Recipe(src, ops, dst, "h2d")


def recipe_tc(shape=(128, 128, 1024)):
    """The reference typed-H2D latency table's transpose + cast: f32
    [A, B, C] -> swap axes 0/1 -> f16 [B, A, C] (rows of C move intact)."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    a, b, c = (S.Const(x) for x in shape)
    src = R.TensorSpec((a, b, c), S.dense_strides((a, b, c)), S.Const(0), "float32")
    dst = R.TensorSpec((b, a, c), S.dense_strides((b, a, c)), S.Const(0), "float16")
    return R.Recipe(src, (R.Transpose((1, 0, 2)), R.Cast("float16", "ieee_rne")), dst, "h2d")


def recipe_c4(out_dtype="float16"):
    """C4/C5: int8 [out, in] + per-row f32 scale -> dequantize (axis 0) ->
    cast f16 -> transpose -> f16 [in, out]; out/in symbolic, scale a binding."""
    from sym_b200.reloc_torch import recipe as R
    from sym_b200.reloc_torch import symbolic as S

    o, i = S.Symbol("out_features"), S.Symbol("in_features")
    src = R.TensorSpec((o, i), S.dense_strides((o, i)), S.Const(0), "int8")
    dst = R.TensorSpec((i, o), S.dense_strides((i, o)), S.Const(0), out_dtype)
    ops = [R.Dequantize("float32", R.BindingParam("scale", "float32", (o,)), None, 0, "affine")]
    if out_dtype != "float32":
        ops.append(R.Cast(out_dtype, "ieee_rne"))
    ops.append(R.Transpose((1, 0)))
    return R.Recipe(src, tuple(ops), dst, "h2d")


def encode(recipe):
    from sym_b200.reloc_torch.compiler import encode as enc

    return enc(recipe)


# ---- running the product on the GPU --------------------------------------------

_RES = None


def resources():
    global _RES
    from sym_b200 import pyreloc

    if _RES is None:
        _RES = pyreloc.DispatchResources()
    return _RES


def dense(extents):
    strides, run = [], 1
    for e in reversed(extents):
        strides.append(run)
        run *= e
    return list(reversed(strides))


def run_typed_gpu(blob, symbols, params, src: np.ndarray, route="auto", device=0, pinned=True, chunk_size=0,
                  n_buffers=4, implementation=""):
    """Execute a typed plan host->device through the C-ABI; returns (bytes, report)."""
    import torch
    from sym_b200 import pyreloc

    plan = pyreloc.load_typed_plan(blob)
    bound = pyreloc.bind_typed(plan, symbols, params)
    tmpl = pyreloc.prepare_dispatch_template(bound, "h2d", "cuda", implementation=implementation)
    info = bound.describe()
    host = torch.from_numpy(np.ascontiguousarray(src).view(np.uint8).reshape(-1).copy())
    if pinned:
        host = host.pin_memory()
    out = torch.empty(max(1, bound.destination_bytes), dtype=torch.uint8, device=f"cuda:{device}")
    sw = WIDTH[info["source_dtype"]]
    dw = WIDTH[info["result_dtype"]]
    sv = pyreloc.BufferView(host.data_ptr(), host.numel(), 0, info["source_extents"],
                            dense(info["source_extents"]), sw, "host", -1)
    dv = pyreloc.BufferView(out.data_ptr(), out.numel(), 0, info["result_extents"],
                            dense(info["result_extents"]), dw, "cuda", device)
    req = pyreloc.prepare_dispatch_from_template(tmpl, sv, dv)
    rep = pyreloc.execute_dispatch(req, resources=resources(), route=route, chunk_size=chunk_size,
                                   n_buffers=n_buffers)
    return out.cpu().numpy()[: bound.destination_bytes], dict(rep)
