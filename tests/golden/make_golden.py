#!/usr/bin/env python3
"""Regenerate the committed golden fixtures from the reference (run where the
reference checkout and the reference runtime build, oracle/_ref, exist).

Two sources, both written as small JSON fixtures beside this script:

* ``typed_corpus.json`` -- the reference's typed conformance corpus
  (``libreloc/test/corpus/typed/*.{bin,json}``): the wire v1 blob, the runtime
  parameters, and per binding the symbols, source bits and the reference's
  committed expected bits. Copied as data (hex), not as code.
* ``layout_corpus.json`` -- the reference's layout corpus
  (``libreloc/test/corpus/*.bin``); those fixtures carry no expected output, so
  for each plan a seeded source is relocated with the reference runtime
  (``executeH2DThreaded`` via oracle/_ref) and its sha256 recorded.
* ``config_cases.json`` -- small plans shaped like the benchmark configurations,
  encoded by this repository's plan encoder, executed by the reference runtime
  (decode + bindTyped + executeHost) on seeded inputs; sha256 of the output.

Usage: python tests/golden/make_golden.py [--reference PATH-TO-THE-REFERENCE-CHECKOUT]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import ref  # noqa: E402


def typed_corpus(corpus: Path):
    cases = []
    for meta_path in sorted((corpus / "typed").glob("*.json")):
        meta = json.loads(meta_path.read_text())
        blob = (corpus / "typed" / (meta_path.stem + ".bin")).read_bytes()
        params = {}
        for name, p in (meta.get("parameters") or {}).items():
            width = {"float32": 4, "int32": 4, "int8": 1, "float16": 2}[p["dtype"]]
            data = b"".join(int(b, 16).to_bytes(width, "little") for b in p["bits"])
            params[name] = {"dtype": p["dtype"], "shape": p["shape"], "hex": data.hex()}
        bindings = []
        for b in meta["bindings"]:
            bindings.append({
                "symbols": b["symbols"],
                "source": b["source"],
                "expected": b["expected"],
                "footprints": b.get("footprints"),
            })
        cases.append({"name": meta["name"], "blob": blob.hex(), "parameters": params,
                      "bindings": bindings, "stages": meta.get("stages"),
                      "recipe": meta.get("recipe")})
    return cases


def layout_corpus(corpus: Path):
    cases = []
    rng = np.random.default_rng(20260710)
    for meta_path in sorted(corpus.glob("*.json")):
        meta = json.loads(meta_path.read_text())
        blob = (corpus / (meta_path.stem + ".bin")).read_bytes()
        symbols = {}
        for name, spec in (meta.get("symbols") or {}).items():
            symbols[name] = spec.get("multiple_of", 1) * spec.get("max_factor", 1)
        plan = ref.LayoutPlan(blob, symbols)
        width = plan.info["element_size"]
        # Source span = the plan's valid source elements (dense source).
        n_src = 1
        for e in plan.info["extents"]:
            n_src *= e
        src = rng.integers(0, 256, size=n_src * width, dtype=np.uint8)
        out = plan.execute(src)
        cases.append({"name": meta["name"], "blob": blob.hex(), "symbols": symbols,
                      "element_size": width, "seed_hex_len": len(src),
                      "source_sha256": hashlib.sha256(src.tobytes()).hexdigest(),
                      "source_hex": src.tobytes().hex() if len(src) <= 65536 else None,
                      "expected_sha256": hashlib.sha256(out.tobytes()).hexdigest(),
                      "expected_bytes": int(out.size)})
    return cases


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference",
                        default=os.environ.get("SYM_REFERENCE_DIR", str(HERE.parent.parent.parent / "reference")),
                        help="the reference checkout ($SYM_REFERENCE_DIR, else a `reference` directory beside "
                             "the repository)")
    args = parser.parse_args()
    corpus = Path(args.reference) / "libreloc" / "test" / "corpus"
    (HERE / "typed_corpus.json").write_text(json.dumps(typed_corpus(corpus), indent=1) + "\n")
    (HERE / "layout_corpus.json").write_text(json.dumps(layout_corpus(corpus), indent=1) + "\n")
    print("wrote", HERE / "typed_corpus.json", HERE / "layout_corpus.json")


if __name__ == "__main__":
    main()
