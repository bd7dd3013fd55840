"""Build the native libraries in-tree (no JIT cache, so they travel with the repo).

* ``sym_b200/_lib/libsb_cuda.so``    -- the thin C-ABI CUDA layer and the
  sm_100a kernels (nvcc, ``-gencode arch=compute_100a,code=sm_100a``).
* ``sym_b200/_lib/libsb_runtime.so`` -- the C++ host runtime (decoder, binder,
  dispatch, typed contexts) exporting the drop-in C-ABI of ``include/sym_b200.h``;
  it links ``libsb_cuda.so`` and nothing from CUDA directly.

Usage: ``python -m sym_b200.build [--force]``. Rebuilds only when a source is
newer than its library.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB_DIR = PKG / "_lib"
CUDA_SOURCES = sorted((PKG / "csrc" / "cuda").glob("*.cu"))
RUNTIME_SOURCES = sorted((PKG / "csrc" / "runtime").glob("*.cpp"))
HEADERS = (sorted((ROOT / "include").rglob("*.h")) + sorted((PKG / "csrc").rglob("*.hpp"))
           + sorted((PKG / "csrc").rglob("*.h")))
CUDA_LIB = LIB_DIR / "libsb_cuda.so"
RUNTIME_LIB = LIB_DIR / "libsb_runtime.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cxx() -> str:
    # The system g++ links libstdc++ dynamically, sharing the C++ runtime of
    # the Python process (torch) that loads these libraries.
    for cand in ("/usr/bin/g++", shutil.which("g++")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("no g++ found")


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: Path, sources) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build(force: bool = False, verbose: bool = False) -> None:
    LIB_DIR.mkdir(exist_ok=True)
    inc = ["-I", ROOT / "include"]
    if force or _stale(CUDA_LIB, CUDA_SOURCES + HEADERS):
        # SYM_B200_NVCC_DEFINES: extra -D tuning definitions (e.g. "SBC_TMA_STAGES=8")
        defines = [f"-D{d}" for d in os.environ.get("SYM_B200_NVCC_DEFINES", "").split() if d]
        cmd = [_nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
               "-ccbin", _cxx(), *defines, *inc, *CUDA_SOURCES, "-o", CUDA_LIB]
        _run(cmd, verbose)
    if force or _stale(RUNTIME_LIB, RUNTIME_SOURCES + HEADERS + [CUDA_LIB]):
        cmd = [_cxx(), "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
               "-Wall", "-Wextra", "-Wno-unused-parameter", *inc, "-I", PKG / "csrc" / "runtime",
               "-I", PKG / "csrc" / "cuda",
               *RUNTIME_SOURCES, "-L", LIB_DIR, "-lsb_cuda", "-Wl,-rpath,$ORIGIN", "-pthread",
               "-o", RUNTIME_LIB]
        _run(cmd, verbose)


def main(argv=None):
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("-v", "--verbose", action="store_true")
    args = parser.parse_args(argv)
    build(force=args.force, verbose=args.verbose)
    print(f"built {CUDA_LIB.relative_to(ROOT)} and {RUNTIME_LIB.relative_to(ROOT)}")


if __name__ == "__main__":
    sys.exit(main())
