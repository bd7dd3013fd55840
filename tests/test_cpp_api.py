"""The C++ runtime API as a C++ caller sees it (tests/cpp/transfer_api_test.cpp):
compiled against include/reloc/*.h, linked to libsb_runtime.so, no C-ABI in
between. The reference boundary it checks: validateTransfer / executeTransfer
for layout plans (libreloc/include/reloc/Transfer.h:100-200), the CopyBackend
interface (Backend.h:34-89) and executeDispatch(DispatchRequest&,
CopyBackend&, const TransferOptions&) with backend_mismatch for a backend
that is not a CudaBackend (Dispatch.h:263-271).

The CPU half runs the validation and backend-mismatch checks; the GPU half
runs config 1 both ways through executeTransfer and config 4 through
executeDispatch, and compares the bytes with the reference executor."""
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from helpers import ROOT, encode, recipe_c1, recipe_c4

SOURCE = ROOT / "tests" / "cpp" / "transfer_api_test.cpp"
LIB = ROOT / "sym_b200" / "_lib"


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    if not (LIB / "libsb_runtime.so").exists():
        pytest.skip("native libraries not built")
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no g++")
    out = tmp_path_factory.mktemp("cpp") / "transfer_api_test"
    subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-I", str(ROOT / "include"), str(SOURCE), "-o", str(out),
                    "-L", str(LIB), "-lsb_runtime", "-lsb_cuda", f"-Wl,-rpath,{LIB}", "-pthread"], check=True,
                   capture_output=True, text=True)
    return out


def _blobs(tmp_path):
    c1, c4 = tmp_path / "c1.blob", tmp_path / "c4.blob"
    c1.write_bytes(encode(recipe_c1()))
    c4.write_bytes(encode(recipe_c4()))
    return c1, c4


def test_cpp_caller_validation_and_backend_checks(program, tmp_path):
    c1, c4 = _blobs(tmp_path)
    r = subprocess.run([str(program), "cpu", str(c1), str(c4)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("cpu ok"), r.stdout + r.stderr
    assert "FAIL" not in r.stdout


@pytest.mark.gpu
def test_cpp_caller_runs_configs_1_and_4_like_the_reference(program, tmp_path, ref_lib):
    c1, c4 = _blobs(tmp_path)
    n = 1 << 22
    x = np.random.default_rng(0).uniform(-1.0, 1.0, n).astype(np.float32)
    (tmp_path / "c1.src").write_bytes(x.tobytes())
    out_f, in_f = 11008, 4096
    rng = np.random.default_rng(1)
    q = rng.integers(-127, 128, size=(out_f, in_f), dtype=np.int8)
    scale = np.exp(rng.normal(-5.0, 0.5, out_f)).astype(np.float32)
    (tmp_path / "c4.src").write_bytes(q.tobytes())
    (tmp_path / "c4.scale").write_bytes(scale.tobytes())
    args = [str(program), "gpu", str(c1), str(n), str(tmp_path / "c1.src"), str(tmp_path / "c1.h2d"),
            str(tmp_path / "c1.d2h"), str(c4), str(out_f), str(in_f), str(tmp_path / "c4.src"),
            str(tmp_path / "c4.scale"), str(tmp_path / "c4.out")]
    r = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("gpu ok"), r.stdout + r.stderr
    threads = len(os.sched_getaffinity(0))
    want1 = ref_lib.LayoutPlan(encode(recipe_c1()), {"N": n}).execute(x.view(np.uint8), threads=threads)
    assert np.array_equal(np.frombuffer((tmp_path / "c1.h2d").read_bytes(), np.uint8), want1)
    assert np.array_equal(np.frombuffer((tmp_path / "c1.d2h").read_bytes(), np.uint8), want1)
    want4 = ref_lib.TypedProgram(encode(recipe_c4()), {"out_features": out_f, "in_features": in_f},
                                 {"scale": ("float32", [out_f], scale.tobytes())}).execute(q.view(np.uint8).reshape(-1))
    assert np.array_equal(np.frombuffer((tmp_path / "c4.out").read_bytes(), np.uint8), want4)
