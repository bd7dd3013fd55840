"""The drop-in boundary loads on a CPU-only host and exports every function the
public headers declare (include/sym_b200.h from libsb_runtime.so,
include/sb_cuda.h from libsb_cuda.so); plan-level calls (decode, bind,
capability, templates) work without a GPU, and execution fails loudly rather
than falling back."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared(header):
    text = (ROOT / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:sb|sbc)_[a-z0-9_]+)\s*\(", text)))


@pytest.mark.parametrize("header,lib", [("sym_b200.h", "libsb_runtime.so"), ("sb_cuda.h", "libsb_cuda.so")])
def test_every_declared_function_is_exported(header, lib):
    names = _declared(header)
    assert len(names) > 10
    so = ctypes.CDLL(str(ROOT / "sym_b200" / "_lib" / lib))
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing


def test_version_and_wire_version():
    from sym_b200 import pyreloc

    assert "sm_100a" in pyreloc.version()
    assert pyreloc.wire_version(b"RPLN\x01\x00\x00\x00") == 1
    assert pyreloc.wire_version(b"XXXX\x01\x00\x00\x00") is None
    assert pyreloc.wire_version(b"RPL") is None


def test_decode_errors_carry_offsets():
    from sym_b200 import pyreloc

    with pytest.raises(pyreloc.DecodeError) as e:
        pyreloc.load_typed_plan(b"RPLN\x00\x00\x00\x00")
    assert e.value.offset == 4 and "unsupported wire format version" in str(e.value)
    with pytest.raises(pyreloc.DecodeError) as e:
        pyreloc.load_plan(b"NOPE")
    assert e.value.offset == 0


def test_execution_without_a_gpu_fails_loudly():
    """No CPU fallback exists: on a host without a usable GPU the execute
    call reports a backend failure instead of producing data elsewhere."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import numpy as np

    from helpers import encode, recipe_c3
    from sym_b200 import pyreloc

    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(encode(recipe_c3("quantize"))), {"B": 1, "S": 1}, {})
    tmpl = pyreloc.prepare_dispatch_template(bound)
    src = np.zeros(4096, np.float32)
    dst = np.zeros(4096, np.int8)
    sv = pyreloc.BufferView(src.ctypes.data, src.nbytes, 0, [1, 1, 4096], [4096, 4096, 1], 4, "host", -1)
    dv = pyreloc.BufferView(dst.ctypes.data, dst.nbytes, 0, [1, 1, 4096], [4096, 4096, 1], 1, "cuda", 0)
    req = pyreloc.prepare_dispatch_from_template(tmpl, sv, dv)
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.execute_dispatch(req)
    assert e.value.code == "backend_failure"
    assert not dst.any()


def test_missing_native_library_is_an_import_error(monkeypatch, tmp_path):
    from sym_b200 import _native

    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "RUNTIME_LIB", tmp_path / "absent.so")
    with pytest.raises(_native.NativeLibraryMissing):
        _native.lib()
