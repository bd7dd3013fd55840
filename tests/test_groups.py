"""Transfer groups on the host side: the native group validator
(pyreloc.prepare_dispatch_group over sb_prepare_dispatch_group, reference
dispatch::prepareDispatchGroup, Dispatch.h:213) and the Torch group bridge
(reloc_torch.group, reference group.py:41-70) reject what the reference
rejects before anything is allocated or launched. Buffers here are fake
addresses: nothing executes."""
import numpy as np
import pytest

from helpers import dense, encode, recipe_c3, recipe_c4


def _template(out_f=64, in_f=128):
    from sym_b200 import pyreloc

    scale = np.ones(out_f, np.float32)
    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(encode(recipe_c4())),
                               {"out_features": out_f, "in_features": in_f},
                               {"scale": ("float32", [out_f], scale.tobytes())})
    return pyreloc.prepare_dispatch_template(bound), out_f, in_f


def _views(src_base, dst_base, out_f, in_f, device=0):
    from sym_b200 import pyreloc

    sv = pyreloc.BufferView(src_base, out_f * in_f, 0, [out_f, in_f], dense([out_f, in_f]), 1, "host", -1)
    dv = pyreloc.BufferView(dst_base, out_f * in_f * 2, 0, [in_f, out_f], dense([in_f, out_f]), 2, "cuda", device)
    return sv, dv


def test_valid_group_prepares_without_a_gpu():
    from sym_b200 import pyreloc

    t, o, i = _template()
    entries = []
    for k in range(3):
        sv, dv = _views(0x10000000 + k * 0x100000, 0x7f0000000000 + k * 0x100000, o, i)
        entries.append((t, sv, dv, "h2d"))
    g = pyreloc.prepare_dispatch_group(entries)
    rep = g.report
    assert rep["logical_transfers"] == 3 and not rep["consumed"]
    assert rep["output_bytes"] == 3 * o * i * 2


def test_group_size_limits():
    from sym_b200 import pyreloc

    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.prepare_dispatch_group([])
    assert e.value.code == "invalid_options"
    t, o, i = _template(8, 16)
    entries = [(t, *_views(0x10000000 + k * 4096, 0x7f0000000000 + k * 4096, o, i), "h2d") for k in range(257)]
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.prepare_dispatch_group(entries)
    assert e.value.code == "invalid_options"


def test_overlapping_destinations_are_rejected():
    from sym_b200 import pyreloc

    t, o, i = _template()
    a = _views(0x10000000, 0x7f0000000000, o, i)
    b = _views(0x20000000, 0x7f0000000000 + 1000, o, i)  # overlaps a's destination
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.prepare_dispatch_group([(t, *a, "h2d"), (t, *b, "h2d")])
    assert e.value.code == "invalid_view" and "overlapping destinations" in str(e.value)


def test_destination_over_a_source_is_rejected():
    from sym_b200 import pyreloc

    t, o, i = _template()
    a = _views(0x10000000, 0x7f0000000000, o, i)
    b = _views(0x7f0000100000, 0x7f0000200000, o, i)
    # member 1 writes where member 0 reads
    b2 = (b[0], pyreloc.BufferView(0x10000000, o * i * 2, 0, [i, o], dense([i, o]), 2, "cuda", 0))
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.prepare_dispatch_group([(t, *a, "h2d"), (t, *b2, "h2d")])
    assert e.value.code == "invalid_view" and "overlaps the source" in str(e.value)


def test_mixed_devices_and_directions_are_rejected():
    from sym_b200 import pyreloc

    t, o, i = _template()
    a = _views(0x10000000, 0x7f0000000000, o, i, device=0)
    b = _views(0x20000000, 0x7f0000100000, o, i, device=1)
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.prepare_dispatch_group([(t, *a, "h2d"), (t, *b, "h2d")])
    assert e.value.code == "device_mismatch"
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.prepare_dispatch_group([(t, *a, "d2h")])
    assert e.value.code == "implementation_unavailable"


def test_member_view_errors_name_the_member():
    from sym_b200 import pyreloc

    t, o, i = _template()
    a = _views(0x10000000, 0x7f0000000000, o, i)
    bad = _views(0x20000000, 0x7f0000100000, o, i + 1)  # wrong extents
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.prepare_dispatch_group([(t, *a, "h2d"), (t, *bad, "h2d")])
    assert e.value.code == "plan_mismatch" and "group member 1" in str(e.value)


def test_group_execution_without_a_gpu_fails_loudly():
    """No CPU fallback: executing a group on a host without a GPU is a backend
    failure, and the group is consumed."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from sym_b200 import pyreloc

    t, o, i = _template(8, 16)
    src = np.zeros(o * i, np.int8)
    dst = np.zeros(o * i * 2, np.uint8)
    sv = pyreloc.BufferView(src.ctypes.data, src.nbytes, 0, [o, i], dense([o, i]), 1, "host", -1)
    dv = pyreloc.BufferView(dst.ctypes.data, dst.nbytes, 0, [i, o], dense([i, o]), 2, "cuda", 0)
    g = pyreloc.prepare_dispatch_group([(t, sv, dv, "h2d")])
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.execute_dispatch_group(g)
    assert e.value.code == "backend_failure"
    assert g.consumed and not dst.any()
    with pytest.raises(pyreloc.TransferError) as e:
        pyreloc.submit_dispatch_group(g)
    assert e.value.code == "already_executed"


def test_torch_group_bridge_validation():
    """reloc_torch.prepare_transfer_group: 1..256 fresh typed members on one
    canonical CUDA device, no member twice (no GPU needed to prepare)."""
    import torch
    from sym_b200.reloc_torch import dispatch, prepare_transfer_group
    from sym_b200.reloc_torch.compiler import CompilerClient
    from sym_b200.workloads import weight_recipe

    compiled = CompilerClient.from_environment().compile(weight_recipe("out_in_f16"))

    def req(rows, cols, device="cuda:0"):
        q = torch.zeros((rows, cols), dtype=torch.int8)
        return dispatch.prepare_typed_transfer(compiled, q, device, parameters={"scale": torch.ones(rows)})

    a, b = req(64, 128), req(32, 64)
    g = prepare_transfer_group([a, b])
    assert g.device == torch.device("cuda", 0)
    assert [d.shape for d in g.destinations] == [(128, 64), (64, 32)]
    assert g.destinations[0].strides == (64, 1) and g.destinations[0].dtype == "float16"
    with pytest.raises(ValueError):
        prepare_transfer_group([])
    with pytest.raises(ValueError):
        prepare_transfer_group([a, a])
    with pytest.raises(ValueError):
        prepare_transfer_group([req(8, 8, "cuda:0"), req(8, 8, "cuda:1")])
    with pytest.raises(TypeError):
        prepare_transfer_group([object()])
    used = req(8, 8)
    used.consumed = True
    with pytest.raises(RuntimeError):
        prepare_transfer_group([used])


def test_typed_and_quantize_members_mix():
    """Members with different plans, shapes and dtypes validate together."""
    from sym_b200 import pyreloc

    t, o, i = _template()
    qb = pyreloc.bind_typed(pyreloc.load_typed_plan(encode(recipe_c3("quantize"))), {"B": 1, "S": 2}, {})
    qt = pyreloc.prepare_dispatch_template(qb)
    n = 2 * 4096
    qs = pyreloc.BufferView(0x30000000, n * 4, 0, [1, 2, 4096], dense([1, 2, 4096]), 4, "host", -1)
    qd = pyreloc.BufferView(0x7f0000800000, n, 0, [1, 2, 4096], dense([1, 2, 4096]), 1, "cuda", 0)
    g = pyreloc.prepare_dispatch_group([(t, *_views(0x10000000, 0x7f0000000000, o, i), "h2d"), (qt, qs, qd, "h2d")])
    assert g.report["logical_transfers"] == 2
