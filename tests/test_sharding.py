"""Sharded weight fetch, host logic on CPU: world-size-2 ``gloo`` ranks each
produce their result-row window of a config-5-shaped matrix with the checker
(the device path's window semantics, typed::executeHostChunk), all-gather the
windows, and must reassemble exactly the whole-matrix result. The GPU path of
the same windows is covered by test_gpu_parity.py::test_c4_row_windows."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out_f, in_f, result_path):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "tests")]
    import torch
    import torch.distributed as dist

    from helpers import encode, recipe_c4
    from oracle import oracle
    from sym_b200 import pyreloc
    from sym_b200.workloads import shard_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(21)
    q = rng.integers(-127, 128, size=(out_f, in_f), dtype=np.int8)
    scale = np.exp(rng.normal(-5, 0.5, out_f)).astype(np.float32)
    blob = encode(recipe_c4())
    sym = {"out_features": out_f, "in_features": in_f}
    params = {"scale": ("float32", [out_f], scale.tobytes())}
    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(blob), sym, params).describe()
    prog = oracle.Program.from_description(bound, ["int8", "float32", "float16"])
    b, e = shard_bounds(in_f, world, rank)
    shard = torch.from_numpy(prog.execute_rows(q.reshape(-1).view(np.uint8), b, e).copy())
    full = torch.empty(in_f * out_f * 2, dtype=torch.uint8)
    dist.all_gather_into_tensor(full, shard)
    if rank == 0:
        np.save(result_path, full.numpy())
        np.save(str(result_path) + ".whole.npy", prog.execute(q.reshape(-1).view(np.uint8)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("in_f", [256, 1024])
def test_two_rank_windows_reassemble_the_matrix(tmp_path, in_f):
    import torch.multiprocessing as mp

    out_f = 96
    result = tmp_path / "full.npy"
    mp.start_processes(_rank_main, args=(2, _free_port(), out_f, in_f, str(result)), nprocs=2,
                       start_method="spawn")
    full = np.load(result)
    whole = np.load(str(result) + ".whole.npy")
    assert np.array_equal(full, whole)


def test_shard_bounds_partition():
    from sym_b200.workloads import shard_bounds

    for extent in (1, 7, 8192, 28672):
        for world in (1, 2, 3, 4, 8):
            bounds = [shard_bounds(extent, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == extent
            assert all(bounds[i][1] == bounds[i + 1][0] for i in range(world - 1))
            assert max(e - b for b, e in bounds) - min(e - b for b, e in bounds) <= 1


def test_weighted_row_bounds():
    """Shard sizes follow the weights, on 64-row multiples where possible, and
    always tile the rows exactly."""
    from sym_b200.workloads import weighted_row_bounds

    assert weighted_row_bounds(28672, [1] * 8) == [3584 * k for k in range(9)]
    b = weighted_row_bounds(28672, [23] * 4 + [35] * 4)
    assert b[0] == 0 and b[-1] == 28672 and all(x % 64 == 0 for x in b)
    sizes = [b[i + 1] - b[i] for i in range(8)]
    assert sizes[0] < sizes[7] and abs(sizes[7] / sizes[0] - 35 / 23) < 0.05
    assert weighted_row_bounds(100, [1, 1, 1]) == [0, 33, 67, 100]  # no 64-row alignment possible
    assert weighted_row_bounds(1024, [1, 0.001]) == [0, 1024, 1024]  # a rank may get nothing
    import pytest

    with pytest.raises(ValueError):
        weighted_row_bounds(64, [1, 0])
