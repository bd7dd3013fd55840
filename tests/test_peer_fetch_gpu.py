"""The multi-GPU weight fetch over NVLink (workloads.PeerShardedFetch) on 2
GPUs: every rank copies its int8 source rows, every rank's kernels read both
shards (the peer's through a CUDA IPC mapping) and both ranks end with the
exact single-GPU result, with equal and with uneven shards, from host and
from preloaded shards. Skips with fewer than 2 GPUs."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(256, 512), (1024, 256), (192, 1024)]


def _worker(rank, world, port, weights, failures):
    import datetime

    import torch
    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        from helpers import encode, recipe_c4
        from sym_b200 import pyreloc
        from sym_b200.workloads import PeerShardedFetch, WeightFetcher

        res = pyreloc.DispatchResources()
        plan = pyreloc.load_typed_plan(encode(recipe_c4()))
        layers = []
        for layer in range(2):
            rng = np.random.default_rng(100 + layer)
            mats = []
            for out_f, in_f in SHAPES:
                q = torch.from_numpy(rng.integers(-128, 128, size=(out_f, in_f), dtype=np.int8)).pin_memory()
                s = np.exp(rng.normal(-5, 0.5, out_f)).astype(np.float32)
                bound = pyreloc.bind_typed(plan, {"out_features": out_f, "in_features": in_f},
                                           {"scale": ("float32", [out_f], s.tobytes())})
                mats.append((q, torch.from_numpy(s), pyreloc.prepare_dispatch_template(bound)))
            layers.append(mats)
        fetcher = PeerShardedFetch(res, rank, world, rank, SHAPES, weights=weights, buffers=2)
        outs = [[torch.empty((i, o), dtype=torch.float16, device=dev) for o, i in SHAPES] for _ in range(2)]

        def check(l):
            torch.cuda.synchronize(dev)
            for (q, s, _), out in zip(layers[l % 2], outs[l % 2]):
                want = WeightFetcher.reference(q, s, dev, layout="out_in_f16")
                if not torch.equal(out.view(torch.int16), want.view(torch.int16)):
                    raise AssertionError(f"rank {rank} layer {l} differs")

        for l in range(5):  # host sources, buffers reused every other layer
            mats = layers[l % 2]
            fetcher.fetch([m[2] for m in mats], outs[l % 2], l % 2, [m[0] for m in mats])
            if l >= 1:
                check(l - 1)
        check(4)
        for d in range(2):  # preloaded shards (device-resident)
            fetcher.preload(d, [m[0] for m in layers[d]])
        torch.cuda.synchronize(dev)
        dist.barrier()
        for o in outs:
            for t in o:
                t.zero_()
        for l in range(2):
            fetcher.fetch([m[2] for m in layers[l]], outs[l], l, None)
            check(l)
        fetcher.close()
        dist.destroy_process_group()
    except Exception as error:  # reported to the parent
        failures.put(f"rank {rank}: {error!r}")
        raise


@pytest.mark.parametrize("weights", [None, [1.0, 3.0]])
def test_two_rank_peer_fetch(weights):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = 29600 + (0 if weights is None else 1)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, weights, failures)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not failures.empty():
        msgs.append(failures.get())
    assert codes == [0, 0], (codes, msgs)
