"""The shard fetch (workloads.PeerShardedFetch) with one rank, the path the
benchmark's single-GPU `value` runs: each matrix is one int8 copy from pinned
host memory into the shard arena (raw bytes) and one tile launch from there.
Results must equal the reference executor (oracle/_ref) bit for bit, from
host sources with the two shard buffers reused layer after layer, with copies
in pieces, and from preloaded (device-resident) shards. No process group is
needed for one rank."""
import numpy as np
import pytest

from helpers import encode, recipe_c4

pytestmark = pytest.mark.gpu

# out rows: 256 and 1024 are whole 128-row tiles (the tall kernel), 192 is not
SHAPES = [(256, 512), (1024, 256), (192, 1024)]


def _layers(count):
    import torch
    from sym_b200 import pyreloc

    plan = pyreloc.load_typed_plan(encode(recipe_c4()))
    layers = []
    for layer in range(count):
        rng = np.random.default_rng(300 + layer)
        mats = []
        for out_f, in_f in SHAPES:
            q = rng.integers(-128, 128, size=(out_f, in_f), dtype=np.int8)
            s = np.exp(rng.normal(-5, 0.5, out_f)).astype(np.float32)
            sym = {"out_features": out_f, "in_features": in_f}
            params = {"scale": ("float32", [out_f], s.tobytes())}
            bound = pyreloc.bind_typed(plan, sym, params)
            mats.append({"host": torch.from_numpy(q).pin_memory(), "q": q, "sym": sym, "params": params,
                         "tmpl": pyreloc.prepare_dispatch_template(bound)})
        layers.append(mats)
    return layers


def _want(ref_lib, m):
    return ref_lib.TypedProgram(encode(recipe_c4()), m["sym"], m["params"]).execute(m["q"].view(np.uint8).reshape(-1))


@pytest.mark.parametrize("chunk", [0, 96 << 10])
def test_one_rank_shard_fetch_matches_the_reference(ref_lib, chunk):
    import torch
    from sym_b200 import pyreloc
    from sym_b200.workloads import PeerShardedFetch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    res = pyreloc.DispatchResources()
    layers = _layers(2)
    wants = [[_want(ref_lib, m) for m in mats] for mats in layers]
    fetcher = PeerShardedFetch(res, 0, 1, 0, SHAPES, buffers=2, copy_chunk_bytes=chunk)
    outs = [[torch.full((i, o), -1, dtype=torch.float16, device=dev) for o, i in SHAPES] for _ in range(2)]

    def check(l):
        torch.cuda.synchronize(dev)
        for want, out in zip(wants[l % 2], outs[l % 2]):
            assert np.array_equal(out.view(torch.uint8).cpu().numpy().reshape(-1), want), f"layer {l}"

    for l in range(5):  # host sources; each shard buffer is refilled every other layer
        mats = layers[l % 2]
        fetcher.fetch([m["tmpl"] for m in mats], outs[l % 2], l % 2, [m["host"] for m in mats])
        if l >= 1:
            check(l - 1)
    check(4)
    for parity, mats in enumerate(layers):  # device-resident shards
        fetcher.preload(parity, [m["host"] for m in mats])
    for out in outs[0] + outs[1]:
        out.fill_(-1)
    for parity, mats in enumerate(layers):
        fetcher.fetch([m["tmpl"] for m in mats], outs[parity], parity)
    check(0)
    check(1)
    fetcher.close()
    res.close()
