"""Helpers for wire v0 (layout-only) plans on the GPU and their checker."""
import numpy as np

from helpers import dense, resources


def expected_layout(blob, symbols, src):
    from oracle import oracle, ref

    src = np.ascontiguousarray(src).view(np.uint8).reshape(-1)
    if ref.available():
        return ref.LayoutPlan(blob, symbols).execute(src)
    from sym_b200 import pyreloc

    b = pyreloc.bind(pyreloc.load_plan(blob), symbols).describe()
    desc = {"layout": b, "result_extents": [b["total_bytes"] // b["element_size"]], "stages": [],
            "destination_bytes": b["total_bytes"]}
    dt = {1: "int8", 2: "float16", 4: "float32"}[b["element_size"]]
    return oracle.Program.from_description(desc, [dt]).execute(src)


def run_layout_gpu(blob, symbols, src, route="auto", device=0, chunk_size=0):
    import torch
    from sym_b200 import pyreloc

    bound = pyreloc.bind(pyreloc.load_plan(blob), symbols)
    host = torch.from_numpy(np.ascontiguousarray(src).view(np.uint8).reshape(-1).copy()).pin_memory()
    out = torch.empty(bound.total_bytes, dtype=torch.uint8, device=f"cuda:{device}")
    es = bound.element_size
    sv = pyreloc.BufferView(host.data_ptr(), host.numel(), 0, [host.numel() // es], [1], es, "host", -1)
    dv = pyreloc.BufferView(out.data_ptr(), out.numel(), 0, [out.numel() // es], [1], es, "cuda", device)
    req = pyreloc.make_transfer(bound, sv, dv)
    pyreloc.execute_transfer(req, resources=resources(), route=route, chunk_size=chunk_size)
    return out.cpu().numpy()
