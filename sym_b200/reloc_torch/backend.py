"""``RelocBackend``: a ``torch.compile`` backend that hands CPU -> GPU
relocation regions to the B200 executor (reference
``reloc_torch.backend.RelocBackend``, libreloc/python/reloc_torch/backend.py:91-430).

For each region ``fx_import.import_graph`` accepts, the backend compiles the
region's recipe once (in-process encoder), replaces the region's nodes by one
call of a ``_Region`` and returns the rewritten graph's ``forward`` wrapped in
a ``GraphCallable``. Per call a region

* checks its inputs against the captured metadata (CPU, dense, dtype, rank,
  every static extent as captured and every dynamic one bindable to its
  symbol, runtime parameters as declared; autograd off for inputs that
  require grad) and otherwise runs the ORIGINAL region's nodes, so a
  mismatched call never sees different semantics;
* runs typed recipes through ``dispatch.prepare_typed_transfer`` /
  ``execute_typed_transfer`` and layout-only recipes through
  ``pyreloc.make_transfer`` / ``execute_transfer``, ordered after the
  caller's current CUDA stream, into a fresh dense CUDA tensor.

The GPU work is the fused sm_100a kernels; there is no CPU path in the
replacement. Regions the importer rejects keep their original nodes, and
their reasons are available from ``stats()``.
"""
from __future__ import annotations

import threading
from collections import Counter

from .. import pyreloc
from . import dispatch
from . import symbolic as sx
from .compiler import CompilerClient, UnsupportedRecipe
from .fx_import import Exclusion, import_graph


def _needs_autograd(values):
    import torch

    return torch.is_grad_enabled() and any(isinstance(v, torch.Tensor) and v.requires_grad for v in values)


class _Region:
    """The replacement of one region: the compiled recipe plus the original
    nodes as a fallback callable with the same signature."""

    def __init__(self, backend, candidate, compiled, original):
        import torch

        self.backend = backend
        self.candidate = candidate
        self.compiled = compiled
        self.original = original
        src = candidate.recipe.source
        # None marks a dynamic extent (a plan symbol bound per call)
        self.shape = tuple(int(e.value) if isinstance(e, sx.Const) else None for e in src.shape)
        self.dtype = getattr(torch, src.dtype)
        dst = candidate.recipe.destination
        self.out_extents = tuple(dst.shape)
        self.out_dtype = getattr(torch, dst.dtype)
        self.device = candidate.device  # index None: the current device at call time
        self.vector = {b.name: len(b.extents) == 1 for b in compiled.recipe.parameter_bindings}
        self.__name__ = f"reloc_region_{candidate.tail}"

    def _eligible(self, src, params):
        import torch

        if not isinstance(src, torch.Tensor) or src.device.type != "cpu" or src.dtype != self.dtype:
            return False
        if src.dim() != len(self.shape) or not src.is_contiguous() or src.is_quantized:
            return False
        if any(want is not None and have != want for have, want in zip(src.shape, self.shape)):
            return False
        if src.numel() == 0:
            return False
        try:
            bindings = self.compiled.source_symbols(tuple(src.shape))
        except UnsupportedRecipe:
            return False  # one symbol at two different sizes
        declared = self.compiled.parameter_extents(bindings)
        if _needs_autograd((src, *params)):
            return False
        for name, p in zip(self.candidate.parameters, params):
            if not isinstance(p, torch.Tensor) or p.device.type != "cpu" or not p.is_contiguous():
                return False
            # f32 scales; integer zero points (the snapshot narrows them to int32, range-checked)
            want = (torch.float32,) if declared[name][0] == "float32" else (torch.int32, torch.int64, torch.int16,
                                                                            torch.int8)
            if p.dtype not in want:
                return False
            count = 1
            for e in declared[name][1]:
                count *= e
            if p.numel() != count:
                return False
        return True

    def __call__(self, src, *inputs):
        # inputs: the runtime parameters, then the scalar graph inputs the
        # original nodes read (SymInt sizes; the plan binds them from src)
        params = inputs[:len(self.candidate.parameters)]
        if not self._eligible(src, params):
            self.backend._count("fallbacks")
            return self.original(src, *inputs)
        self.backend._count("executions")
        import torch

        device = self.device if self.device.index is not None else \
            torch.device("cuda", torch.cuda.current_device())
        if self.compiled.typed:
            # per-channel scales are declared 1-D, per-tensor ones as one value
            parameters = {name: p.reshape(-1) if self.vector[name] else p.reshape(())
                          for name, p in zip(self.candidate.parameters, params)}
            request = dispatch.prepare_typed_transfer(self.compiled, src, device, parameters=parameters)
            return dispatch.execute_typed_transfer(request, resources=self.backend.resources).tensor
        return self._layout(src, device)

    def _layout(self, src, device):
        import torch

        bindings = self.compiled.source_symbols(tuple(src.shape))
        bound = self.backend._bound(self.compiled, bindings)
        out_shape = tuple(sx.expression(e).evaluate(bindings) for e in self.out_extents)
        out = torch.empty(out_shape, dtype=self.out_dtype, device=device)
        es = src.element_size()
        sv = pyreloc.BufferView(src.data_ptr(), src.numel() * es, 0, [src.numel()], [1], es, "host", -1)
        dv = pyreloc.BufferView(out.data_ptr(), out.numel() * es, 0, [out.numel()], [1], es, "cuda",
                                out.device.index)
        request = pyreloc.make_transfer(bound, sv, dv)
        stream = torch.cuda.current_stream(out.device).cuda_stream
        owner = None if self.backend.resources is None else self.backend.resources.native_typed
        pyreloc.execute_transfer(request, caller_stream=stream, resources=owner)
        return out


class GraphCallable:
    """The compiled function: the rewritten graph, or the original one when a
    call needs autograd (the replacement implements no backward)."""

    def __init__(self, original, rewritten, regions, backend):
        self.original = original
        self.rewritten = rewritten
        self.regions = tuple(regions)
        self._backend = backend

    def __call__(self, *args, **kwargs):
        self._backend._require_open()
        if self.rewritten is None or _needs_autograd(args):
            return self.original(*args, **kwargs)
        return self.rewritten(*args, **kwargs)


class RelocBackend:
    """``torch.compile(fn, backend=RelocBackend())``. ``stats()`` returns the
    counters and the importer's exclusions; ``close()`` disables the
    compiled functions (later calls raise)."""

    def __init__(self, *, compiler=None, transfer_resources=None, importer=None, **_):
        self.compiler = compiler or CompilerClient.from_environment()
        self.resources = transfer_resources
        self.importer = importer or import_graph
        self._lock = threading.Lock()
        self._counters = Counter()
        self._exclusions = []
        self._closed = False
        self._bound_cache = {}

    def _count(self, name, n=1):
        with self._lock:
            self._counters[name] += n

    def _require_open(self):
        if self._closed:
            raise RuntimeError("RelocBackend is closed")

    def _bound(self, compiled, bindings):
        key = (id(compiled), tuple(sorted(bindings.items())))
        with self._lock:
            hit = self._bound_cache.get(key)
        if hit is None or hit[0] is not compiled:
            if len(self._bound_cache) >= 256:  # dynamic regions bind once per distinct size
                with self._lock:
                    self._bound_cache.clear()
            hit = (compiled, pyreloc.bind(compiled.decoded_plan, bindings))
            with self._lock:
                self._bound_cache[key] = hit
        return hit[1]

    def stats(self):
        with self._lock:
            return {**self._counters, "exclusions": [(e.node, e.reason) for e in self._exclusions],
                    "closed": self._closed}

    def close(self):
        self._closed = True

    def __call__(self, gm, example_inputs):
        self._require_open()
        self._count("graphs")
        report = self.importer(gm, example_inputs)
        with self._lock:
            self._exclusions.extend(report.exclusions)
        if not report.candidates:
            return GraphCallable(gm.forward, None, (), self)
        import copy

        rewritten = copy.deepcopy(gm)
        graph = rewritten.graph
        by_name = {n.name: n for n in graph.nodes}
        regions = []
        for cand in report.candidates:
            try:
                compiled = self.compiler.compile(cand.recipe)
            except UnsupportedRecipe as error:
                with self._lock:
                    self._exclusions.append(Exclusion(cand.tail, error.reason))
                continue
            self._count("plan_compiles")
            members = [by_name[m] for m in cand.members]
            root = by_name[cand.source]
            params = [by_name[p] for p in cand.parameters]
            member_set = set(members)
            extras = []  # scalar graph inputs the members read (SymInt sizes)
            for m in members:
                for n in m.all_input_nodes:
                    if n not in member_set and n is not root and n not in params and n not in extras \
                            and n.op == "placeholder":
                        extras.append(n)
            try:
                original = _extract(rewritten, root, members, params + extras)
            except UnsupportedRecipe as error:
                with self._lock:
                    self._exclusions.append(Exclusion(cand.tail, error.reason))
                continue
            region = _Region(self, cand, compiled, original)
            tail = members[-1]
            with graph.inserting_before(tail):
                call = graph.call_function(region, (root, *params, *extras))
            tail.replace_all_uses_with(call)
            for m in reversed(members):
                graph.erase_node(m)
            regions.append(region)
            self._count("regions")
        graph.eliminate_dead_code()
        graph.lint()
        rewritten.recompile()
        return GraphCallable(gm.forward, rewritten.forward, regions, self)


def _extract(gm, root, members, params):
    """The region's original nodes as a standalone callable ``(src, *inputs)``
    (node_copy keeps the exact call targets and arguments); ``params`` are
    the other graph inputs the members read, in call order."""
    from torch.fx import Graph, GraphModule

    graph = Graph()
    mapping = {root: graph.placeholder("src")}
    for p in params:
        mapping[p] = graph.placeholder(p.name)
    member_set = set(members)
    needed = []

    def visit(n):
        if n in mapping or n in needed:
            return
        if n in member_set or n.op in ("call_function", "call_method"):
            for a in n.all_input_nodes:
                visit(a)
            needed.append(n)
            return
        raise UnsupportedRecipe("unsupported_symbolic_expr", f"region input {n.name} is not the source or a parameter")

    for m in members:
        visit(m)
    for n in gm.graph.nodes:
        if n in needed:
            mapping[n] = graph.node_copy(n, lambda x: mapping[x])
    graph.output(mapping[members[-1]])
    return GraphModule(gm, graph)


__all__ = ("GraphCallable", "RelocBackend")
