"""Transfer resource ownership (reference ``reloc_torch.resources.TransferResources``,
libreloc/python/reloc_torch/resources.py:51-143): a bounded owner of typed
contexts retained across blocking transfers. Here a typed context is one
device's streams, HBM ring and parameter buffers (``pyreloc.DispatchResources``);
there are no host worker pools because no plan runs on the CPU.
"""
from __future__ import annotations

import os


class TransferResources:
    __slots__ = ("_typed", "_pid", "_configuration", "__weakref__")

    def __init__(self, *, max_retained_bytes=256 << 20, max_contexts=4, max_contexts_per_device=2,
                 max_background_workers=64, max_live_staging_bytes=None, acquire_timeout_ms=None,
                 max_typed_retained_bytes=64 << 20, max_typed_live_bytes=0, max_typed_streams=8,
                 max_typed_background_workers=64, max_typed_contexts=1, max_typed_contexts_per_device=1,
                 typed_acquire_timeout_ms=None):
        from .. import pyreloc

        self._configuration = {k: v for k, v in locals().items() if k not in ("self", "pyreloc")}
        self._pid = os.getpid()
        self._typed = pyreloc.DispatchResources(max_retained_bytes=max_typed_retained_bytes,
                                                max_live_bytes=max_typed_live_bytes,
                                                max_contexts=max_typed_contexts,
                                                acquire_timeout_ms=typed_acquire_timeout_ms)

    @property
    def native_typed(self):
        if os.getpid() != self._pid:
            raise RuntimeError("process_mismatch: transfer resources belong to another process")
        return self._typed

    native = native_typed

    @property
    def closed(self):
        return self._typed.closed

    def stats(self):
        return {"typed": self.native_typed.stats()}

    def clear(self):
        self.native_typed.clear()

    def close(self):
        self.native_typed.close()

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        self.close()
        return False

    def __reduce_ex__(self, protocol):
        raise TypeError("transfer resources cannot be serialized")
