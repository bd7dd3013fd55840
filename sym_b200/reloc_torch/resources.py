"""Transfer resource ownership: the constructor and methods of the
reference's ``reloc_torch.resources.TransferResources``
(libreloc/python/reloc_torch/resources.py:51-143).

Here every transfer -- typed or layout-only -- runs on the typed contexts of
one ``pyreloc.DispatchResources`` (per device: a copy-engine and a compute
stream, the HBM ring, parameter buffers). What each keyword does:

* forwarded to the typed contexts: ``max_typed_retained_bytes``,
  ``max_typed_live_bytes``, ``max_typed_contexts``,
  ``typed_acquire_timeout_ms``;
* caps this executor meets by construction, checked for range:
  ``max_typed_streams`` (a context uses 2 streams, so at least 2),
  ``max_typed_contexts_per_device`` (one context per device, at least 1),
  ``max_typed_background_workers`` (no background transform workers: no plan
  runs on the CPU; at least 1);
* the reference's separate pool for layout-only transfers
  (``max_retained_bytes``, ``max_contexts``, ``max_contexts_per_device``,
  ``max_background_workers``, ``max_live_staging_bytes``,
  ``acquire_timeout_ms``) does not exist here: layout transfers share the
  typed contexts. Their defaults are accepted; any other value raises
  ``ValueError`` instead of being silently ignored.
"""
from __future__ import annotations

import operator
import os

# The reference's layout-transfer pool: the defaults it takes when not passed.
_LAYOUT_POOL_DEFAULTS = {"max_retained_bytes": 256 << 20, "max_contexts": 4, "max_contexts_per_device": 2,
                         "max_background_workers": 64, "max_live_staging_bytes": None, "acquire_timeout_ms": None}


def _at_least(name, value, minimum):
    if isinstance(value, bool):
        raise TypeError(f"{name} must be an integer")
    value = operator.index(value)
    if value < minimum:
        raise ValueError(f"{name} must be at least {minimum} on this executor")
    return value


class TransferResources:
    __slots__ = ("_typed", "_pid", "_configuration", "__weakref__")

    def __init__(self, *, max_retained_bytes=256 << 20, max_contexts=4, max_contexts_per_device=2,
                 max_background_workers=64, max_live_staging_bytes=None, acquire_timeout_ms=None,
                 max_typed_retained_bytes=64 << 20, max_typed_live_bytes=0, max_typed_streams=8,
                 max_typed_background_workers=64, max_typed_contexts=1, max_typed_contexts_per_device=1,
                 typed_acquire_timeout_ms=None):
        from .. import pyreloc

        given = {"max_retained_bytes": max_retained_bytes, "max_contexts": max_contexts,
                 "max_contexts_per_device": max_contexts_per_device,
                 "max_background_workers": max_background_workers,
                 "max_live_staging_bytes": max_live_staging_bytes, "acquire_timeout_ms": acquire_timeout_ms}
        for name, value in given.items():
            if value != _LAYOUT_POOL_DEFAULTS[name]:
                raise ValueError(f"{name}: layout-only transfers run on the typed contexts of this executor; "
                                 "size them with the max_typed_* / typed_* arguments")
        _at_least("max_typed_streams", max_typed_streams, 2)
        _at_least("max_typed_contexts_per_device", max_typed_contexts_per_device, 1)
        _at_least("max_typed_background_workers", max_typed_background_workers, 1)
        self._configuration = {**given, "max_typed_retained_bytes": max_typed_retained_bytes,
                               "max_typed_live_bytes": max_typed_live_bytes, "max_typed_streams": max_typed_streams,
                               "max_typed_background_workers": max_typed_background_workers,
                               "max_typed_contexts": max_typed_contexts,
                               "max_typed_contexts_per_device": max_typed_contexts_per_device,
                               "typed_acquire_timeout_ms": typed_acquire_timeout_ms}
        self._pid = os.getpid()
        self._typed = pyreloc.DispatchResources(max_retained_bytes=max_typed_retained_bytes,
                                                max_live_bytes=max_typed_live_bytes,
                                                max_contexts=_at_least("max_typed_contexts", max_typed_contexts, 1),
                                                acquire_timeout_ms=typed_acquire_timeout_ms)

    @property
    def native_typed(self):
        if os.getpid() != self._pid:
            raise RuntimeError("process_mismatch: transfer resources belong to another process")
        return self._typed

    native = native_typed

    @property
    def configuration(self):
        """The keywords this owner was built with."""
        return dict(self._configuration)

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
