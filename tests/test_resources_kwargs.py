"""TransferResources / DispatchResources keywords: each one is forwarded,
checked as a cap the executor meets, or refused -- none is silently dropped
(reference constructor: libreloc/python/reloc_torch/resources.py:69-97)."""
import pytest


def test_forwarded_keywords_reach_the_typed_contexts():
    from sym_b200.reloc_torch.resources import TransferResources

    with TransferResources(max_typed_retained_bytes=3 << 20, max_typed_live_bytes=5 << 20,
                           max_typed_contexts=2) as owner:
        stats = owner.stats()["typed"]
        assert stats["retained_limit"] == 3 << 20
        assert stats["live_limit"] == 5 << 20
        assert stats["context_limit"] == 2
        assert owner.configuration["max_typed_contexts"] == 2


def test_reference_defaults_are_accepted():
    from sym_b200.reloc_torch.resources import TransferResources

    TransferResources(max_retained_bytes=256 << 20, max_contexts=4, max_contexts_per_device=2,
                      max_background_workers=64, max_live_staging_bytes=None, acquire_timeout_ms=None,
                      max_typed_streams=8, max_typed_background_workers=64, max_typed_contexts_per_device=1).close()


@pytest.mark.parametrize("name,value", [("max_retained_bytes", 1 << 20), ("max_contexts", 8),
                                        ("max_contexts_per_device", 1), ("max_background_workers", 2),
                                        ("max_live_staging_bytes", 1 << 20), ("acquire_timeout_ms", 10)])
def test_layout_pool_keywords_are_refused_not_ignored(name, value):
    from sym_b200.reloc_torch.resources import TransferResources

    with pytest.raises(ValueError, match=name):
        TransferResources(**{name: value})


@pytest.mark.parametrize("name,value", [("max_typed_streams", 1), ("max_typed_contexts_per_device", 0),
                                        ("max_typed_background_workers", 0), ("max_typed_contexts", 0)])
def test_caps_below_what_a_context_needs_are_refused(name, value):
    from sym_b200.reloc_torch.resources import TransferResources

    with pytest.raises(ValueError, match=name):
        TransferResources(**{name: value})


def test_dispatch_resources_checks_its_caps():
    from sym_b200 import pyreloc

    with pytest.raises(ValueError, match="max_streams"):
        pyreloc.DispatchResources(max_streams=1)
    pyreloc.DispatchResources(max_streams=2, max_contexts_per_device=1).close()
