"""Torch bridge of the B200 executor (reference package ``reloc_torch``):
recipes and the in-process plan encoder, typed transfers, transfer groups,
asynchronous submission and transfer resources."""
from . import dispatch
from .asynchronous import PrefetchWindow, TransferCompletion, TransferQueue
from .backend import GraphCallable, RelocBackend
from .group import GroupResult, PreparedTransferGroup, execute_transfer_group, prepare_transfer_group
from .resources import TransferResources

__all__ = ("GraphCallable", "GroupResult", "PrefetchWindow", "RelocBackend", "PreparedTransferGroup", "TransferCompletion", "TransferQueue",
           "TransferResources", "dispatch", "execute_transfer_group", "prepare_transfer_group")
