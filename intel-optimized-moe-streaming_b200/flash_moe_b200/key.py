"""Expert identity, the same value type as the reference's
``flash_moe.key.ExpertKey`` (``src/flash_moe/key.py:3-6``), plus store
counters in the spirit of ``StoreStats`` (``key.py:8-23``) for a store that
never touches disk."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ExpertKey:
    layer: int
    expert: int


@dataclass
class ArenaStats:
    """Counters of the HBM-resident expert arena.

    ``resident_bytes`` is what was uploaded once; ``host_reads`` counts
    ``read_all``/``read_tensor`` calls that copied an expert back to the host
    (compatibility path); ``prefetch_calls`` counts prefetch requests, which
    are no-ops because every expert is already resident."""

    resident_bytes: int = 0
    layers: int = 0
    host_reads: int = 0
    prefetch_calls: int = 0
