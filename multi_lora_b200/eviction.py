"""Victim choice when the slot pool is full (drop-in for ``multi_lora/eviction.py``).

``lru``: every use moves the name to the back; the front is least recent.
``fifo``: names enter once, on first use, and keep that order.
The base model (``None``) is never queued; it is evicted only as a last resort.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Optional, Set

_KINDS = ("lru", "fifo")


class EvictionPolicy:
    def __init__(self, kind: str = "lru") -> None:
        if kind not in _KINDS:
            raise ValueError(f"eviction policy {kind!r} is not one of {', '.join(_KINDS)}")
        self.kind = kind
        self.order: "OrderedDict[str, None]" = OrderedDict()  # front = evicted first
        self.eviction_count = 0

    def mark_used(self, name: Optional[str]) -> None:
        if name is None:
            return
        if self.kind == "lru" and name in self.order:
            self.order.move_to_end(name)
        else:
            self.order.setdefault(name, None)

    def select_victim(self, candidates: Set[Optional[str]]) -> Optional[str]:
        """Oldest queued name among ``candidates``; the base model only when no adapter is a candidate."""
        for name in self.order:
            if name in candidates:
                self.eviction_count += 1
                return name
        if None in candidates:
            self.eviction_count += 1
            return None
        raise RuntimeError(f"none of the {len(candidates)} candidate(s) {sorted(map(str, candidates))} can be evicted")

    def remove(self, name: Optional[str]) -> None:
        if name is not None:
            self.order.pop(name, None)
