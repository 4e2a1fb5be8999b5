"""Admission of queued tokens into a step whose adapters must fit the slot pool.

The reference refuses a batch that names more distinct adapters than the pool
has slots (``MultiLoRAManager.prepare_lora_batch`` raises,
multi_lora/manager.py:172-180; ``validate_lora_batch``, batching.py:33-39), and
its only batch composer is the bench-side ``TierRotation``
(multi_lora/scheduling.py:22-86), which never asks for more than K adapters.
A server with a heavy-tailed adapter mix (Zipf over hundreds of adapters) has
to choose which tokens run now and which wait; this module is that choice,
so the pool never sees an infeasible batch.

Rule (per step, ``max_tokens`` tokens at most, ``slots`` distinct adapters at
most; ``None`` = the base model, which takes a slot like any adapter):

1. Candidates are taken in three tiers, each in queue order:
   a. tokens deferred by earlier steps (oldest first), so no token waits
      forever;
   b. tokens whose adapter is already resident in the pool (no load);
   c. all other tokens.
   With ``resident_first=False`` tiers b and c merge into queue order.
2. A candidate is admitted while its adapter is already admitted this step or
   fewer than ``slots`` adapters are; otherwise it is deferred.
3. Admitted tokens are returned in their original queue order (row order of
   the batch is preserved), deferred ones in the order they should be retried.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Hashable, Iterable, List, Optional, Sequence, Set


@dataclass
class Admission:
    """Outcome of one step: queue positions admitted (ascending) and deferred (retry order)."""

    admitted: List[int]
    deferred: List[int]
    adapters: Set[Optional[Hashable]] = field(default_factory=set)


class AdmissionPolicy:
    """Chooses the tokens of one step so that they name at most ``slots`` adapters."""

    def __init__(self, slots: int, *, resident_first: bool = True) -> None:
        if slots < 1:
            raise ValueError(f"slots must be >= 1 (got {slots})")
        self.slots = slots
        self.resident_first = resident_first

    def admit(self, names: Sequence[Optional[Hashable]], *, resident: Iterable[Optional[Hashable]] = (),
              n_deferred: int = 0, max_tokens: Optional[int] = None) -> Admission:
        """``names[i]`` is the adapter of queued token i; the first ``n_deferred``
        entries are tokens deferred by earlier steps (oldest first)."""
        if not 0 <= n_deferred <= len(names):
            raise ValueError(f"n_deferred {n_deferred} outside [0, {len(names)}]")
        cap = len(names) if max_tokens is None else max(0, int(max_tokens))
        res = set(resident)
        order = list(range(n_deferred))
        fresh = range(n_deferred, len(names))
        if self.resident_first:
            order += [i for i in fresh if names[i] in res]
            order += [i for i in fresh if names[i] not in res]
        else:
            order += list(fresh)
        chosen: Set[Optional[Hashable]] = set()
        admitted, deferred = [], []
        for i in order:
            n = names[i]
            if len(admitted) < cap and (n in chosen or len(chosen) < self.slots):
                chosen.add(n)
                admitted.append(i)
            else:
                deferred.append(i)
        admitted.sort()
        return Admission(admitted=admitted, deferred=deferred, adapters=chosen)


class TokenQueue:
    """Queued tokens (adapter names) carried across steps with an admission policy.

    ``step(new)`` appends new arrivals, admits up to ``max_tokens`` of the
    queue and keeps the rest (deferred first next time). It returns the
    admitted tokens' adapter names in queue order.
    """

    def __init__(self, policy: AdmissionPolicy, max_tokens: int) -> None:
        self.policy = policy
        self.max_tokens = max_tokens
        self.pending: List[Optional[Hashable]] = []

    def step(self, new: Sequence[Optional[Hashable]], *, resident: Iterable[Optional[Hashable]] = ()) -> List:
        queue = self.pending + list(new)
        adm = self.policy.admit(queue, resident=resident, n_deferred=len(self.pending),
                                max_tokens=self.max_tokens)
        self.pending = [queue[i] for i in adm.deferred]
        return [queue[i] for i in adm.admitted]
