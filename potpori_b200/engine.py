"""Model-agnostic interfaces the speculative-decode drivers use (``src/engine.rs``).

``argmax`` is the greedy pick of ``src/engine.rs:14-29``; ``DraftEngine`` and ``TargetChain``
mirror the traits of ``src/engine.rs:33-65``. The drivers only see these, so their
accept/reject logic is tested with synthetic engines.
"""
from __future__ import annotations

import math
from typing import List, Optional, Protocol, Sequence

TokenId = int


def argmax(row: Sequence[float]) -> Optional[TokenId]:
    """First index of the strict maximum; None for an empty row or any non-finite value."""
    if len(row) == 0:
        return None
    best, best_v = 0, -math.inf
    for i, v in enumerate(row):
        if not math.isfinite(v):
            return None
        if v > best_v:
            best, best_v = i, v
    return best


class DraftEngine(Protocol):
    def capacity(self) -> int: ...

    def draft(self, context: List[TokenId], gamma: int) -> List[TokenId]: ...


class TargetChain(Protocol):
    def capacity(self) -> int: ...

    def prefill(self, prompt: List[TokenId]) -> TokenId: ...

    def verify(self, start_pos: int, cur: TokenId, drafts: List[TokenId]) -> List[TokenId]: ...

    def is_eos(self, token: TokenId) -> bool: ...
