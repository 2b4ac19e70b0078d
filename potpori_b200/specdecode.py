"""Greedy speculative decoding, one chunk at a time (``src/specdecode.rs:1-125``).

Each round the draft proposes ``gamma`` tokens, the target verifies ``[cur] + drafts`` in one
pass, and the longest prefix that matches the target's own greedy tokens is committed plus
the target's token at the first mismatch. Only the target's picks are committed, so the
output equals plain greedy decoding of the target whatever the draft proposes.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple


@dataclass
class SpecConfig:
    gamma: int
    max_new: int


@dataclass
class SpecStats:
    committed: int = 0
    traversals: int = 0

    def toks_per_traversal(self) -> float:
        return self.committed / max(self.traversals, 1)


def accept(drafts: List[int], r: List[int]) -> int:
    """Longest prefix where the draft matched the target's argmax (src/specdecode.rs:92-95)."""
    n = 0
    while n < len(drafts) and n < len(r) and drafts[n] == r[n]:
        n += 1
    return n


def run_spec_decode(draft, target, prompt: List[int], cfg: SpecConfig) -> Tuple[List[int], SpecStats]:
    assert cfg.gamma > 0, "gamma must be positive"
    if cfg.max_new == 0:
        return [], SpecStats()
    capacity = min(target.capacity(), draft.capacity())
    assert prompt and len(prompt) < capacity, "prompt must leave room in the KV cache"
    max_new = min(cfg.max_new, capacity - len(prompt))
    gamma = cfg.gamma
    out: List[int] = []
    traversals = 0
    cur = target.prefill(prompt)
    base = len(prompt)
    while True:
        if target.is_eos(cur) or len(out) >= max_new:
            break
        context = list(prompt) + out + [cur]
        drafts = [] if capacity - base <= gamma else draft.draft(context, gamma)
        r = target.verify(base, cur, drafts)
        assert len(r) == len(drafts) + 1, "verify must return drafts.len()+1 argmaxes"
        traversals += 1
        n = accept(drafts, r)
        correction = r[n]
        stop = False
        for t in [cur] + drafts[:n]:
            if target.is_eos(t):
                stop = True
                break
            out.append(t)
            if len(out) >= max_new:
                stop = True
                break
        if stop:
            break
        cur = correction
        base += n + 1
    return out, SpecStats(len(out), traversals)
