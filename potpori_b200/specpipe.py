"""Depth-N pipelined speculative decoding (``src/specpipe.rs:29-194``).

Up to ``depth`` verification chunks are in flight, each drafted on the previous chunk's
drafts. When a chunk diverges from the target every chunk still in flight was drafted on a
wrong prefix: their results are drained and discarded, and drafting restarts from the
committed prefix. There is no rollback call: every shard writes its KV at absolute
positions and attends only below the chunk it runs, so a re-submission overwrites the stale
tail.
"""
from __future__ import annotations

from collections import deque
from typing import List, Protocol, Tuple

from .specdecode import SpecConfig, SpecStats, accept


class PipelinedChain(Protocol):
    """src/specpipe.rs:29-43: several chunks in flight, completing in FIFO order."""

    def capacity(self) -> int: ...

    def prefill(self, prompt: List[int]) -> int: ...

    def submit(self, start_pos: int, cur: int, drafts: List[int]) -> None: ...

    def poll(self) -> List[int]: ...

    def is_eos(self, token: int) -> bool: ...


class ChainError(RuntimeError):
    pass


def run_spec_decode_pipelined(draft, chain, prompt: List[int], cfg: SpecConfig,
                              depth: int) -> Tuple[List[int], SpecStats]:
    assert cfg.gamma > 0, "gamma must be positive"
    if cfg.max_new == 0:
        return [], SpecStats()
    capacity = min(chain.capacity(), draft.capacity())
    assert prompt and len(prompt) < capacity, "prompt must leave room in the KV cache"
    max_new = min(cfg.max_new, capacity - len(prompt))
    gamma = cfg.gamma
    depth = max(depth, 1)
    prompt_len = len(prompt)

    cur0 = chain.prefill(prompt)
    out: List[int] = []
    done = chain.is_eos(cur0)
    if not done:
        out.append(cur0)
    done = done or len(out) >= max_new
    dprefix = list(prompt) + [cur0]
    send_pos = prompt_len
    inflight: deque = deque()
    discard = 0
    traversals = 0
    while True:
        # FILL (src/specpipe.rs:89-121)
        while len(inflight) < depth and not done and discard == 0:
            cur = dprefix[-1]
            if chain.is_eos(cur):
                break
            remaining = max(capacity - send_pos, 0)
            if remaining == 0:
                break
            single = remaining <= gamma
            if single and inflight:
                break
            ds = [] if single else draft.draft(dprefix, gamma)
            assert single or len(ds) == gamma, "draft returned the wrong token count"
            chain.submit(send_pos, cur, ds)
            dprefix.extend(ds)
            inflight.append(ds)
            send_pos += gamma
            if single:
                break
        if not inflight:
            break
        # READ (src/specpipe.rs:126-183)
        r = chain.poll()
        ds = inflight.popleft()
        if len(r) != len(ds) + 1:
            raise ChainError(f"chain returned {len(r)} tokens for a {len(ds) + 1}-token chunk")
        traversals += 1
        if discard > 0:
            discard -= 1
            continue
        n = accept(ds, r)
        diverged = (not ds) or n != len(ds)
        committed = ds[:n] + [r[n]] if diverged else list(ds)
        for t in committed:
            if chain.is_eos(t):
                done = True
                break
            out.append(t)
            if len(out) >= max_new:
                done = True
                break
        if done:
            discard = len(inflight)
        elif diverged:
            discard = len(inflight)
            keep = prompt_len + len(out) - 1
            dprefix = list(prompt) + out
            send_pos = keep
    return out, SpecStats(len(out), traversals)
