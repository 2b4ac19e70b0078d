"""Depth-N pipelined speculative decoding (``src/specpipe.rs:29-194``).

Up to ``depth`` verification chunks are in flight, each drafted on the previous chunk's
drafts. When a chunk diverges from the target every chunk still in flight was drafted on a
wrong prefix: their results are drained and discarded, and drafting restarts from the
committed prefix. There is no rollback call: every shard writes its KV at absolute
positions and attends only below the chunk it runs, so a re-submission overwrites the stale
tail.

``PipelinedDriver`` is the same loop cut into steps (one FILL + one READ per step) so a
benchmark can time a fixed number of them; ``run_spec_decode_pipelined`` runs it to the end.
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


class PipelinedDriver:
    def __init__(self, draft, chain, prompt: List[int], cfg: SpecConfig, depth: int):
        assert cfg.gamma > 0, "gamma must be positive"
        self.draft, self.chain, self.cfg = draft, chain, cfg
        self.prompt = list(prompt)
        self.capacity = min(chain.capacity(), draft.capacity())
        assert self.prompt and len(self.prompt) < self.capacity, \
            "prompt must leave room in the KV cache"
        self.max_new = min(cfg.max_new, self.capacity - len(self.prompt))
        self.gamma = cfg.gamma
        self.depth = max(depth, 1)
        self.out: List[int] = []
        self.traversals = 0
        self.finished = cfg.max_new == 0
        self.started = False

    def start(self) -> None:
        """Prefill the prompt (src/specpipe.rs:68-81)."""
        self.started = True
        if self.finished:
            return
        cur0 = self.chain.prefill(self.prompt)
        self.done = self.chain.is_eos(cur0)
        if not self.done:
            self.out.append(cur0)
        self.done = self.done or len(self.out) >= self.max_new
        self.dprefix = self.prompt + [cur0]
        self.send_pos = len(self.prompt)
        self.inflight: deque = deque()
        self.discard = 0

    def step(self) -> bool:
        """One FILL + one READ (src/specpipe.rs:87-183). False once generation has ended."""
        if not self.started:
            self.start()
        if self.finished:
            return False
        chain, gamma = self.chain, self.gamma
        while len(self.inflight) < self.depth and not self.done and self.discard == 0:
            cur = self.dprefix[-1]
            if chain.is_eos(cur):
                break
            remaining = max(self.capacity - self.send_pos, 0)
            if remaining == 0:
                break
            single = remaining <= gamma
            if single and self.inflight:
                break
            ds = [] if single else self.draft.draft(self.dprefix, gamma)
            assert single or len(ds) == gamma, "draft returned the wrong token count"
            chain.submit(self.send_pos, cur, ds)
            self.dprefix.extend(ds)
            self.inflight.append(ds)
            self.send_pos += gamma
            if single:
                break
        if not self.inflight:
            self.finished = True
            return False
        r = chain.poll()
        ds = self.inflight.popleft()
        if len(r) != len(ds) + 1:
            raise ChainError(f"chain returned {len(r)} tokens for a {len(ds) + 1}-token chunk")
        self.traversals += 1
        if self.discard > 0:
            self.discard -= 1
            return True
        n = accept(ds, r)
        diverged = (not ds) or n != len(ds)
        committed = ds[:n] + [r[n]] if diverged else list(ds)
        for t in committed:
            if chain.is_eos(t):
                self.done = True
                break
            self.out.append(t)
            if len(self.out) >= self.max_new:
                self.done = True
                break
        if self.done:
            self.discard = len(self.inflight)
        elif diverged:
            self.discard = len(self.inflight)
            keep = len(self.prompt) + len(self.out) - 1
            self.dprefix = self.prompt + self.out
            self.send_pos = keep
        return True

    def stats(self) -> SpecStats:
        return SpecStats(len(self.out), self.traversals)


def run_spec_decode_pipelined(draft, chain, prompt: List[int], cfg: SpecConfig,
                              depth: int) -> Tuple[List[int], SpecStats]:
    d = PipelinedDriver(draft, chain, prompt, cfg, depth)
    if cfg.max_new == 0:
        return [], SpecStats()
    d.start()
    while d.step():
        pass
    return d.out, d.stats()
