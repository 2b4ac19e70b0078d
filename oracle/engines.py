"""Oracle-backed engines for the speculative-decode drivers (test infrastructure and the
timed CPU baseline): a chain of oracle shards (``src/node.rs`` head/middle/tail, each hop a
plain array) and the incremental draft of ``src/qwen/draft.rs:14-93`` on an oracle model.
The greedy pick is ``src/engine.rs:14-29`` on the host, as the reference's tail does
(``src/node.rs:265-267``)."""
from __future__ import annotations

from collections import deque
from typing import List

from . import OracleShard, argmax

EOS_TOKENS = (151645, 151643)


class OracleChain:
    def __init__(self, stages: List[OracleShard], chunk: int):
        self.stages = stages
        self.chunk = chunk
        self.q: deque = deque()
        self.forwards = 0

    def capacity(self) -> int:
        return min(s.capacity for s in self.stages)

    def _run(self, pos: int, tokens: List[int]) -> List[int]:
        h = self.stages[0].forward(pos, tokens=tokens)
        for s in self.stages[1:]:
            h = s.forward(pos, hidden=h)
        self.forwards += 1
        picks = [argmax(row) for row in h]
        if any(p is None for p in picks):
            raise RuntimeError("non-finite or empty logits")
        return picks

    def prefill(self, prompt: List[int]) -> int:
        pos, last = 0, 0
        while pos < len(prompt):
            take = self.chunk if len(prompt) - pos >= self.chunk else 1
            last = self._run(pos, prompt[pos:pos + take])[-1]
            pos += take
        return last

    def submit(self, pos: int, cur: int, drafts: List[int]) -> None:
        self.q.append(self._run(pos, [cur] + list(drafts)))

    def poll(self) -> List[int]:
        return self.q.popleft()

    def verify(self, pos: int, cur: int, drafts: List[int]) -> List[int]:
        return self._run(pos, [cur] + list(drafts))

    def is_eos(self, t: int) -> bool:
        return t in EOS_TOKENS


class OracleDraft:
    def __init__(self, model: OracleShard, chunk: int):
        self.model = model
        self.chunk = chunk
        self.fed: List[int] = []
        self.forwards = 0

    def capacity(self) -> int:
        return self.model.capacity

    def _pick(self, pos: int, tokens: List[int]) -> int:
        self.forwards += 1
        row = self.model.forward(pos, tokens=tokens)[-1]
        p = argmax(row)
        if p is None:
            raise RuntimeError("non-finite or empty logits")
        return p

    def draft(self, context: List[int], gamma: int) -> List[int]:
        n = len(context)
        agree = 0
        for a, b in zip(self.fed, context):
            if a != b:
                break
            agree += 1
        pos = min(agree, max(n - 1, 0))
        start = pos
        cur = 0
        while pos < n:
            take = self.chunk if self.chunk > 1 and n - pos >= self.chunk else 1
            cur = self._pick(pos, context[pos:pos + take])
            pos += take
        del self.fed[start:]
        self.fed.extend(context[start:n])
        out = [cur]
        for p in range(n, n + gamma - 1):
            self.fed.append(cur)
            cur = self._pick(p, [cur])
            out.append(cur)
        return out
