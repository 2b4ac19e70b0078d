"""In-box chains of shards: the reference's head/middle/tail chain (src/node.rs:372-633) with
the QUIC hop replaced by device-to-device copies.

``LocalChain`` runs every stage in this process (stages may sit on different GPUs; the
hidden rows move with a peer copy over NVLink, ordered by events, and nothing waits on the
host until a result is polled). It implements the ``PipelinedChain`` contract of
src/specpipe.rs:29-43 (submit / poll in FIFO order) and the ``TargetChain`` contract of
src/engine.rs:55-65 (prefill / verify).
"""
from __future__ import annotations

from collections import deque
from typing import List, Sequence

from .config import is_eos
from .shard import Shard
from .target import NonFiniteLogits

RING = 64


class HandshakeError(RuntimeError):
    """Two adjacent stages disagree on the session (src/transport.rs:299-358)."""


def hello_mismatch(expected: dict, got: dict) -> str:
    """Why `got` (the upstream stage's hello) does not fit `expected` (what this stage serves):
    SessionHello::mismatch, src/transport.rs:256-291."""
    diffs = []
    if got["model"] != expected["model"]:
        diffs.append(f"model {got['model']!r} (this node has {expected['model']!r})")
    if got["next_layer"] != expected["next_layer"]:
        diffs.append(f"next layer {got['next_layer']} (this node starts at {expected['next_layer']})")
    if got["max_seq"] != expected["max_seq"]:
        diffs.append(f"max_seq {got['max_seq']} (this node has {expected['max_seq']})")
    if got["chunk"] != expected["chunk"]:
        diffs.append(f"chunk {got['chunk']} (this node has {expected['chunk']})")
    if got["taps"] != expected["taps"]:
        diffs.append(f"tapped layers {got['taps']} (this node has {expected['taps']})")
    return "upstream expects " + ", ".join(diffs)


def check_link(up_range, up_hello: dict, down_range, down_hello: dict) -> None:
    """receive_hello (src/transport.rs:339-358) for one link: the downstream stage accepts the
    session only if the upstream hello equals its own; the error names the downstream node
    and the settings that differ."""
    if up_hello != down_hello:
        raise HandshakeError(f"node [{down_range[0]}, {down_range[1]}): "
                             f"{hello_mismatch(down_hello, up_hello)}")


def session_taps(stages) -> List[int]:
    """The session's tapped layers: every stage's, ascending (each node reports its own)."""
    return sorted({l for s in stages for l in s.tap_layers()})


class LocalChain:
    def __init__(self, stages: Sequence[Shard]):
        assert stages and stages[0].first
        for a, b in zip(stages, stages[1:]):
            assert a.range()[1] == b.range()[0], "stages must be contiguous"
        # The handshake of src/transport.rs:299-358 on every link: each stage's hello carries
        # the session's tapped layers; the chain must end at the model's last layer (Ready).
        taps = session_taps(stages)
        for a, b in zip(stages, stages[1:]):
            up = dict(a.hello(a.range()[1]), taps=taps)
            down = dict(b.hello(b.range()[0]), taps=taps)
            check_link(a.range(), up, b.range(), down)
        if not stages[-1].last:
            raise HandshakeError(f"the chain ends at layer {stages[-1].range()[1]}, but the "
                                 f"model has {stages[-1].model_layers()}")
        self.stages = list(stages)
        self.chunk = stages[0].chunk_size() or 8
        self.inflight: deque = deque()
        self.slot = 0
        self.submitted = 0

    # ---- PipelinedChain ----
    def capacity(self) -> int:
        return min(s.capacity() for s in self.stages)

    def submit(self, start_pos: int, cur: int, drafts: List[int]) -> None:
        if len(self.inflight) >= RING:
            raise RuntimeError("too many chunks in flight")
        tokens = [cur] + list(drafts)
        m = len(tokens)
        width = max(self.chunk, m)
        first, last = self.stages[0], self.stages[-1]
        first.set_step(start_pos, m, tokens=tokens, drafts=drafts if first.last else ())
        first.step_device(width)
        for prev, st in zip(self.stages, self.stages[1:]):
            st.handoff_from(prev, m)
            st.set_step(start_pos, m, drafts=drafts if st.last else ())
            st.step_device(width)
        last.result_enqueue(self.slot)
        self.inflight.append((self.slot, m))
        self.slot = (self.slot + 1) % RING
        self.submitted += 1

    def poll(self) -> List[int]:
        slot, m = self.inflight.popleft()
        r = self.stages[-1].result_wait(slot, m)
        if not r.finite:
            raise NonFiniteLogits("the shard produced missing or non-finite logits")
        return r.argmax

    def prefill(self, prompt: List[int], one_pass: bool = True) -> int:
        """The greedy pick after the prompt. The reference streams the prompt through the
        chain in chunk-sized steps (src/node.rs:538-566); when every stage can
        (Shard.can_prefill), the stages write the K/V rows of all but the last token in one
        pass each instead, the output rows of each stage handed to the next (a peer copy
        across devices), and the last token is submitted as the step that yields the pick.
        Several stages take up to 2048 prompt rows in one pass; one stage any number.
        one_pass=False keeps the chunked steps."""
        n = len(prompt) - 1
        if (one_pass and n > 0 and all(s.can_prefill() for s in self.stages)
                and (len(self.stages) == 1 or n <= Shard.PREFILL_MAX)):
            while self.inflight:
                self.poll()
            self.stages[0].prefill(0, prompt[:-1])
            for prev, st in zip(self.stages, self.stages[1:]):
                st.prefill_handoff_from(prev, n)
                st.prefill_hidden(0, n)
            self.submit(n, prompt[-1], [])
            return self.poll()[-1]
        pos = 0
        while pos < len(prompt):
            take = self.chunk if len(prompt) - pos >= self.chunk else 1
            piece = prompt[pos:pos + take]
            self.submit(pos, piece[0], piece[1:])
            pos += take
            while len(self.inflight) > RING // 2:
                self.poll()
        last = 0
        while self.inflight:
            last = self.poll()[-1]
        return last

    # ---- TargetChain ----
    def verify(self, start_pos: int, cur: int, drafts: List[int]) -> List[int]:
        self.submit(start_pos, cur, drafts)
        return self.poll()

    def is_eos(self, token: int) -> bool:
        return is_eos(token)

    def reset(self) -> None:
        for s in self.stages:
            s.reset()
