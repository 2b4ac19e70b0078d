"""The speculative-decode drivers against plain greedy decoding, with synthetic engines
(the reference's own driver tests, src/specdecode.rs:127-267 and src/specpipe.rs:196-662,
restated): both drivers must reproduce greedy decoding for every draft quality, gamma,
depth and stop condition, leave nothing in flight, and keep speculation within bounds."""
from collections import deque

import pytest

from potpori_b200.specdecode import SpecConfig, run_spec_decode
from potpori_b200.specpipe import PipelinedDriver, run_spec_decode_pipelined

EOS = 9999


class Truth:
    """Next token = a hash of the whole prefix; EOS once `eos_at` tokens were generated."""

    def __init__(self, prompt_len, eos_at=None):
        self.prompt_len, self.eos_at = prompt_len, eos_at

    def next(self, prefix):
        if self.eos_at is not None and len(prefix) - self.prompt_len >= self.eos_at:
            return EOS
        h = 0x9E3779B9
        for t in prefix:
            h = (((h << 5) | (h >> 27)) & 0xFFFFFFFF)
            h = (h * 0x85EBCA6B) & 0xFFFFFFFF
            h ^= t & 0xFFFFFFFF
        return h % 50 + 1

    def greedy(self, prompt, max_new):
        ctx, out = list(prompt), []
        while len(out) < max_new:
            t = self.next(ctx)
            if t == EOS:
                break
            out.append(t)
            ctx.append(t)
        return out


class KvPipe:
    """Position-indexed 'KV' of fed tokens; results computed at submit time from the KV as
    it stands, so stale chunks see stale state and overwrite-rollback is exercised."""

    def __init__(self, truth, capacity=1 << 30):
        self.truth, self.kv, self.q, self.used, self.cap = truth, [], deque(), 0, capacity
        self.singles = 0

    def capacity(self):
        return self.cap

    def feed(self, start, tokens):
        assert start <= len(self.kv), "chunk leaves a KV gap"
        del self.kv[start:]
        out = []
        for t in tokens:
            self.kv.append(t)
            out.append(self.truth.next(self.kv))
        self.used = max(self.used, len(self.kv))
        return out

    def prefill(self, prompt):
        self.q.clear()
        return self.feed(0, prompt)[-1]

    def submit(self, pos, cur, drafts):
        assert pos + len(drafts) < self.cap
        if not drafts:
            self.singles += 1
        self.q.append(self.feed(pos, [cur] + list(drafts)))

    def poll(self):
        return self.q.popleft()

    def verify(self, pos, cur, drafts):
        return self.feed(pos, [cur] + list(drafts))

    def is_eos(self, t):
        return t == EOS


class TruthDraft:
    def __init__(self, truth, quality):
        self.truth, self.quality, self.calls = truth, quality, 0

    def capacity(self):
        return 1 << 30

    def draft(self, context, gamma):
        self.calls += 1
        ctx, out = list(context), []
        for _ in range(gamma):
            t = self.truth.next(ctx)
            out.append(t)
            ctx.append(t)
        if self.quality == "garbage":
            out = [-(2 ** 31)] * gamma
        elif self.quality == "flaky" and self.calls % 2 == 0:
            out[self.calls % gamma] = 77
        elif self.quality == "eos_at_chunk_end":
            out[-1] = EOS
        elif self.quality == "all_eos":
            out = [EOS] * gamma
        return out


QUALITIES = ["perfect", "garbage", "flaky", "eos_at_chunk_end", "all_eos"]


def test_drivers_equal_greedy_across_the_grid():
    prompt, max_new = [11, 12, 13], 17
    for eos_at in list(range(0, 23)) + [None]:
        truth = Truth(len(prompt), eos_at)
        expected = truth.greedy(prompt, max_new)
        for gamma in range(1, 6):
            cfg = SpecConfig(gamma, max_new)
            for q in QUALITIES:
                out, _ = run_spec_decode(TruthDraft(truth, q), KvPipe(truth), prompt, cfg)
                assert out == expected, ("sync", eos_at, gamma, q)
                for depth in range(1, 7):
                    chain = KvPipe(truth)
                    out, stats = run_spec_decode_pipelined(TruthDraft(truth, q), chain, prompt,
                                                           cfg, depth)
                    assert out == expected, ("pipe", eos_at, gamma, q, depth)
                    assert stats.committed == len(out)
                    assert not chain.q, "driver left chunks in flight"
                    assert chain.used <= len(prompt) + max_new + depth * gamma


def test_unverified_eos_does_not_stop_output():
    class EarlyEos:
        def capacity(self):
            return 1 << 30

        def draft(self, context, gamma):
            d = [-100] * gamma
            d[-1] = EOS
            return d

    truth = Truth(1)
    expected = truth.greedy([100], 10)
    for depth in [1, 2, 4, 8]:
        out, _ = run_spec_decode_pipelined(EarlyEos(), KvPipe(truth), [100], SpecConfig(2, 10),
                                           depth)
        assert out == expected


def test_caps_and_verified_eos():
    truth = Truth(1, eos_at=3)
    for max_new in [0, 1, 2, 10]:
        for depth in [1, 4]:
            chain = KvPipe(truth)
            out, _ = run_spec_decode_pipelined(TruthDraft(truth, "perfect"), chain, [100],
                                               SpecConfig(2, max_new), depth)
            assert out == truth.greedy([100], max_new)
            assert not chain.q


def test_lookahead_stays_within_capacity():
    """Near capacity the pipelined driver drains and advances with single-token steps
    (src/specpipe.rs:99-120); chunks are always 1 or gamma + 1 tokens."""
    truth = Truth(740)
    for depth in [1, 4, 8]:
        chain = KvPipe(truth, capacity=768)
        out, _ = run_spec_decode_pipelined(TruthDraft(truth, "perfect"), chain, [100] * 740,
                                           SpecConfig(7, 28), depth)
        assert out == truth.greedy([100] * 740, 28)
        assert chain.singles > 0


def test_stepwise_driver_matches_the_loop():
    truth = Truth(3)
    a, _ = run_spec_decode_pipelined(TruthDraft(truth, "flaky"), KvPipe(truth), [1, 2, 3],
                                     SpecConfig(3, 20), 3)
    d = PipelinedDriver(TruthDraft(truth, "flaky"), KvPipe(truth), [1, 2, 3], SpecConfig(3, 20), 3)
    d.start()
    steps = 0
    while d.step():
        steps += 1
    assert d.out == a and steps == d.traversals


class _HelloStage:
    """What LocalChain reads from a stage before the first chunk: range, role, hello."""

    def __init__(self, a, b, layers=4, max_seq=768, chunk=8, model="qwen3:4:64:128:64:2:1",
                 taps=()):
        self._r, self._layers = (a, b), layers
        self.first, self.last = a == 0, b == layers
        self._hello = {"model": model, "max_seq": max_seq, "chunk": chunk}
        self._taps = list(taps)

    def range(self):
        return self._r

    def model_layers(self):
        return self._layers

    def chunk_size(self):
        return self._hello["chunk"]

    def tap_layers(self):
        return self._taps

    def hello(self, next_layer):
        return dict(self._hello, next_layer=next_layer, taps=self._taps)


def test_local_chain_handshake():
    """src/transport.rs:299-358 on LocalChain's links: matching stages (with taps on some of
    them) are accepted; a different model, max_seq or chunk on one link, or a chain that stops
    before the model's last layer, is refused with the settings that differ."""
    from potpori_b200.chain import HandshakeError, LocalChain

    LocalChain([_HelloStage(0, 2, taps=[1]), _HelloStage(2, 4)])
    cases = [
        ([_HelloStage(0, 2), _HelloStage(2, 4, model="qwen3:4:64:128:64:4:1")], "model"),
        ([_HelloStage(0, 2), _HelloStage(2, 4, max_seq=512)], "max_seq 768 (this node has 512)"),
        ([_HelloStage(0, 1), _HelloStage(1, 3, chunk=4), _HelloStage(3, 4, chunk=4)],
         "node [1, 3): upstream expects chunk 8 (this node has 4)"),
        ([_HelloStage(0, 2), _HelloStage(2, 3)], "the chain ends at layer 3, but the model has 4"),
    ]
    for stages, words in cases:
        with pytest.raises(HandshakeError) as e:
            LocalChain(stages)
        assert words in str(e.value)
