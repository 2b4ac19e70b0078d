"""A whole model in one shard, and the head's incremental draft engine.

``QwenTarget`` mirrors ``src/qwen/target.rs:15-96`` (prefill in chunk-sized pieces then single
tokens; verify returns the greedy token after every fed token) and ``IncrementalDraft``
mirrors ``src/qwen/draft.rs:14-93`` (feed only what differs from what was fed, then gamma
greedy single-token steps whose tokens stay in the KV). The greedy pick runs on the device;
a non-finite row raises, as the reference's local argmax panics (target.rs:9-13).
"""
from __future__ import annotations

from typing import List

from ._lib import PP_E_NONFINITE, PPError
from .config import QwenConfig, is_eos
from .shard import Shard


class NonFiniteLogits(RuntimeError):
    pass


class QwenTarget:
    def __init__(self, shard: Shard):
        assert shard.first and shard.last, "a target is one shard holding every layer"
        self.shard = shard

    @classmethod
    def random(cls, cfg: QwenConfig, capacity: int, chunk: int = 8, seed: int = 0,
               std: float = 0.02, device: int = 0) -> "QwenTarget":
        return cls(Shard.random(cfg, (0, cfg.layers), capacity, chunk, seed, std, device))

    @classmethod
    def load_chunked(cls, cfg: QwenConfig, path: str, capacity: int, search: int = 0,
                     chunk: int = 8, device: int = 0) -> "QwenTarget":
        return cls(Shard.load_chunked(cfg, (0, cfg.layers), True, True, path, capacity, search,
                                      chunk, device))

    def capacity(self) -> int:
        return self.shard.capacity()

    def reset(self) -> None:
        self.shard.reset()

    def _pick(self, pos: int, tokens: List[int]) -> List[int]:
        r = self.shard.verify_tokens(pos, tokens)
        if not r.finite:
            raise NonFiniteLogits("non-finite or empty logits")
        return r.argmax

    def prefill(self, prompt: List[int], one_pass: bool = True) -> int:
        """The greedy pick after the prompt. The reference feeds the prompt in chunk-sized
        verify steps (target.rs:62-84); a shard that can (Shard.can_prefill) writes the K/V
        rows of all but the last token in one pass per 2048 rows on the tensor cores instead,
        and the last token runs as the 1-row step that yields the pick, the same result to
        the rounding of F32 arithmetic. one_pass=False keeps the chunked steps."""
        if one_pass and len(prompt) > 1 and self.shard.can_prefill():
            self.shard.prefill(0, prompt[:-1])
            return self._pick(len(prompt) - 1, prompt[-1:])[0]
        chunk = self.shard.chunk_size() or len(prompt)
        pos, last = 0, 0
        while pos < len(prompt):
            take = chunk if len(prompt) - pos >= chunk else 1
            last = self._pick(pos, prompt[pos:pos + take])[-1]
            pos += take
        return last

    def verify(self, pos: int, cur: int, drafts: List[int]) -> List[int]:
        return self._pick(pos, [cur] + list(drafts))

    def decode(self, pos: int, cur: int, n: int) -> List[int]:
        """n greedy single-token steps from `cur` at `pos`, each fed the previous pick (on the
        device); the n picks."""
        try:
            return self.shard.decode_greedy(pos, cur, n)
        except PPError as e:
            if e.status == PP_E_NONFINITE:
                raise NonFiniteLogits("non-finite or empty logits") from e
            raise

    def is_eos(self, token: int) -> bool:
        return is_eos(token)


class IncrementalDraft:
    def __init__(self, model: QwenTarget, chunk: int):
        self.model = model
        self.chunk = chunk
        self.fed: List[int] = []
        self.steps = 0  # forward passes issued (for reports)

    def capacity(self) -> int:
        return self.model.capacity()

    def _feed_range(self, ctx: List[int], start: int, end: int) -> int:
        if end - start > self.chunk and self.model.shard.can_prefill():
            # A long catch-up (the prompt): one prefill pass, then the last token's 1-row step.
            self.model.shard.prefill(start, ctx[start:end - 1])
            self.steps += 1
            last = self.model.verify(end - 1, ctx[end - 1], [])[-1]
            self.steps += 1
            return last
        pos, last = start, 0
        while pos < end:
            take = self.chunk if self.chunk > 1 and end - pos >= self.chunk else 1
            piece = ctx[pos:pos + take]
            last = self.model.verify(pos, piece[0], piece[1:])[-1]
            self.steps += 1
            pos += take
        return last

    def draft(self, context: List[int], gamma: int) -> List[int]:
        n = len(context)
        agree = 0
        for a, b in zip(self.fed, context):
            if a != b:
                break
            agree += 1
        start = min(agree, max(n - 1, 0))
        cur = self._feed_range(context, start, n)
        del self.fed[start:]
        self.fed.extend(context[start:n])
        out = [cur]
        if gamma > 1:
            # gamma - 1 greedy single-token steps, each pick fed to the next on the device
            picks = self.model.decode(n, cur, gamma - 1)
            self.fed.extend([cur] + picks[:-1])
            self.steps += gamma - 1
            out.extend(picks)
        return out
