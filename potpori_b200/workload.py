"""The benchmark and test workloads: Qwen3 targets and drafts with seeded random weights,
seeded prompts, layer splits per GPU count, and the algorithmic byte counts of a verify pass.

Weights come from the counter-based generator of the C ABI (pp_shard_init_random): every
matrix N(0, 0.02) rounded to BF16, norms 1. Prompts are uniform token ids from
numpy.random.default_rng(prompt_seed). No dataset is involved.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

from .config import QWEN3_0_6B, QWEN3_1_7B, QWEN3_4B, QwenConfig


def even_split(layers: int, n: int) -> List[Tuple[int, int]]:
    base, extra = divmod(layers, n)
    out, a = [], 0
    for i in range(n):
        b = a + base + (1 if i < extra else 0)
        out.append((a, b))
        a = b
    return out


@dataclass
class Workload:
    name: str
    target: QwenConfig
    target_seed: int
    draft: Optional[QwenConfig]
    draft_seed: int
    gamma: int
    depth: int
    max_seq: int
    prompt_len: int
    max_new: int
    prompt_seed: int
    splits: Dict[int, List[Tuple[int, int]]] = field(default_factory=dict)
    draft_is_target: bool = False

    def split(self, n_gpus: int) -> List[Tuple[int, int]]:
        return self.splits.get(n_gpus) or even_split(self.target.layers, n_gpus)

    def prompt(self) -> List[int]:
        rng = np.random.default_rng(self.prompt_seed)
        return rng.integers(0, self.target.vocab_size, self.prompt_len).tolist()

    @property
    def chunk(self) -> int:
        return self.gamma + 1


WORKLOADS = {
    # Qwen3-0.6B, seed 0, whole model in one process, the same weights as draft.
    "qwen3-0.6b-selfdraft": Workload("qwen3-0.6b-selfdraft", QWEN3_0_6B, 0, QWEN3_0_6B, 0, 7, 1,
                                     768, 41, 128, 100, {1: [(0, 28)]}, draft_is_target=True),
    # Qwen3-1.7B (seed 1) in 2 shards, Qwen3-0.6B draft.
    "qwen3-1.7b-2stage": Workload("qwen3-1.7b-2stage", QWEN3_1_7B, 1, QWEN3_0_6B, 0, 7, 4, 768,
                                  256, 256, 101, {2: [(0, 14), (14, 28)]}),
    # Qwen3-4B (seed 2) head/middle/tail, Qwen3-0.6B draft.
    "qwen3-4b-3stage": Workload("qwen3-4b-3stage", QWEN3_4B, 2, QWEN3_0_6B, 0, 7, 4, 768, 41,
                                128, 102, {3: [(0, 12), (12, 24), (24, 36)]}),
    # Qwen3-4B (seed 3) as an 8-stage pipeline, 2048-token prompt, and the 1/2/4-GPU even
    # splits of the same model.
    "qwen3-4b-8stage": Workload(
        "qwen3-4b-8stage", QWEN3_4B, 3, QWEN3_0_6B, 0, 7, 8, 4096, 2048, 1024, 103,
        {1: [(0, 36)], 2: [(0, 18), (18, 36)], 4: [(0, 9), (9, 18), (18, 27), (27, 36)],
         8: [(0, 5), (5, 10), (10, 15), (15, 20), (20, 24), (24, 28), (28, 32), (32, 36)]}),
}


def verify_pass_bytes(cfg: QwenConfig, layer_range: Tuple[int, int], m: int, c: int,
                      kv_bytes: int = 4) -> int:
    """Algorithmic HBM bytes of one verify pass of layers [a, b) over m rows with c positions
    visible: every BF16 weight and F32 norm once, the KV rows read (c - m old rows) and
    written (m rows), the hidden rows in and out, the embedding rows on the first shard and
    the vocab matrix, final norm and m picks on the last. Intermediates are not counted."""
    a, b = layer_range
    h, q, kv, i = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.intermediate
    per_layer = (2 * (h * (q + 2 * kv) + q * h + 3 * h * i) + 4 * (2 * h + 2 * cfg.head_dim)
                 + 2 * kv * kv_bytes * (c - m) + 2 * kv * kv_bytes * m)
    total = (b - a) * per_layer
    total += 2 * m * h if a == 0 else 4 * m * h       # embedding rows, or the hidden input
    if b == cfg.layers:
        total += 2 * cfg.vocab_size * h + 4 * h + 4 * m  # vocab matrix, final norm, picks
    else:
        total += 4 * m * h                              # hidden output
    return total


def kernel_bytes(cfg: QwenConfig, kind: str, m: int, c: int, kv_bytes: int = 4) -> int:
    """Algorithmic bytes of one launch of a kernel kind (weights + the activations it must
    read and write once)."""
    h, q, kv, i, v = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.intermediate, cfg.vocab_size
    if kind == "qkv":
        return 2 * h * (q + 2 * kv) + 4 * h + 4 * 2 * cfg.head_dim + 4 * m * h + 4 * m * (q + 2 * kv)
    if kind == "o_proj":
        return 2 * q * h + 4 * m * q + 2 * 4 * m * h
    if kind == "gate_up":
        return 2 * 2 * h * i + 4 * h + 4 * m * h + 4 * m * i
    if kind == "down":
        return 2 * h * i + 4 * m * i + 2 * 4 * m * h
    if kind == "attn":
        return 2 * kv * kv_bytes * c + 2 * 4 * m * q
    if kind == "head":
        return 2 * v * h + 4 * h + 4 * m * h + 4 * m
    return 0
