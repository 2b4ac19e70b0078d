"""Qwen3 geometry and the chain/workload settings of the verify path.

``QwenConfig`` mirrors ``src/qwen/model.rs:11-68`` (field for field, with the same three
presets); ``EOS_TOKENS`` and ``is_eos`` mirror ``src/qwen/mod.rs:40-45``.
"""
from __future__ import annotations

from dataclasses import dataclass, asdict


@dataclass(frozen=True)
class QwenConfig:
    layers: int
    hidden: int
    intermediate: int
    head_dim: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def kv_groups(self) -> int:
        return self.n_heads // self.n_kv_heads

    def hello_model(self) -> str:
        """The model string a shard announces in its handshake (``src/qwen/shard.rs:89-105``)."""
        return (f"qwen3:{self.layers}:{self.hidden}:{self.intermediate}:{self.head_dim}:"
                f"{self.n_heads}:{self.n_kv_heads}")

    def layer_weight_bytes(self) -> int:
        """BF16 matrix bytes of one decoder layer (QKV, O, gate, up, down)."""
        h, q, kv, i = self.hidden, self.q_dim, self.kv_dim, self.intermediate
        return 2 * (h * (q + 2 * kv) + q * h + 3 * h * i)

    def to_dict(self) -> dict:
        return asdict(self)


QWEN3_0_6B = QwenConfig(28, 1024, 3072, 128, 16, 8, 151936, 1e-6, 1e6)
QWEN3_1_7B = QwenConfig(28, 2048, 6144, 128, 16, 8, 151936, 1e-6, 1e6)
QWEN3_4B = QwenConfig(36, 2560, 9728, 128, 32, 8, 151936, 1e-6, 1e6)
# The tiny model of src/qwen/tiny.rs:140-150.
TINY = QwenConfig(2, 8, 12, 4, 2, 1, 16, 1e-6, 10000.0)

PRESETS = {
    "Qwen/Qwen3-0.6B": QWEN3_0_6B,
    "Qwen/Qwen3-1.7B": QWEN3_1_7B,
    "Qwen/Qwen3-4B": QWEN3_4B,
}

EOS_TOKENS = (151645, 151643)


def is_eos(token: int) -> bool:
    return token in EOS_TOKENS


def config_for(repo: str):
    """``src/qwen/mod.rs:48-55``: exact match only."""
    return PRESETS.get(repo)


def from_hf_dict(d: dict) -> QwenConfig:
    """A QwenConfig from a transformers-style config dict (``cpu_check.rs:42-52`` fields)."""
    theta = d.get("rope_theta")
    if theta is None:
        theta = d.get("rope_parameters", {}).get("rope_theta", 1e6)
    return QwenConfig(
        layers=d["num_hidden_layers"], hidden=d["hidden_size"],
        intermediate=d["intermediate_size"], head_dim=d["head_dim"],
        n_heads=d["num_attention_heads"], n_kv_heads=d["num_key_value_heads"],
        vocab_size=d["vocab_size"], rms_norm_eps=d.get("rms_norm_eps", 1e-6),
        rope_theta=float(theta),
    )
