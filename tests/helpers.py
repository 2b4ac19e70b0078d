"""Test-side helpers: the reference's tiny generated model and fixture loading."""
from __future__ import annotations

import json
import os

import numpy as np

from potpori_b200.config import QwenConfig, TINY

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

LAYER_PARAMS = [
    ("input_layernorm", True), ("self_attn.q_proj", False), ("self_attn.k_proj", False),
    ("self_attn.v_proj", False), ("self_attn.o_proj", False), ("self_attn.q_norm", True),
    ("self_attn.k_norm", True), ("post_attention_layernorm", True), ("mlp.gate_proj", False),
    ("mlp.up_proj", False), ("mlp.down_proj", False),
]


def param_shapes(cfg: QwenConfig) -> list:
    """Parameters of a whole-model graph in QwenGraph::build order (src/qwen/model.rs:231-319)."""
    H, Q, KV, I = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.intermediate
    shapes = {
        "input_layernorm": (H,), "self_attn.q_proj": (Q, H), "self_attn.k_proj": (KV, H),
        "self_attn.v_proj": (KV, H), "self_attn.o_proj": (H, Q), "self_attn.q_norm": (cfg.head_dim,),
        "self_attn.k_norm": (cfg.head_dim,), "post_attention_layernorm": (H,),
        "mlp.gate_proj": (I, H), "mlp.up_proj": (I, H), "mlp.down_proj": (H, I),
    }
    out = [("model.embed_tokens.weight", (cfg.vocab_size, H))]
    for layer in range(cfg.layers):
        for name, _ in LAYER_PARAMS:
            out.append((f"model.layers.{layer}.{name}.weight", shapes[name]))
    out.append(("model.norm.weight", (H,)))
    return out


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def tiny_weights(cfg: QwenConfig = TINY) -> dict:
    """The deterministic tiny model of src/qwen/tiny.rs:152-179: parameter number `seed` in
    graph order gets sin((i + 13 seed) * 0.37) * 0.1 (BF16), norms 1 (F32)."""
    out = {}
    for seed, (name, shape) in enumerate(param_shapes(cfg)):
        n = int(np.prod(shape))
        if "norm" in name:
            out[name] = np.ones(n, np.float32)
        else:
            i = np.arange(n, dtype=np.int64) + seed * 13
            v = (np.sin(i.astype(np.float32) * np.float32(0.37)) * np.float32(0.1)).astype(np.float32)
            out[name] = f32_to_bf16_bits(v)
    return out


def load_fixture():
    """The reference's dspark_tiny golden vectors (see tests/golden/make_golden.py)."""
    import torch
    from safetensors.torch import load_file
    from potpori_b200.config import from_hf_dict

    with open(os.path.join(GOLDEN, "dspark_tiny.json")) as f:
        meta = json.load(f)
    cfg = from_hf_dict(meta["target"])
    raw = load_file(os.path.join(GOLDEN, "dspark_tiny_target.safetensors"))
    weights = {}
    for k, t in raw.items():
        if t.dtype == torch.bfloat16:
            weights[k] = t.view(torch.int16).numpy().view(np.uint16).reshape(-1).copy()
        else:
            weights[k] = t.float().numpy().reshape(-1).copy()
    exp = load_file(os.path.join(GOLDEN, "dspark_tiny_expected.safetensors"))
    return cfg, meta, weights, exp["target_logits"].numpy(), exp["features"].numpy()


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def tile_weights(w: np.ndarray) -> np.ndarray:
    """W [n][k] BF16 bits in the shards' tiled layout: blocks of 128 rows x 64 columns, tile
    major, the 16-byte unit u of row r of a block at u ^ (r % 8); padding zero."""
    n, k = w.shape
    kc, tiles = -(-k // 64), -(-n // 128)
    out = np.zeros(tiles * kc * 128 * 64, np.uint16)
    j = np.arange(n, dtype=np.int64)[:, None]
    c = np.arange(k, dtype=np.int64)[None, :]
    off = ((((j // 128) * kc + c // 64) * 128 + j % 128) * 64) + ((((c % 64) // 8) ^ (j % 8)) * 8) + c % 8
    out[off] = w
    return out


def random_weights(cfg: QwenConfig, seed: int, std: float = 0.02) -> dict:
    """Every parameter of a whole-model graph: matrices N(0, std) as BF16 bits, norms
    1 + 0.1 N(0, 1) as F32 (numpy's generator, not the shards' seeded one)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in param_shapes(cfg):
        if "norm" in name:
            out[name] = (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
        else:
            out[name] = f32_to_bf16_bits((std * rng.standard_normal(shape)).astype(np.float32))
    return out


def write_prepared(path: str, cfg: QwenConfig, weights: dict, matrix_dtype: str = "bf16") -> None:
    """A prepared weights file in the layout of src/qwen/hf.rs:20,85-91 (the
    model_combined_bf16_v1.safetensors the reference writes): one safetensors file, matrices
    BF16 (or F32 with matrix_dtype="f32", as a checkpoint used as published may store them),
    norms F32, the tied embedding as model.embed_tokens.weight."""
    import torch
    from safetensors.torch import save_file

    shapes = dict(param_shapes(cfg))
    tensors = {}
    for name, value in weights.items():
        shape = shapes[name]
        if "norm" in name:
            tensors[name] = torch.from_numpy(np.asarray(value, np.float32).reshape(shape).copy())
        elif matrix_dtype == "f32":
            tensors[name] = torch.from_numpy(bf16_bits_to_f32(value).reshape(shape).copy())
        else:
            bits = np.asarray(value, np.uint16).reshape(shape).view(np.int16).copy()
            tensors[name] = torch.from_numpy(bits).view(torch.bfloat16)
    save_file(tensors, path)
