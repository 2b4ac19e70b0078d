"""The allocation-free RMSNorm + GEMV entry point against the shard path.

pp_norm_gemv_static exists for callers that cannot allocate device memory (a host framework
or memory pool that owns every allocation, or a context where cudaMalloc/cudaFree are not
allowed); it keeps its scratch in a static device array. Here it must reproduce the vocab
projection of a last shard, through the C ABI, on two calls in a row: the shard's one layer
has all-zero matrices, so its output is its input and the shard's logits are exactly
RMSNorm(x, model.norm) . embed^T, computed by the existing entry point
(pp_shard_forward_hidden with logits requested). A ragged case (3 rows, k = 200, which
pads to a fourth 64-column chunk) is checked against a float64 RMSNorm . W^T, and a
non-finite input must set the caller's error word. This file sorts last so that a run that
stops at the first failure has run every other test first.
"""
import ctypes

import numpy as np
import pytest

from helpers import f32_to_bf16_bits, rel_l2
from potpori_b200 import _lib
from potpori_b200.config import QwenConfig
from potpori_b200.shard import Shard

pytestmark = pytest.mark.gpu


def tile_bf16(w: np.ndarray) -> np.ndarray:
    """W [n][k] BF16 bits in the tiled layout documented for pp_norm_gemv_static."""
    n, k = w.shape
    kc, tiles = -(-k // 64), -(-n // 128)
    out = np.zeros(tiles * kc * 128 * 64, np.uint16)
    j = np.arange(n, dtype=np.int64)[:, None]
    c = np.arange(k, dtype=np.int64)[None, :]
    off = ((((j // 128) * kc + c // 64) * 128 + j % 128) * 64) + ((((c % 64) // 8) ^ (j % 8)) * 8) + c % 8
    out[off] = w
    return out


def test_norm_gemv_static_matches_the_shard_head(gpu):
    import torch

    cfg = QwenConfig(layers=2, hidden=256, intermediate=512, head_dim=128, n_heads=2,
                     n_kv_heads=1, vocab_size=1000, rms_norm_eps=1e-6, rope_theta=1e6)
    rng = np.random.default_rng(5)
    embed = f32_to_bf16_bits((0.05 * rng.standard_normal((cfg.vocab_size, cfg.hidden)))
                             .astype(np.float32))
    fnorm = (1 + 0.3 * rng.standard_normal(cfg.hidden)).astype(np.float32)
    shard = Shard(cfg, (1, 2), capacity=16, chunk=8)
    shapes = {"self_attn.q_proj": (cfg.q_dim, cfg.hidden), "self_attn.k_proj": (cfg.kv_dim, cfg.hidden),
              "self_attn.v_proj": (cfg.kv_dim, cfg.hidden), "self_attn.o_proj": (cfg.hidden, cfg.q_dim),
              "mlp.gate_proj": (cfg.intermediate, cfg.hidden), "mlp.up_proj": (cfg.intermediate, cfg.hidden),
              "mlp.down_proj": (cfg.hidden, cfg.intermediate)}
    for name, shape in shapes.items():
        shard.set_tensor(f"model.layers.1.{name}.weight", np.zeros(shape, np.uint16))
    for name, n in [("input_layernorm", cfg.hidden), ("post_attention_layernorm", cfg.hidden),
                    ("self_attn.q_norm", cfg.head_dim), ("self_attn.k_norm", cfg.head_dim)]:
        shard.set_tensor(f"model.layers.1.{name}.weight", np.ones(n, np.float32))
    shard.set_tensor("model.embed_tokens.weight", embed.reshape(-1))
    shard.set_tensor("model.norm.weight", fnorm)
    assert not shard.missing()

    m = 8
    x = rng.standard_normal((m, cfg.hidden)).astype(np.float32)
    want = shard.verify_hidden(0, x, logits=True).logits  # the existing entry point
    assert np.isfinite(want).all()

    L = _lib.load()
    dev = torch.device("cuda", 0)
    w_t = torch.from_numpy(tile_bf16(embed).view(np.int16)).to(dev)
    x_t = torch.from_numpy(x).to(dev)
    n_t = torch.from_numpy(fnorm).to(dev)
    y_t = torch.empty((m, cfg.vocab_size), dtype=torch.float32, device=dev)
    err_t = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        y_t.fill_(float("nan"))
        st = L.pp_norm_gemv_static(w_t.data_ptr(), x_t.data_ptr(), n_t.data_ptr(),
                                   ctypes.c_float(cfg.rms_norm_eps), cfg.vocab_size, cfg.hidden,
                                   m, y_t.data_ptr(), err_t.data_ptr(), ctypes.c_void_p(stream))
        assert st == _lib.PP_OK, _lib.last_error(None)
        torch.cuda.synchronize(dev)
        got = y_t.cpu().numpy()
        assert int(err_t.item()) == 0, f"call {call}: status {int(err_t.item())}"
        assert np.isfinite(got).all(), f"call {call}"
        assert rel_l2(got, want) <= 1e-3, f"call {call}"
        assert np.abs(got - want).max() <= 1e-4, f"call {call}"

    # A ragged case: 3 of the 8 rows, k = 200 (a padded fourth 64-column chunk), 1000 outputs
    # (a partial 128-row tile), against float64 RMSNorm(x) . W^T.
    n2, k2, m2 = 1000, 200, 3
    w2 = f32_to_bf16_bits((0.05 * rng.standard_normal((n2, k2))).astype(np.float32))
    x2 = rng.standard_normal((m2, k2)).astype(np.float32)
    g2 = (1 + 0.3 * rng.standard_normal(k2)).astype(np.float32)
    w64 = (w2.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    x64 = x2.astype(np.float64)
    xn = x64 / np.sqrt((x64 * x64).mean(axis=1, keepdims=True) + 1e-6) * g2.astype(np.float64)
    want2 = xn @ w64.T
    w2_t = torch.from_numpy(tile_bf16(w2).view(np.int16)).to(dev)
    x2_t = torch.from_numpy(x2).to(dev)
    g2_t = torch.from_numpy(g2).to(dev)
    y2_t = torch.full((m2, n2), float("nan"), dtype=torch.float32, device=dev)
    st = L.pp_norm_gemv_static(w2_t.data_ptr(), x2_t.data_ptr(), g2_t.data_ptr(),
                               ctypes.c_float(1e-6), n2, k2, m2, y2_t.data_ptr(),
                               err_t.data_ptr(), ctypes.c_void_p(stream))
    assert st == _lib.PP_OK, _lib.last_error(None)
    torch.cuda.synchronize(dev)
    got2 = y2_t.cpu().numpy()
    assert int(err_t.item()) == 0
    assert rel_l2(got2, want2) <= 5e-5

    # A non-finite input value is reported in the error word (status bit 2).
    x2_t[1, 17] = float("inf")
    st = L.pp_norm_gemv_static(w2_t.data_ptr(), x2_t.data_ptr(), g2_t.data_ptr(),
                               ctypes.c_float(1e-6), n2, k2, m2, y2_t.data_ptr(),
                               err_t.data_ptr(), ctypes.c_void_p(stream))
    assert st == _lib.PP_OK
    torch.cuda.synchronize(dev)
    assert int(err_t.item()) & 2

    # Sizes past the static scratch are refused with a clear error.
    st = L.pp_norm_gemv_static(w_t.data_ptr(), x_t.data_ptr(), n_t.data_ptr(),
                               ctypes.c_float(1e-6), cfg.vocab_size, cfg.hidden, 9,
                               y_t.data_ptr(), None, None)
    assert st == _lib.PP_E_INVALID and "8" in _lib.last_error(None)
