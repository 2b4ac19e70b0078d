"""One-pass prompt prefill of a whole Qwen3 shard on one GPU (pp_shard_prefill).

Random BF16 weights (Qwen3-4B seed 3, or Qwen3-0.6B seed 0) and a seeded random prompt of
`--tokens` ids. Reports the host-synchronous time of the K/V pass over all but the last
token (Shard.prefill, after one warm-up call), of the whole QwenTarget.prefill (that pass
plus the 1-row step of the last token, which gives the greedy pick), the same prompt fed in
8-row verify steps as the reference's chunked prefill does (unless --no-chunked), and the
useful F32-product rate of the pass: 2 * rows * layer parameters plus the causal attention's
4 * heads * head_dim * rows * (rows + 1) / 2 per layer.

    python -m potpori_b200.prefill_step [--model 4b|0.6b] [--tokens 2048] [--iters 3] [--no-chunked]
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np

from .config import QWEN3_0_6B, QWEN3_4B
from .target import QwenTarget


def pass_flops(cfg, rows: int) -> float:
    """Useful flops of the K/V pass over `rows` prompt rows from position 0."""
    H, I, hd = cfg.hidden, cfg.intermediate, cfg.head_dim
    q, kv = cfg.n_heads * hd, cfg.n_kv_heads * hd
    params = H * (q + 2 * kv) + q * H + 3 * H * I
    attn = 4.0 * cfg.n_heads * hd * rows * (rows + 1) / 2
    return cfg.layers * (2.0 * rows * params + attn)


def main():
    import torch

    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--model", choices=("4b", "0.6b"), default="4b")
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--no-chunked", action="store_true")
    a = ap.parse_args()
    cfg, seed = (QWEN3_4B, 3) if a.model == "4b" else (QWEN3_0_6B, 0)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, a.tokens).tolist()
    tgt = QwenTarget.random(cfg, max(4096, a.tokens + 16), 8, seed)
    try:
        if not tgt.shard.can_prefill():
            raise SystemExit("this shard cannot run the one-pass prefill")

        def timed(fn):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            out = fn()
            torch.cuda.synchronize()
            return (time.perf_counter() - t0) * 1e3, out

        timed(lambda: tgt.shard.prefill(0, prompt[:-1]))  # warm-up: buffers, graphs
        kv_ms = min(timed(lambda: tgt.shard.prefill(0, prompt[:-1]))[0] for _ in range(a.iters))
        whole_ms, pick = timed(lambda: tgt.prefill(prompt))
        res = {"model": a.model, "tokens": a.tokens, "kv_pass_ms": round(kv_ms, 2),
               "prefill_ms": round(whole_ms, 2), "pick": pick,
               "useful_tflops": round(pass_flops(cfg, a.tokens - 1) / kv_ms / 1e9, 1)}
        if not a.no_chunked:
            chunk_ms, pick2 = timed(lambda: tgt.prefill(prompt, one_pass=False))
            res.update({"chunked_ms": round(chunk_ms, 2), "chunked_pick": pick2})
        print(json.dumps(res))
    finally:
        tgt.shard.close()


if __name__ == "__main__":
    main()
