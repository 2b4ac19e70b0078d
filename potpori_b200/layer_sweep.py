"""Single Qwen3-4B decoder layer verify-kernel sweep.

One Qwen3-4B decoder layer (random BF16 weights, seed 4) as a middle shard: F32 hidden rows
~N(0,1) in, hidden rows out. For every KV length in {128, 512, 2048, 4096} (the cache filled
with seeded random K/V) and chunk width M in {1, 4, 8, 16} it runs a few verify steps, each
appending M positions and rolling back a random 0..M-1 rejected suffix, then times every
kernel of the step (graph replay, event per kernel) and reports latency and achieved HBM
GB/s against the algorithmic bytes of that kernel. The tail (final norm + vocab projection
+ argmax over 151936 rows at hidden 2560) is timed the same way on a last-layer shard.

    python bench.py --probe layer-sweep [--kv 128 512 2048 4096] [--m 1 4 8 16] [--json]
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np

from .config import QWEN3_4B
from .shard import Shard
from .workload import kernel_bytes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def sweep(kv_lens, ms, steps=3, iters=5, device=0, seed=4, tail=True):
    cfg = QWEN3_4B
    cap = max(kv_lens) + 64
    peak, src = hbm_peak()
    rows = []
    layer = Shard.random(cfg, (4, 5), cap, 0, seed=seed, device=device)
    rng = np.random.default_rng(seed)
    for kv in kv_lens:
        for m in ms:
            layer.fill_kv(seed + kv, kv)
            pos = kv
            for _ in range(steps):
                h = rng.standard_normal((m, cfg.hidden)).astype(np.float32)
                layer.forward_hidden(pos, m, h)
                pos += m - int(rng.integers(0, m)) if m > 1 else 1
            prof = layer.profile_kernels(m, iters)
            c = pos + m
            for kind, ms_ in prof:
                if kind in ("begin",):
                    continue
                b = kernel_bytes(cfg, kind, m, c)
                gbs = b / (ms_ / 1e3) / 1e9 if (b and ms_ > 0) else None
                rows.append({"kv": kv, "m": m, "kernel": kind, "us": round(ms_ * 1e3, 2),
                             "bytes": b, "gbs": round(gbs, 1) if gbs else None,
                             "frac": round(gbs / peak, 4) if gbs else None})
    layer.close()
    if tail:
        head = Shard.random(cfg, (35, 36), 64, 0, seed=seed, device=device)
        for m in ms:
            h = rng.standard_normal((m, cfg.hidden)).astype(np.float32)
            head.verify_hidden(0, h)
            for kind, ms_ in head.profile_kernels(m, iters):
                if kind != "head":
                    continue
                b = kernel_bytes(cfg, kind, m, m)
                gbs = b / (ms_ / 1e3) / 1e9 if ms_ > 0 else None
                rows.append({"kv": 0, "m": m, "kernel": "head(vocab+argmax)",
                             "us": round(ms_ * 1e3, 2), "bytes": b,
                             "gbs": round(gbs, 1) if gbs else None,
                             "frac": round(gbs / peak, 4) if gbs else None})
        head.close()
    return rows, peak, src


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--kv", type=int, nargs="+", default=[128, 512, 2048, 4096])
    ap.add_argument("--m", type=int, nargs="+", default=[1, 4, 8, 16])
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--no-tail", action="store_true")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    rows, peak, src = sweep(a.kv, a.m, a.steps, a.iters, tail=not a.no_tail)
    if a.json:
        for r in rows:
            print(json.dumps(r))
        return
    print(f"HBM peak {peak:.0f} GB/s ({src})")
    print(f"{'kv':>5} {'m':>2} {'kernel':<20} {'us':>9} {'MB':>8} {'GB/s':>8} {'frac':>6}")
    for r in rows:
        print(f"{r['kv']:>5} {r['m']:>2} {r['kernel']:<20} {r['us']:>9.2f} "
              f"{r['bytes'] / 1e6:>8.2f} {r['gbs'] or 0:>8.1f} {r['frac'] or 0:>6.3f}")


if __name__ == "__main__":
    main()
