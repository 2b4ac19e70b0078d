"""One-row step of a whole Qwen3-0.6B shard (the draft model's greedy step) on one GPU.

Random BF16 weights (seed 0), a KV cache warmed with `--kv` seeded positions, and the step
at the next position, run by the persistent decode kernel (pp_shard_set_decode_kernel) and,
unless --decode-only, by the per-layer kernels. For each it reports the device time of a
step (graphs replayed back to back, CUDA events on the shard's stream), the host-synchronous
time of verify_tokens, the per-kernel breakdown and the achieved HBM GB/s of the layers
against their algorithmic bytes (every layer weight and norm once, the KV rows read and
the new row written; the vocabulary head is its own kernel).

    python -m potpori_b200.draft_step [--kv 2048] [--iters 50] [--decode-only] [--json]
"""
from __future__ import annotations

import argparse
import json
import time

from .config import QWEN3_0_6B
from .shard import Shard
from .workload import kernel_bytes, verify_pass_bytes


def layers_bytes(cfg, c: int) -> int:
    """Algorithmic bytes of every layer of a 1-row step at c visible positions."""
    return verify_pass_bytes(cfg, (0, cfg.layers), 1, c) - kernel_bytes(cfg, "head", 1, c)


def time_step(sh: Shard, pos: int, iters: int) -> dict:
    import torch

    for _ in range(3):
        sh.verify_tokens(pos, [5])
    t = time.perf_counter()
    for _ in range(iters):
        sh.verify_tokens(pos, [5])
    host = (time.perf_counter() - t) / iters * 1e3
    st = torch.cuda.ExternalStream(sh.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sh.set_step(pos, 1, [5], stream=sh.stream())
    sh.step_device(1, sh.stream())
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(iters):
        sh.set_step(pos, 1, [5], stream=sh.stream())
        sh.step_device(1, sh.stream())
    e1.record(st)
    torch.cuda.synchronize()
    dev = e0.elapsed_time(e1) / iters
    per = {}
    for kind, ms in sh.profile_kernels(1, 5):
        per.setdefault(kind, []).append(ms)
    kernels = {k: {"launches": len(v), "us_mean": round(sum(v) / len(v) * 1e3, 2)} for k, v in per.items()}
    return {"device_ms": round(dev, 4), "host_sync_ms": round(host, 4), "kernels": kernels,
            "launches": sh.last_launches()}


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--kv", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--decode-only", action="store_true")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    cfg = QWEN3_0_6B
    sh = Shard.random(cfg, (0, cfg.layers), a.kv + 64, 8, seed=0)
    sh.fill_kv(7, a.kv)
    rows = {}
    if not a.decode_only:
        rows["layer_kernels"] = time_step(sh, a.kv, a.iters)
    sh.set_decode_kernel(True)
    rows["decode_kernel"] = time_step(sh, a.kv, a.iters)
    c = a.kv + 1
    lb = layers_bytes(cfg, c)
    for name, r in rows.items():
        us = sum(k["us_mean"] * k["launches"] for kind, k in r["kernels"].items()
                 if kind not in ("head", "begin", "embed"))
        r["layers_us"] = round(us, 1)
        r["layers_bytes"] = lb
        r["layers_gbs"] = round(lb / (us * 1e-6) / 1e9, 1) if us > 0 else None
    sh.close()
    if a.json:
        print(json.dumps(rows))
        return
    for name, r in rows.items():
        print(f"{name}: step {r['device_ms']:.3f} ms on the device, {r['host_sync_ms']:.3f} ms "
              f"host-synchronous, {r['launches']} launches; layers {r['layers_us']:.1f} us "
              f"({r['layers_gbs']} GB/s of {r['layers_bytes'] / 1e6:.1f} MB)")
        print("   ", r["kernels"])


if __name__ == "__main__":
    main()
