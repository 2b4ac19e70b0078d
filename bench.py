#!/usr/bin/env python3
"""Benchmark: Qwen3-4B greedy speculative decoding on B200 through the sm_100a verify pass.

Workload (default ``qwen3-4b-8stage``): Qwen3-4B target with seeded random BF16 weights
(seed 3), Qwen3-0.6B draft (seed 0), gamma 7 (verify chunks of 8 rows), the depth-8
pipelined driver of src/specpipe.rs, KV capacity 4096, a 2048-token seeded random prompt.
With N GPUs the target is split into N contiguous layer ranges (1: 0-36, 2: 18+18, 4: 9x4,
8: 5,5,5,5,4,4,4,4), one process per GPU, stages joined by CUDA IPC copies on the copy
engines with mailboxes in shared host memory; rank 0 also runs the draft model and the
driver.

A step is the run of driver iterations — FILL (draft and submit chunks until `depth` are in
flight) and READ (take the oldest chunk's verified picks; commit, or drain a stale chunk) —
that ends when the committed prefix grows, so every step commits at least one token. With
the random draft and target the drafts are never accepted: a step commits one token and
costs eight traversals (one verified, seven drained) and 56 draft forwards.
value = committed tokens of the K timed steps / their device time (CUDA events on the stage
streams, max over ranks); the
weights (8.3 GB per verify pass) are far larger than L2, so no flush is needed between steps.
e2e = committed tokens of the same K steps / their host wall time through the public API
(every step's header uploads from pinned memory and result reads inside); the whole session
from the prompt upload and prefill on is reported beside it as e2e.session.

``--impl reference`` times the CPU restatement of the reference math (the reference is Rust
with an unvendored dependency and cannot be built here) on the same workload, using all
host threads, over a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "Qwen3-4B committed tok/s at 1/2/4/8 B200; verify-pass HBM GB/s vs peak"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="qwen3-4b-8stage")
    ap.add_argument("--cpu-budget", type=float, default=20.0,
                    help="seconds of CPU work for the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-profile", action="store_true")
    ap.add_argument("--draft-kernel", default="decode", choices=["decode", "layers"],
                    help="1-row draft steps: one persistent decode kernel, or six kernels per "
                         "layer")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "of measured"
    except Exception:
        return FALLBACK_HBM_GBS, "of fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)], stdout=self.file,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax.append(float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.file.name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# --------------------------------------------------------------------------- shared parts
def workload_config(wl) -> dict:
    """The `config` object of the JSON line, identical in both arms."""
    return {
        "workload": wl.name,
        "target": f"Qwen3-4B (36 layers, random BF16 weights, seed {wl.target_seed})",
        "draft": f"Qwen3-0.6B (28 layers, random BF16 weights, seed {wl.draft_seed})",
        "gamma": wl.gamma, "depth": wl.depth, "max_seq": wl.max_seq,
        "prompt_len": wl.prompt_len, "global_batch": 1,
        "step": "driver iterations (FILL + READ, src/specpipe.rs:87-183) until the committed "
                "prefix grows",
        "weights": "bf16 storage, f32 arithmetic",
        "l2": "no flush: 8.3 GB of target weights streamed per verify pass, far above the "
              "126 MB L2",
    }


def advance(drv):
    """One timed step: driver iterations until the committed prefix grows (or generation
    ends). Returns (iterations, whether generation continues)."""
    n0, it = len(drv.out), 0
    while len(drv.out) == n0:
        if not drv.step():
            return it, False
        it += 1
    return it, True


def stream_hash(tokens) -> str:
    import hashlib
    return hashlib.sha256(",".join(str(int(t)) for t in tokens).encode()).hexdigest()[:16]


# ------------------------------------------------------------------------------------ CPU
def cpu_sample(wl, budget_s: float, max_steps=None, warmup=0):
    """The oracle (CPU restatement of the reference math, all host threads) running the same
    driver on the same models. Bounded sample: both caches hold prompt_len - 1 seeded
    positions (the prompt's prefill would take minutes on the CPU), the last prompt token is
    fed, then `warmup` untimed steps, then timed steps (each: driver iterations until the
    committed prefix grows) until `max_steps` or `budget_s` has passed."""
    import oracle
    from oracle.engines import OracleChain, OracleDraft
    from potpori_b200.specdecode import SpecConfig
    from potpori_b200.specpipe import PipelinedDriver

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    oracle.set_threads(cores)
    tcfg, dcfg = wl.target, wl.draft
    tgt = oracle.OracleShard(tcfg, 0, tcfg.layers, wl.max_seq, wl.chunk)
    tgt.init_random(wl.target_seed)
    dm = oracle.OracleShard(dcfg, 0, dcfg.layers, wl.max_seq, wl.chunk)
    dm.init_random(wl.draft_seed)
    prompt = wl.prompt()
    warm = len(prompt) - 1
    tgt.fill_kv(11, warm)
    dm.fill_kv(12, warm)
    chain = OracleChain([tgt], wl.chunk)
    draft = OracleDraft(dm, wl.chunk)
    draft.fed = list(prompt[:warm])
    chain.prefill = lambda p: chain._run(warm, [p[warm]])[-1]
    drv = PipelinedDriver(draft, chain, prompt, SpecConfig(wl.gamma, wl.max_new), wl.depth)
    drv.start()
    for _ in range(warmup):
        if not advance(drv)[1]:
            break
    base, f0, d0 = len(drv.out), chain.forwards, draft.forwards
    t0 = time.perf_counter()
    steps = iters = 0
    while max_steps is None or steps < max_steps:
        it, more = advance(drv)
        iters += it
        if len(drv.out) > base + steps:
            steps += 1
        if not more or time.perf_counter() - t0 >= budget_s:
            break
    el = time.perf_counter() - t0
    committed = len(drv.out) - base
    sample = (f"{steps} steps ({iters} driver iterations, {chain.forwards - f0} target verify "
              f"passes, {draft.forwards - d0} draft forwards) from position {warm} over a "
              f"seeded warm cache after {warmup} warm-up steps, {el:.1f} s")
    return {"value": committed / el if el > 0 else 0.0, "unit": "tok/s", "cores": cores,
            "kind": "port", "sample": sample, "committed": committed, "seconds": el,
            "steps": steps}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from potpori_b200.workload import WORKLOADS
    wl = WORKLOADS[args.workload]
    # One CPU step is eight 4B verify passes and 56 0.6B draft forwards (seconds each), so the
    # warm-up is capped at one step and the timed steps at PP_REF_BUDGET seconds.
    warmup = min(args.warmup, 1)
    res = cpu_sample(wl, float(os.environ.get("PP_REF_BUDGET", 60.0)), max_steps=args.steps,
                     warmup=warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": "tok/s",
        "n_gpus": args.gpus, "steps": res["steps"], "warmup": warmup,
        "ms_per_step": 1000.0 * res["seconds"] / max(res["steps"], 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(wl),
        "cpu_baseline": {"value": res["value"], "unit": "tok/s", "cores": res["cores"],
                         "kind": "port", "sample": res["sample"]},
        "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------ GPU
def run_ours(args):
    import torch

    from potpori_b200.chain import LocalChain
    from potpori_b200.shard import Shard
    from potpori_b200.specdecode import SpecConfig
    from potpori_b200.specpipe import PipelinedDriver
    from potpori_b200.target import IncrementalDraft, QwenTarget
    from potpori_b200.workload import WORKLOADS, kernel_bytes, verify_pass_bytes

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    wl = WORKLOADS[args.workload]
    ranges = wl.split(world)
    if world > 1:
        import datetime

        import torch.distributed as dist
        # NCCL carries the setup and the final timing reduction only; the stages' chunks move
        # by CUDA IPC copies on the copy engines (potpori_b200/distchain.py).
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    stage = Shard.random(wl.target, ranges[rank], wl.max_seq, wl.chunk, wl.target_seed,
                         device=local)
    width = wl.chunk
    if world > 1:
        dist.barrier()
    if rank != 0:
        from potpori_b200.distchain import run_stage
        ms = run_stage(stage, rank, world, width)
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        torch.cuda.synchronize()
        stage.close()  # before the process group and the CUDA runtime are torn down
        dist.destroy_process_group()
        return

    dmodel = QwenTarget(stage) if wl.draft_is_target and world == 1 else \
        QwenTarget.random(wl.draft, wl.max_seq, wl.chunk, wl.draft_seed, device=local)
    if args.draft_kernel == "decode":
        dmodel.shard.set_decode_kernel(True)
    draft = IncrementalDraft(dmodel, wl.chunk)
    if world == 1:
        chain = LocalChain([stage])
    else:
        from potpori_b200.distchain import FLAG_WINDOW_END, FLAG_WINDOW_START, DistChain
        chain = DistChain(stage, world, width)
    prompt = wl.prompt()
    drv = PipelinedDriver(draft, chain, prompt, SpecConfig(wl.gamma, wl.max_new), wl.depth)
    stream = torch.cuda.ExternalStream(stage.stream())

    t_e2e = time.perf_counter()
    drv.start()
    for _ in range(args.warmup):
        if not advance(drv)[1]:
            break
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0, s0, d0 = len(drv.out), chain.submitted, draft.steps
    if world > 1:
        chain.mark(FLAG_WINDOW_START)
    t0 = time.perf_counter()
    ev0.record(stream)
    steps = iters = 0
    for _ in range(args.steps):
        it, more = advance(drv)
        iters += it
        if not more:
            break
        steps += 1
    ev1.record(stream)
    if world > 1:
        chain.mark(FLAG_WINDOW_END)
        chain.send_marks()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    clocks = sampler.stop()
    e2e_s = t1 - t0
    session_s = t1 - t_e2e
    committed = len(drv.out) - c0
    chunks = chain.submitted - s0
    dsteps = draft.steps - d0
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        chain.stop()
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = committed / (ms / 1000.0) if ms > 0 else 0.0

    # ---- kernel- and pass-level roofline on this rank's stage (after the timed region) ----
    peak, peak_src = peaks()
    cfg = wl.target
    c_now = min(drv.send_pos + width, wl.max_seq)
    roofline, kernels, vpass = None, {}, None
    if not args.no_profile:
        prof = stage.profile_kernels(width, iters=3)
        per_kind = {}
        for kind, t in prof:
            per_kind.setdefault(kind, []).append(t)
        total = sum(t for _, t in prof)
        for kind, ts in per_kind.items():
            b = kernel_bytes(cfg, kind, width, c_now)
            kernels[kind] = {"launches": len(ts), "ms_total": round(sum(ts), 4),
                             "ms_mean": round(sum(ts) / len(ts), 5),
                             "share": round(sum(ts) / total, 4),
                             "gbs": round(b / (sum(ts) / len(ts)) / 1e6, 1) if b else None}
        dom = max(per_kind, key=lambda k: sum(per_kind[k]))
        dmean = sum(per_kind[dom]) / len(per_kind[dom])
        dbytes = kernel_bytes(cfg, dom, width, c_now)
        ach = dbytes / (dmean / 1000.0) / 1e9
        traffic = None
        tfile = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tfile):
            with open(tfile) as f:
                traffic = json.load(f).get(f"{wl.name}:{dom}")
        roofline = {"bound": "hbm", "kernel": dom, "achieved": round(ach, 1), "peak": peak,
                    "unit": "GB/s", "frac": round(ach / peak, 4), "peak_source": peak_src,
                    "bytes_per_launch": dbytes, "ms_per_launch": round(dmean, 5),
                    "traffic": traffic}
        # The whole verify pass of this stage, graph replayed back to back.
        reps = 20
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stage.step_device(width)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            stage.step_device(width)
        e1.record(stream)
        torch.cuda.synchronize()
        vms = e0.elapsed_time(e1) / reps
        vb = verify_pass_bytes(cfg, ranges[0], width, c_now)
        vpass = {"layers": list(ranges[0]), "rows": width, "context": c_now,
                 "ms": round(vms, 4), "bytes": vb, "gbs": round(vb / (vms / 1000) / 1e9, 1),
                 "frac": round(vb / (vms / 1000) / 1e9 / peak, 4), "peak_source": peak_src}

    hdr, res_b = 144, 208
    per_chunk_h2d = hdr + (0 if world == 1 else 0)
    h2d = (chunks * per_chunk_h2d + dsteps * hdr) / max(steps, 1)
    d2h = ((chunks + dsteps) * res_b) / max(steps, 1)
    launches = chunks * stage.last_launches() + dsteps * dmodel.shard.last_launches()

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_sample(wl, args.cpu_budget)
            cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as e:  # the CPU baseline must not sink the GPU measurement
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "port",
                   "sample": f"failed: {e}"}

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms / max(steps, 1), 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(wl),
        "setup": {
            "layers_per_gpu": ranges, "sm_budget": stage.sm_limit(),
            "draft_sm_budget": dmodel.shard.sm_limit(),
            "draft_step": ("one persistent decode kernel + vocab head" if dmodel.shard.decode_kernel()
                           else "per-layer kernels"),
        },
        "committed_tokens": committed, "driver_iterations": iters, "traversals": chunks,
        "draft_forwards": dsteps,
        "stream": {"tokens": len(drv.out), "sha256_16": stream_hash(drv.out),
                   "scope": "every committed token from the first pick after the prompt"},
        "tokens_per_traversal": round(committed / max(chunks, 1), 4),
        "roofline": roofline, "verify_pass": vpass, "kernels": kernels,
        "cpu_baseline": cpu,
        "e2e": {"value": round(committed / e2e_s, 3) if e2e_s > 0 else 0.0, "unit": "tok/s",
                "h2d_bytes_per_step": round(h2d, 1), "d2h_bytes_per_step": round(d2h, 1),
                "scope": "the timed steps, host wall clock through the driver's public calls",
                "seconds": round(e2e_s, 3),
                "session": {"value": round(len(drv.out) / session_s, 3), "tokens": len(drv.out),
                            "seconds": round(session_s, 3),
                            "scope": "prompt upload + prefill + warmup + timed steps"}},
        "gpu_launches": launches, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
    # Release the shards explicitly, before the process group and the CUDA runtime are torn
    # down (destructors that run at interpreter exit may find them gone).
    torch.cuda.synchronize()
    del drv, draft, chain
    dmodel.shard.close()
    stage.close()
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- kernel probes
# `python bench.py --probe NAME [options]` times one piece of the path on one GPU; the
# profiles/ summaries name these commands.

def _probe_draft_step(argv):
    """One-row step of a whole Qwen3-0.6B shard (the draft model's greedy step) on one GPU.

    Random BF16 weights (seed 0), a KV cache warmed with `--kv` seeded positions, and the step
    at the next position, run by the persistent decode kernel (pp_shard_set_decode_kernel)
    and, unless --decode-only, by the per-layer kernels. For each it reports the device time
    of a step (graphs replayed back to back, CUDA events on the shard's stream), the
    host-synchronous time of verify_tokens, the per-kernel breakdown and the achieved HBM GB/s
    of the layers against their algorithmic bytes (every layer weight and norm once, the KV
    rows read and the new row written; the vocabulary head is its own kernel)."""
    import torch

    from potpori_b200.config import QWEN3_0_6B
    from potpori_b200.shard import Shard
    from potpori_b200.workload import kernel_bytes, verify_pass_bytes

    ap = argparse.ArgumentParser(prog="bench.py --probe draft-step")
    ap.add_argument("--kv", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--decode-only", action="store_true")
    a = ap.parse_args(argv)

    def time_step(sh, pos, iters):
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
        kernels = {k: {"launches": len(v), "us_mean": round(sum(v) / len(v) * 1e3, 2)}
                   for k, v in per.items()}
        return {"device_ms": round(dev, 4), "host_sync_ms": round(host, 4), "kernels": kernels,
                "launches": sh.last_launches()}

    cfg = QWEN3_0_6B
    sh = Shard.random(cfg, (0, cfg.layers), a.kv + 64, 8, seed=0)
    sh.fill_kv(7, a.kv)
    rows = {}
    if not a.decode_only:
        rows["layer_kernels"] = time_step(sh, a.kv, a.iters)
    sh.set_decode_kernel(True)
    rows["decode_kernel"] = time_step(sh, a.kv, a.iters)
    c = a.kv + 1
    lb = verify_pass_bytes(cfg, (0, cfg.layers), 1, c) - kernel_bytes(cfg, "head", 1, c)
    for r in rows.values():
        us = sum(k["us_mean"] * k["launches"] for kind, k in r["kernels"].items()
                 if kind not in ("head", "begin", "embed"))
        r["layers_us"] = round(us, 1)
        r["layers_bytes"] = lb
        r["layers_gbs"] = round(lb / (us * 1e-6) / 1e9, 1) if us > 0 else None
    sh.close()
    print(json.dumps(rows))


def _probe_prefill_step(argv):
    """One-pass prompt prefill of a whole Qwen3 shard on one GPU (pp_shard_prefill).

    Random BF16 weights (Qwen3-4B seed 3, or Qwen3-0.6B seed 0) and a seeded random prompt of
    `--tokens` ids. Reports the host-synchronous time of the K/V pass over all but the last
    token (after one warm-up call), of the whole QwenTarget.prefill (that pass plus the 1-row
    step of the last token, which gives the greedy pick), the same prompt fed in 8-row verify
    steps as the reference's chunked prefill does (unless --no-chunked), and the useful
    F32-product rate of the pass: 2 * rows * layer parameters plus the causal attention's
    4 * heads * head_dim * rows * (rows + 1) / 2 per layer."""
    import numpy as np
    import torch

    from potpori_b200.config import QWEN3_0_6B, QWEN3_4B
    from potpori_b200.target import QwenTarget

    ap = argparse.ArgumentParser(prog="bench.py --probe prefill-step")
    ap.add_argument("--model", choices=("4b", "0.6b"), default="4b")
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--no-chunked", action="store_true")
    a = ap.parse_args(argv)
    cfg, seed = (QWEN3_4B, 3) if a.model == "4b" else (QWEN3_0_6B, 0)

    def pass_flops(rows):
        H, I, hd = cfg.hidden, cfg.intermediate, cfg.head_dim
        q, kv = cfg.n_heads * hd, cfg.n_kv_heads * hd
        params = H * (q + 2 * kv) + q * H + 3 * H * I
        attn = 4.0 * cfg.n_heads * hd * rows * (rows + 1) / 2
        return cfg.layers * (2.0 * rows * params + attn)

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
               "useful_tflops": round(pass_flops(a.tokens - 1) / kv_ms / 1e9, 1)}
        if not a.no_chunked:
            chunk_ms, pick2 = timed(lambda: tgt.prefill(prompt, one_pass=False))
            res.update({"chunked_ms": round(chunk_ms, 2), "chunked_pick": pick2})
        print(json.dumps(res))
    finally:
        tgt.shard.close()


def _probe_prefill_gemm(argv):
    """Rate of the tensor-core prompt projection (pp_rows_gemm) at a prefill shape on one GPU.

    Random BF16 weights [n][k] in the shards' tiled layout and F32 activations [t][k]; each
    call splits the activations into BF16 hi + lo blocks and runs the tcgen05 GEMM. Reports
    the device time per call (CUDA events, after warm-up) and the rate counted two ways:
    useful (2 t n k flops) and issued (both MMAs per K step, W.hi and W.lo). The default shape
    is the Qwen3-4B gate/up projection over a 2048-row prompt chunk."""
    import ctypes

    import numpy as np
    import torch

    from potpori_b200 import _lib

    ap = argparse.ArgumentParser(prog="bench.py --probe prefill-gemm")
    ap.add_argument("--t", type=int, default=2048)
    ap.add_argument("--n", type=int, default=19456)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    L = _lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    tiles, kc = -(-a.n // 128), -(-a.k // 64)
    # Random bit patterns of small BF16 values stand in for a packed weight matrix: the rate
    # does not depend on the values.
    w = (torch.randint(0x3a00, 0x3c80, (tiles * kc * 128 * 64,), generator=g, device=dev,
                       dtype=torch.int32)).to(torch.int16)
    x = torch.randn((a.t, a.k), generator=g, device=dev, dtype=torch.float32)
    y = torch.empty((a.t, a.n), device=dev, dtype=torch.float32)
    wb = int(L.pp_rows_gemm_work_bytes(a.t, a.k))
    work = torch.empty(wb + 1024, dtype=torch.uint8, device=dev)
    base = (work.data_ptr() + 1023) // 1024 * 1024
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def call():
        st = L.pp_rows_gemm(w.data_ptr(), a.n, a.k, x.data_ptr(), a.t, y.data_ptr(),
                            ctypes.c_void_p(base), wb, err.data_ptr(), ctypes.c_void_p(stream))
        if st != _lib.PP_OK:
            raise RuntimeError(_lib.last_error(None))

    for _ in range(3):
        call()
    torch.cuda.synchronize(dev)
    ms = []
    for _ in range(a.iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        call()
        e1.record()
        torch.cuda.synchronize(dev)
        ms.append(e0.elapsed_time(e1))
    if int(err.item()):
        raise RuntimeError("a bounded device wait expired")
    best = float(np.min(ms))
    flops = 2.0 * a.t * a.n * a.k
    print(json.dumps({"t": a.t, "n": a.n, "k": a.k, "ms_best": round(best, 4),
                      "ms_median": round(float(np.median(ms)), 4),
                      "useful_tflops": round(flops / best / 1e9, 1),
                      "issued_tflops": round(2 * flops / best / 1e9, 1)}))


def _probe_verify_pass(argv):
    """One whole verify pass of a Qwen3-4B shard (seed 3, the workload's target) on one GPU:
    chunk rows over a seeded cache of --kv positions, the step graph replayed back to back
    (CUDA events on the shard's stream), against the pass's algorithmic bytes."""
    import torch

    from potpori_b200.config import QWEN3_4B
    from potpori_b200.shard import Shard
    from potpori_b200.workload import verify_pass_bytes

    ap = argparse.ArgumentParser(prog="bench.py --probe verify-pass")
    ap.add_argument("--kv", type=int, default=2048)
    ap.add_argument("--rows", type=int, default=8)
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    cfg = QWEN3_4B
    rng = (0, a.layers)
    sh = Shard.random(cfg, rng, 4096, 8, seed=3)
    sh.fill_kv(11, a.kv)
    toks = list(range(100, 100 + a.rows))
    st = torch.cuda.ExternalStream(sh.stream())
    for _ in range(3):
        sh.set_step(a.kv, a.rows, toks if sh.first else None, stream=sh.stream())
        sh.step_device(a.rows, sh.stream())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(a.iters):
        sh.step_device(a.rows, sh.stream())
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    b = verify_pass_bytes(cfg, rng, a.rows, a.kv + a.rows)
    peak, src = peaks()
    print(json.dumps({"layers": list(rng), "rows": a.rows, "kv": a.kv, "ms": round(ms, 4),
                      "bytes": b, "gbs": round(b / ms / 1e6, 1),
                      "frac": round(b / ms / 1e6 / peak, 4), "peak_source": src}))
    sh.close()


def _probe_layer_sweep(argv):
    """Config 4's single Qwen3-4B layer sweep (potpori_b200.layer_sweep)."""
    from potpori_b200 import layer_sweep
    layer_sweep.main(argv)


PROBES = {"draft-step": _probe_draft_step, "prefill-step": _probe_prefill_step,
          "prefill-gemm": _probe_prefill_gemm, "layer-sweep": _probe_layer_sweep,
          "verify-pass": _probe_verify_pass}


def main():
    if len(sys.argv) > 2 and sys.argv[1] == "--probe":
        if sys.argv[2] not in PROBES:
            raise SystemExit(f"--probe: one of {sorted(PROBES)}")
        PROBES[sys.argv[2]](sys.argv[3:])
        return
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
