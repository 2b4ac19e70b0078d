"""Rate of the tensor-core prompt projection (pp_rows_gemm) at a prefill shape on one GPU.

Random BF16 weights [n][k] in the shards' tiled layout and F32 activations [t][k]; each call
splits the activations into BF16 hi + lo blocks and runs the tcgen05 GEMM. Reports the
device time per call (CUDA events, after warm-up) and the rate counted two ways: useful
(2 t n k flops) and issued (both MMAs per K step, W.hi and W.lo). The default shape is the
Qwen3-4B gate/up projection over a 2048-row prompt chunk.

    python -m potpori_b200.prefill_gemm [--t 2048] [--n 19456] [--k 2560] [--iters 10]
"""
from __future__ import annotations

import argparse
import ctypes
import json

import numpy as np

from . import _lib


def main():
    import torch

    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--t", type=int, default=2048)
    ap.add_argument("--n", type=int, default=19456)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
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


if __name__ == "__main__":
    main()
