"""The tensor-core (tcgen05) projection of a prompt chunk against a float64 reference.

pp_rows_gemm computes y = x . W^T for t activation rows from the shards' tiled BF16 weights,
on the 5th-generation tensor cores with x carried as BF16 hi + lo parts. Here it is checked
through the C ABI against numpy in float64 (rel-L2 <= 1e-5, the F32 products and sums of
src/qwen/model.rs:166-183 to their rounding), at a ragged size (t and n not multiples of the
tile), twice in a row on the same buffers, and at the 4B gate/up shape of a 2048-row prompt
chunk, where its rate is reported.
"""
import ctypes

import numpy as np
import pytest

from helpers import f32_to_bf16_bits, rel_l2, tile_weights
from potpori_b200 import _lib

pytestmark = pytest.mark.gpu


def _bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _run(L, torch, w_bits, x, reps=1):
    n, k = w_bits.shape
    t = x.shape[0]
    dev = torch.device("cuda", 0)
    w_t = torch.from_numpy(tile_weights(w_bits).view(np.int16)).to(dev)
    x_t = torch.from_numpy(x).to(dev)
    y_t = torch.full((t, n), float("nan"), dtype=torch.float32, device=dev)
    wb = int(L.pp_rows_gemm_work_bytes(t, k))
    work = torch.empty(wb + 1024, dtype=torch.uint8, device=dev)
    base = (work.data_ptr() + 1023) // 1024 * 1024
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    outs, ms = [], []
    for _ in range(reps):
        y_t.fill_(float("nan"))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        st = L.pp_rows_gemm(w_t.data_ptr(), n, k, x_t.data_ptr(), t, y_t.data_ptr(),
                            ctypes.c_void_p(base), wb, err.data_ptr(), ctypes.c_void_p(stream))
        e1.record()
        assert st == _lib.PP_OK, _lib.last_error(None)
        torch.cuda.synchronize(dev)
        assert int(err.item()) == 0
        ms.append(e0.elapsed_time(e1))
        outs.append(y_t.cpu().numpy())
    return outs, ms


def test_rows_gemm_matches_float64(gpu):
    import torch

    L = _lib.load()
    rng = np.random.default_rng(11)
    n, k, t = 300, 2560, 333
    w = f32_to_bf16_bits((0.02 * rng.standard_normal((n, k))).astype(np.float32))
    x = rng.standard_normal((t, k)).astype(np.float32)
    want = x.astype(np.float64) @ _bf16_to_f32(w).astype(np.float64).T
    outs, _ = _run(L, torch, w, x, reps=2)
    for call, got in enumerate(outs):
        assert np.isfinite(got).all(), f"call {call}"
        e = rel_l2(got, want)
        assert e <= 1e-5, f"call {call}: rel-L2 {e:.2e}"
    assert np.array_equal(outs[0], outs[1])


def test_rows_gemm_prefill_shape(gpu):
    """Qwen3-4B gate/up (19456 x 2560) over a 2048-row prompt chunk: parity on sampled rows,
    and the rate (two BF16 MMAs per K step, W.hi and W.lo)."""
    import torch

    L = _lib.load()
    rng = np.random.default_rng(12)
    n, k, t = 19456, 2560, 2048
    w = f32_to_bf16_bits((0.02 * rng.standard_normal((n, k))).astype(np.float32))
    x = rng.standard_normal((t, k)).astype(np.float32)
    outs, ms = _run(L, torch, w, x, reps=4)
    rows = rng.choice(t, 64, replace=False)
    want = x[rows].astype(np.float64) @ _bf16_to_f32(w).astype(np.float64).T
    e = rel_l2(outs[-1][rows], want)
    assert e <= 1e-5, f"rel-L2 {e:.2e}"
    best = min(ms[1:])
    print(f"rows_gemm {t}x{n}x{k}: {best:.3f} ms, {2 * t * n * k / best / 1e9:.1f} TFLOP/s useful, "
          f"{4 * t * n * k / best / 1e9:.1f} TFLOP/s issued")
