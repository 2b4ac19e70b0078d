"""ctypes front end of the oracle (test infrastructure).

The oracle is a CPU restatement of potpori's per-shard Qwen3 forward (``oracle/oracle.c``;
the reference lines it follows are listed in ``oracle/oracle.h``). Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` import this module, as the
checker or as the timed CPU baseline. The product path never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

OR_OK, OR_E_INVALID, OR_E_NONFINITE, OR_E_MISSING = 0, 1, 2, 3
OR_F32, OR_BF16 = 0, 1
ROPE_F64, ROPE_F32 = 0, 1


class OracleError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: oracle status {code}")
        self.code = code


class _Config(ctypes.Structure):
    _fields_ = [
        ("layers", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("n_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
    ]


def build() -> str:
    """Compile the oracle library with its Makefile (gcc is the only requirement)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_SO):
        build()
    L = ctypes.CDLL(_SO)
    P, I32, I64, U64, F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float
    L.or_shard_create.restype = P
    L.or_shard_create.argtypes = [ctypes.POINTER(_Config), I32, I32, I32, I32]
    L.or_shard_destroy.argtypes = [P]
    L.or_shard_set_tensor.argtypes = [P, ctypes.c_char_p, I32, P, I64]
    L.or_shard_init_random.argtypes = [P, U64, F]
    L.or_shard_fill_kv.argtypes = [P, U64, I32]
    L.or_shard_missing.argtypes = [P, ctypes.c_char_p, I64]
    L.or_shard_set_rope_mode.argtypes = [P, I32]
    L.or_shard_forward.argtypes = [P, I32, I32, P, P, P, P]
    L.or_shard_reset.argtypes = [P]
    L.or_argmax.argtypes = [P, I64, ctypes.POINTER(I32)]
    L.or_top2.argtypes = [P, I64, ctypes.POINTER(F), ctypes.POINTER(F)]
    L.or_set_threads.argtypes = [I32]
    L.or_get_threads.restype = I32
    L.or_gen_bf16.argtypes = [U64, ctypes.c_char_p, I64, I64, F, P]
    L.or_name_hash.restype = U64
    L.or_name_hash.argtypes = [ctypes.c_char_p]
    _lib = L
    return L


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def get_threads() -> int:
    return int(lib().or_get_threads())


def _cfg(cfg) -> _Config:
    return _Config(
        cfg.layers, cfg.hidden, cfg.intermediate, cfg.head_dim, cfg.n_heads,
        cfg.n_kv_heads, cfg.vocab_size, cfg.rms_norm_eps, cfg.rope_theta,
    )


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class OracleShard:
    """Layers [layer_begin, layer_end) of a Qwen3 model with its own F32 KV cache."""

    def __init__(self, cfg, layer_begin: int, layer_end: int, capacity: int, chunk: int = 0,
                 rope_mode: int = ROPE_F64):
        self.cfg = cfg
        self.range = (layer_begin, layer_end)
        self.first = layer_begin == 0
        self.last = layer_end == cfg.layers
        self.capacity = capacity
        self.chunk = chunk
        c = _cfg(cfg)
        self._h = lib().or_shard_create(ctypes.byref(c), layer_begin, layer_end, capacity, chunk)
        if not self._h:
            raise OracleError(OR_E_INVALID, "invalid shard configuration")
        if rope_mode != ROPE_F64:
            lib().or_shard_set_rope_mode(self._h, rope_mode)

    def close(self) -> None:
        if self._h:
            lib().or_shard_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tensor(self, name: str, value: np.ndarray) -> None:
        if value.dtype == np.float32:
            dt = OR_F32
        elif value.dtype in (np.uint16, np.int16):
            dt = OR_BF16
        else:
            raise TypeError(f"{name}: need float32 or bf16 bits (uint16), got {value.dtype}")
        value = np.ascontiguousarray(value)
        rc = lib().or_shard_set_tensor(self._h, name.encode(), dt, _ptr(value), value.size)
        if rc:
            raise OracleError(rc, f"set_tensor {name}")

    def load(self, tensors: dict) -> None:
        for name, value in tensors.items():
            self.set_tensor(name, value)

    def init_random(self, seed: int, std: float = 0.02) -> None:
        lib().or_shard_init_random(self._h, seed, std)

    def fill_kv(self, seed: int, rows: int) -> None:
        rc = lib().or_shard_fill_kv(self._h, seed, rows)
        if rc:
            raise OracleError(rc, "fill_kv")

    def missing(self) -> list:
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().or_shard_missing(self._h, buf, len(buf))
        return [s for s in buf.value.decode().split(";") if s][:n]

    def forward(self, pos: int, tokens=None, hidden=None, taps: bool = False):
        """One chunk at absolute position ``pos``. Returns ``out`` (hidden ``[m, H]`` or
        logits ``[m, V]`` on the last shard) and, with ``taps``, ``[layers, m, H]``."""
        cfg = self.cfg
        if tokens is not None:
            tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
            m = tok.size
            tp, hp = _ptr(tok), None
        else:
            hid = np.ascontiguousarray(np.asarray(hidden, dtype=np.float32))
            m = hid.size // cfg.hidden
            tp, hp = None, _ptr(hid)
        width = cfg.vocab_size if self.last else cfg.hidden
        out = np.empty((m, width), np.float32)
        tap = np.empty((self.range[1] - self.range[0], m, cfg.hidden), np.float32) if taps else None
        rc = lib().or_shard_forward(self._h, pos, m, tp, hp, _ptr(out),
                                    _ptr(tap) if taps else None)
        if rc:
            raise OracleError(rc, f"forward(pos={pos}, m={m})")
        return (out, tap) if taps else out

    def reset(self) -> None:
        lib().or_shard_reset(self._h)


def argmax(row: np.ndarray) -> Optional[int]:
    """``src/engine.rs:14-29``: first index of the strict maximum; None if empty or non-finite."""
    row = np.ascontiguousarray(row, dtype=np.float32)
    idx = ctypes.c_int32(0)
    ok = lib().or_argmax(_ptr(row) if row.size else None, row.size, ctypes.byref(idx))
    return int(idx.value) if ok else None


def top2(row: np.ndarray):
    row = np.ascontiguousarray(row, dtype=np.float32)
    a, b = ctypes.c_float(), ctypes.c_float()
    lib().or_top2(_ptr(row), row.size, ctypes.byref(a), ctypes.byref(b))
    return float(a.value), float(b.value)


def gen_bf16(seed: int, name: str, count: int, start: int = 0, std: float = 0.02) -> np.ndarray:
    out = np.empty(count, np.uint16)
    lib().or_gen_bf16(seed, name.encode(), start, count, std, _ptr(out))
    return out


def name_hash(name: str) -> int:
    return int(lib().or_name_hash(name.encode()))
