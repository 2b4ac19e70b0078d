"""ctypes binding of the C ABI in include/potpori_b200.h.

The library is built in-tree (``potpori_b200/libpotpori_b200.so``, see ``build.py``). There is
no fallback: if the library is missing or cannot be loaded, importing a shard raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpotpori_b200.so")

PP_OK, PP_E_INVALID, PP_E_NONFINITE, PP_E_CUDA, PP_E_TIMEOUT, PP_E_OOM, PP_E_UNSUPPORTED, \
    PP_E_MISSING = range(8)
PP_F32, PP_BF16 = 0, 1
STATUS_NAMES = {
    PP_OK: "PP_OK", PP_E_INVALID: "PP_E_INVALID", PP_E_NONFINITE: "PP_E_NONFINITE",
    PP_E_CUDA: "PP_E_CUDA", PP_E_TIMEOUT: "PP_E_TIMEOUT", PP_E_OOM: "PP_E_OOM",
    PP_E_UNSUPPORTED: "PP_E_UNSUPPORTED", PP_E_MISSING: "PP_E_MISSING",
}

# Every symbol include/potpori_b200.h declares, in declaration order.
EXPORTS = [
    "pp_shard_create", "pp_shard_destroy", "pp_shard_set_tensor", "pp_shard_load_safetensors",
    "pp_shard_init_random", "pp_shard_missing", "pp_shard_forward_tokens",
    "pp_shard_forward_hidden", "pp_shard_step_device", "pp_shard_set_step", "pp_shard_buffers",
    "pp_shard_read_result", "pp_shard_handoff", "pp_shard_result_enqueue",
    "pp_shard_result_wait", "pp_shard_reset", "pp_shard_fill_kv", "pp_shard_capacity",
    "pp_shard_chunk_size", "pp_shard_range", "pp_shard_hidden_dim", "pp_shard_vocab_size",
    "pp_shard_model_layers", "pp_shard_device_bytes", "pp_shard_last_launches",
    "pp_shard_profile_kernels", "pp_shard_stream", "pp_shard_set_graphs", "pp_shard_set_pdl",
    "pp_shard_set_sm_limit", "pp_shard_sm_limit", "pp_shard_decode_greedy",
    "pp_shard_prefill", "pp_shard_prefill_hidden", "pp_shard_prefill_read",
    "pp_shard_prefill_handoff", "pp_shard_prefill_export", "pp_shard_prefill_open",
    "pp_shard_prefill_send", "pp_shard_set_decode_kernel", "pp_shard_decode_kernel",
    "pp_rows_gemm_work_bytes", "pp_rows_gemm", "pp_norm_gemv_static", "pp_shard_set_taps",
    "pp_shard_tap_layers", "pp_shard_read_taps", "pp_shard_set_wait_test", "pp_shard_inbox_export", "pp_shard_outbox_open",
    "pp_shard_send", "pp_shard_recv", "pp_shard_send_result", "pp_host_register",
    "pp_host_unregister", "pp_last_error", "pp_version",
]

KERNEL_KINDS = ["begin", "embed", "qkv", "attn", "attn_combine", "o_proj", "gate_up", "down",
                "head", "decode"]


class PPError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "layers", "hidden", "intermediate", "head_dim", "n_heads", "n_kv_heads", "vocab_size")] + [
        ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)]


class ShardDesc(ctypes.Structure):
    _fields_ = [
        ("cfg", Config),
        ("layer_begin", ctypes.c_uint32),
        ("layer_end", ctypes.c_uint32),
        ("capacity", ctypes.c_uint32),
        ("chunk", ctypes.c_uint32),
        ("cuda_device", ctypes.c_int32),
    ]


class VerifyOut(ctypes.Structure):
    _fields_ = [
        ("argmax", ctypes.POINTER(ctypes.c_int32)),
        ("top1", ctypes.POINTER(ctypes.c_float)),
        ("top2", ctypes.POINTER(ctypes.c_float)),
        ("logits", ctypes.POINTER(ctypes.c_float)),
        ("n_accepted", ctypes.c_int32),
        ("correction", ctypes.c_int32),
        ("nonfinite_rows", ctypes.c_int32),
    ]


_lib = None


def load() -> ctypes.CDLL:
    """Load the in-tree library (raises if it was never built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python -m potpori_b200.build` "
                          "(or __graft_entry__.build()) first")
    L = ctypes.CDLL(LIB_PATH)
    P, U32, I32, U64, F, SZ = (ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int32, ctypes.c_uint64,
                               ctypes.c_float, ctypes.c_size_t)
    pI32 = ctypes.POINTER(ctypes.c_int32)
    sig = {
        "pp_shard_create": (I32, [ctypes.POINTER(ShardDesc), ctypes.POINTER(P)]),
        "pp_shard_destroy": (None, [P]),
        "pp_shard_set_tensor": (I32, [P, ctypes.c_char_p, I32, P, U64]),
        "pp_shard_load_safetensors": (I32, [P, ctypes.c_char_p]),
        "pp_shard_init_random": (I32, [P, U64, F]),
        "pp_shard_missing": (I32, [P, ctypes.c_char_p, SZ]),
        "pp_shard_forward_tokens": (I32, [P, U32, pI32, U32, P, ctypes.POINTER(VerifyOut)]),
        "pp_shard_forward_hidden": (I32, [P, U32, U32, P, pI32, U32, P, ctypes.POINTER(VerifyOut)]),
        "pp_shard_step_device": (I32, [P, U32, P]),
        "pp_shard_set_step": (I32, [P, U32, U32, pI32, pI32, U32, I32, P]),
        "pp_shard_buffers": (I32, [P, ctypes.POINTER(P), ctypes.POINTER(P), ctypes.POINTER(P)]),
        "pp_shard_read_result": (I32, [P, U32, ctypes.POINTER(VerifyOut), P]),
        "pp_shard_handoff": (I32, [P, P, U32]),
        "pp_shard_result_enqueue": (I32, [P, U32]),
        "pp_shard_result_wait": (I32, [P, U32, U32, ctypes.POINTER(VerifyOut)]),
        "pp_shard_reset": (I32, [P]),
        "pp_shard_fill_kv": (I32, [P, U64, U32]),
        "pp_shard_capacity": (U32, [P]),
        "pp_shard_chunk_size": (U32, [P]),
        "pp_shard_range": (None, [P, ctypes.POINTER(U32), ctypes.POINTER(U32)]),
        "pp_shard_hidden_dim": (U32, [P]),
        "pp_shard_vocab_size": (U32, [P]),
        "pp_shard_model_layers": (U32, [P]),
        "pp_shard_device_bytes": (U64, [P]),
        "pp_shard_last_launches": (U32, [P]),
        "pp_shard_profile_kernels": (I32, [P, U32, U32, ctypes.POINTER(F), pI32, U32,
                                           ctypes.POINTER(U32)]),
        "pp_shard_stream": (P, [P]),
        "pp_shard_set_graphs": (I32, [P, I32]),
        "pp_shard_set_pdl": (I32, [P, I32]),
        "pp_shard_set_sm_limit": (I32, [P, U32]),
        "pp_shard_sm_limit": (U32, [P]),
        "pp_shard_prefill": (I32, [P, U32, pI32, U32]),
        "pp_shard_prefill_hidden": (I32, [P, U32, U32, P]),
        "pp_shard_prefill_read": (I32, [P, U32, P]),
        "pp_shard_prefill_handoff": (I32, [P, P, U32]),
        "pp_shard_prefill_export": (I32, [P, P]),
        "pp_shard_prefill_open": (I32, [P, P]),
        "pp_shard_prefill_send": (I32, [P, U32, U32, P, U32]),
        "pp_shard_set_decode_kernel": (I32, [P, I32]),
        "pp_shard_decode_kernel": (I32, [P]),
        "pp_shard_decode_greedy": (I32, [P, U32, I32, U32, pI32]),
        "pp_rows_gemm_work_bytes": (U64, [U32, U32]),
        "pp_rows_gemm": (I32, [P, U32, U32, P, U32, P, P, U64, P, P]),
        "pp_norm_gemv_static": (I32, [P, P, P, F, U32, U32, U32, P, P, P]),
        "pp_shard_set_taps": (I32, [P, ctypes.POINTER(U32), U32]),
        "pp_shard_tap_layers": (U32, [P, ctypes.POINTER(U32), U32]),
        "pp_shard_read_taps": (I32, [P, U32, P, P]),
        "pp_shard_set_wait_test": (I32, [P, U32, I32]),
        "pp_shard_inbox_export": (I32, [P, U32, P]),
        "pp_shard_outbox_open": (I32, [P, P, U32]),
        "pp_shard_send": (I32, [P, U32, U32, P, U32]),
        "pp_shard_recv": (I32, [P, U32, U32]),
        "pp_shard_send_result": (I32, [P, P, P, U32]),
        "pp_host_register": (I32, [P, SZ]),
        "pp_host_unregister": (I32, [P]),
        "pp_last_error": (SZ, [P, ctypes.c_char_p, SZ]),
        "pp_version": (ctypes.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error(handle) -> str:
    L = load()
    buf = ctypes.create_string_buffer(1024)
    L.pp_last_error(handle, buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, handle=None, what: str = "") -> None:
    if status != PP_OK:
        msg = last_error(handle)
        raise PPError(status, f"{what}: {msg}" if what else msg)
