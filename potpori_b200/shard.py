"""One contiguous range of Qwen3 layers on one B200, behind the reference's shard interface.

``Shard`` mirrors ``src/qwen/shard.rs:17-133`` and the ``ShardEngine`` trait of
``src/node.rs:55-86`` (forward_tokens / forward_hidden / reset / capacity / chunk_size /
range / hidden_dim / vocab_size / hello) over the C ABI of ``include/potpori_b200.h``.
The reference's forward returns the full F32 logits of the last shard and picks tokens on
the host; here the tail also computes the greedy pick, top-2 and the accept compare on the
device (``verify_*``), so the default path reads back only a few integers per row.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import PPError, check
from .config import QwenConfig


@dataclass
class VerifyResult:
    """What the tail returns for one chunk (``src/transport.rs`` VerifyResult + accept)."""
    argmax: list
    top1: list
    top2: list
    n_accepted: int
    correction: int
    nonfinite_rows: int
    logits: Optional[np.ndarray] = field(default=None, repr=False)

    @property
    def finite(self) -> bool:
        return self.nonfinite_rows == 0


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


class Shard:
    """Layers ``[begin, end)`` of a Qwen3 model with its own F32 KV cache on one device."""

    def __init__(self, cfg: QwenConfig, layer_range: tuple, capacity: int, chunk: int = 8,
                 device: int = 0):
        L = _lib.load()
        self.cfg = cfg
        self._range = (int(layer_range[0]), int(layer_range[1]))
        self.first = self._range[0] == 0
        self.last = self._range[1] == cfg.layers
        desc = _lib.ShardDesc(
            _lib.Config(cfg.layers, cfg.hidden, cfg.intermediate, cfg.head_dim, cfg.n_heads,
                        cfg.n_kv_heads, cfg.vocab_size, cfg.rms_norm_eps, cfg.rope_theta),
            self._range[0], self._range[1], capacity, chunk, device)
        h = ctypes.c_void_p()
        st = L.pp_shard_create(ctypes.byref(desc), ctypes.byref(h))
        if st != _lib.PP_OK:
            raise PPError(st, f"invalid shard configuration: {_lib.last_error(None)}")
        self._h = h
        self._L = L
        self.device = device
        self._vo = _lib.VerifyOut()
        self._last_m = 1
        self._am = np.zeros(16, np.int32)
        self._t1 = np.zeros(16, np.float32)
        self._t2 = np.zeros(16, np.float32)

    # ---- construction helpers (Shard::load_chunked, src/qwen/shard.rs:28-52) ----
    @classmethod
    def load_chunked(cls, cfg: QwenConfig, layer_range: tuple, first: bool, last: bool, path: str,
                     capacity: int, search: int = 0, chunk: int = 8, device: int = 0) -> "Shard":
        """Build the shard for ``layer_range`` and load its parameters from a prepared
        safetensors file. ``first``/``last`` must match the range (model.rs:210-213);
        ``search`` is accepted for signature parity (there is no kernel search here)."""
        if first != (layer_range[0] == 0) or last != (layer_range[1] == cfg.layers):
            raise PPError(_lib.PP_E_INVALID, "shard role does not match layer range")
        s = cls(cfg, layer_range, capacity, chunk, device)
        s.load_safetensors(path)
        return s

    @classmethod
    def random(cls, cfg: QwenConfig, layer_range: tuple, capacity: int, chunk: int = 8,
               seed: int = 0, std: float = 0.02, device: int = 0) -> "Shard":
        s = cls(cfg, layer_range, capacity, chunk, device)
        s.init_random(seed, std)
        return s

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.pp_shard_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self):
        return self._h

    # ---- parameters ----
    def set_tensor(self, name: str, value: np.ndarray) -> None:
        value = np.ascontiguousarray(value)
        if value.dtype == np.float32:
            dt = _lib.PP_F32
        elif value.dtype in (np.uint16, np.int16):
            dt = _lib.PP_BF16
        else:
            raise TypeError(f"{name}: float32 or bf16 bits (uint16) expected, got {value.dtype}")
        check(self._L.pp_shard_set_tensor(self._h, name.encode(), dt, value.ctypes.data, value.size),
              self._h, f"set_tensor {name}")

    def load(self, tensors: dict) -> None:
        for name, value in tensors.items():
            self.set_tensor(name, value)

    def load_safetensors(self, path: str) -> None:
        check(self._L.pp_shard_load_safetensors(self._h, str(path).encode()), self._h,
              f"load {path}")

    def init_random(self, seed: int, std: float = 0.02) -> None:
        check(self._L.pp_shard_init_random(self._h, seed, std), self._h, "init_random")

    def missing(self) -> list:
        buf = ctypes.create_string_buffer(1 << 16)
        self._L.pp_shard_missing(self._h, buf, len(buf))
        return [s for s in buf.value.decode().split(";") if s]

    def fill_kv(self, seed: int, rows: int) -> None:
        check(self._L.pp_shard_fill_kv(self._h, seed, rows), self._h, "fill_kv")

    # ---- ShardEngine ----
    def range(self) -> tuple:
        return self._range

    def model_layers(self) -> int:
        return self.cfg.layers

    def hidden_dim(self) -> int:
        return self.cfg.hidden

    def vocab_size(self) -> int:
        return self.cfg.vocab_size

    def capacity(self) -> int:
        return int(self._L.pp_shard_capacity(self._h))

    def chunk_size(self) -> int:
        return int(self._L.pp_shard_chunk_size(self._h))

    def hello(self, next_layer: int) -> dict:
        """SessionHello of src/qwen/shard.rs:89-105 (with the tapped layers of
        TappedShards::hello, src/node.rs:160-166)."""
        return {"model": self.cfg.hello_model(), "next_layer": next_layer,
                "max_seq": self.capacity(), "chunk": self.chunk_size(),
                "taps": self.tap_layers()}

    # ---- tapped layers (TappedShards, src/node.rs:108-223) ----
    def set_taps(self, layers: Sequence[int]) -> None:
        """Keep the output rows of these model layers after every step (ascending, inside the
        shard's range, below the model's last layer); [] ends tapping."""
        arr = (ctypes.c_uint32 * max(len(layers), 1))(*[int(l) for l in layers])
        check(self._L.pp_shard_set_taps(self._h, arr, len(layers)), self._h, "set_taps")

    def tap_layers(self) -> List[int]:
        """ShardEngine::tap_layers (src/node.rs:206-213): the tapped layers of this shard."""
        buf = (ctypes.c_uint32 * 256)()
        n = int(self._L.pp_shard_tap_layers(self._h, buf, 256))
        return [int(buf[i]) for i in range(min(n, 256))]

    def take_taps(self, m: Optional[int] = None, bf16: bool = False) -> List[np.ndarray]:
        """ShardEngine::take_taps (src/node.rs:214-216): the last step's output of every tapped
        layer, [m, hidden] each (F32, or the BF16 bits of the wire form LayerTap::from_f32)."""
        m = int(m if m is not None else self._last_m)
        layers = self.tap_layers()
        if not layers:
            return []
        shape = (len(layers), m, self.cfg.hidden)
        f = np.empty(shape, np.float32) if not bf16 else None
        b = np.empty(shape, np.uint16) if bf16 else None
        check(self._L.pp_shard_read_taps(self._h, m, f.ctypes.data if f is not None else None,
                                         b.ctypes.data if b is not None else None),
              self._h, "read_taps")
        out = b if bf16 else f
        return [out[i] for i in range(len(layers))]

    def reset(self) -> None:
        check(self._L.pp_shard_reset(self._h), self._h, "reset KV")

    def device_bytes(self) -> int:
        return int(self._L.pp_shard_device_bytes(self._h))

    def last_launches(self) -> int:
        return int(self._L.pp_shard_last_launches(self._h))

    def stream(self) -> int:
        """The shard's own CUDA stream handle (cudaStream_t as an int)."""
        return int(self._L.pp_shard_stream(self._h) or 0)

    def profile_kernels(self, max_rows: int, iters: int = 5) -> list:
        """Mean duration of every kernel of one step launched in isolation:
        [(kind, ms), ...] in launch order."""
        cap = 4096
        ms = (ctypes.c_float * cap)()
        kinds = (ctypes.c_int32 * cap)()
        n = ctypes.c_uint32()
        check(self._L.pp_shard_profile_kernels(self._h, max_rows, iters, ms, kinds, cap,
                                               ctypes.byref(n)), self._h, "profile")
        return [(_lib.KERNEL_KINDS[kinds[i]], float(ms[i])) for i in range(min(n.value, cap))]

    def set_graphs(self, enabled: bool) -> None:
        check(self._L.pp_shard_set_graphs(self._h, int(enabled)), self._h)

    def set_pdl(self, enabled: bool) -> None:
        check(self._L.pp_shard_set_pdl(self._h, int(enabled)), self._h)

    def decode_greedy(self, pos: int, token: int, n: int) -> List[int]:
        """n single-token greedy steps fed on the device (whole-model shard): the picks."""
        out = np.zeros(n, np.int32)
        check(self._L.pp_shard_decode_greedy(
            self._h, pos, int(token), n, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))),
            self._h, f"decode_greedy(pos={pos}, n={n})")
        return out.tolist()

    def set_sm_limit(self, ctas: int) -> None:
        """Most CTAs (SMs) any kernel of this shard uses; 0 = all. Leave out SMs that other
        work on the device holds (another model's long-running kernels, transfer kernels of a
        communication library)."""
        check(self._L.pp_shard_set_sm_limit(self._h, int(ctas)), self._h, "set_sm_limit")

    def sm_limit(self) -> int:
        return int(self._L.pp_shard_sm_limit(self._h))

    PREFILL_MAX = 2048

    def can_prefill(self) -> bool:
        """Whether the one-pass prefill runs here: head size 128 and 1, 2, 4 or 8 query heads
        per KV head (every Qwen3 size)."""
        cfg = self.cfg
        return cfg.head_dim == 128 and cfg.n_heads // cfg.n_kv_heads in (1, 2, 4, 8)

    def prefill(self, pos: int, tokens: Sequence[int]) -> None:
        """First shard: write the K/V rows of prompt tokens at pos.. through every layer at once
        (tensor-core projections), in pieces of up to 2048 rows; no logits. A shard before the
        last keeps the output rows of its last layer for the next stage (one piece)."""
        for i in range(0, len(tokens), self.PREFILL_MAX):
            piece = np.asarray(tokens[i:i + self.PREFILL_MAX], np.int32)
            check(self._L.pp_shard_prefill(self._h, pos + i, piece.ctypes.data_as(
                ctypes.POINTER(ctypes.c_int32)), len(piece)), self._h, f"prefill(pos={pos + i})")

    def prefill_hidden(self, pos: int, t: int, hidden=None) -> None:
        """Later stage: the prefill pass over t rows in its prefill buffer (filled by a
        handoff or a send), or over `hidden` [t, hidden] when given."""
        hp = None
        if hidden is not None:
            h = np.ascontiguousarray(np.asarray(hidden, np.float32)).reshape(t, self.cfg.hidden)
            hp = h.ctypes.data
        check(self._L.pp_shard_prefill_hidden(self._h, pos, t, hp), self._h,
              f"prefill_hidden(pos={pos}, t={t})")

    def prefill_read(self, t: int) -> np.ndarray:
        out = np.empty((t, self.cfg.hidden), np.float32)
        check(self._L.pp_shard_prefill_read(self._h, t, out.ctypes.data), self._h, "prefill_read")
        return out

    def prefill_handoff_from(self, prev: "Shard", t: int) -> None:
        check(self._L.pp_shard_prefill_handoff(prev._h, self._h, t), self._h, "prefill_handoff")

    def prefill_export(self) -> bytes:
        h = ctypes.create_string_buffer(64)
        check(self._L.pp_shard_prefill_export(self._h, h), self._h, "prefill_export")
        return h.raw

    def prefill_open(self, handle: bytes) -> None:
        buf = ctypes.create_string_buffer(bytes(handle), 64)
        check(self._L.pp_shard_prefill_open(self._h, buf), self._h, "prefill_open")

    def prefill_send(self, seq: int, t: int, mail_ptr: int, info: int) -> None:
        check(self._L.pp_shard_prefill_send(self._h, seq, t, mail_ptr, info), self._h,
              "prefill_send")

    def set_decode_kernel(self, enabled: bool = True) -> None:
        """Run 1-row steps of this whole-model shard as one persistent kernel (plus the vocab
        head) instead of six kernels per layer; keeps a row-major copy of the layer weights."""
        check(self._L.pp_shard_set_decode_kernel(self._h, 1 if enabled else 0), self._h,
              "set_decode_kernel")

    def decode_kernel(self) -> bool:
        return bool(self._L.pp_shard_decode_kernel(self._h))

    def set_wait_test(self, limit_us: int = 0, unreachable: bool = False) -> None:
        """Test hook: the decode kernel's barrier time limit (0: default) and, with
        `unreachable`, barriers that can only end by running out of time."""
        check(self._L.pp_shard_set_wait_test(self._h, int(limit_us), int(bool(unreachable))),
              self._h, "set_wait_test")

    def _verify_struct(self, want_logits: Optional[np.ndarray]):
        vo = self._vo
        vo.argmax = self._am.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
        vo.top1 = self._t1.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        vo.top2 = self._t2.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        vo.logits = (want_logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
                     if want_logits is not None else None)
        return vo

    def _result(self, m: int, logits) -> VerifyResult:
        vo = self._vo
        return VerifyResult(self._am[:m].tolist(), self._t1[:m].tolist(), self._t2[:m].tolist(),
                            int(vo.n_accepted), int(vo.correction), int(vo.nonfinite_rows), logits)

    def _run(self, pos: int, tokens, hidden, drafts, want_logits: bool):
        cfg = self.cfg
        if self.first:
            tok = _i32(tokens)
            m = tok.size
        else:
            hid = np.ascontiguousarray(np.asarray(hidden, dtype=np.float32)).reshape(-1)
            m = hid.size // cfg.hidden
        self._last_m = m
        out_h = None if self.last else np.empty((m, cfg.hidden), np.float32)
        logits = np.empty((m, cfg.vocab_size), np.float32) if (self.last and want_logits) else None
        vo = self._verify_struct(logits) if self.last else None
        vp = ctypes.byref(vo) if vo is not None else None
        hp = out_h.ctypes.data if out_h is not None else None
        if self.first:
            st = self._L.pp_shard_forward_tokens(
                self._h, pos, tok.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), m, hp, vp)
        else:
            d = _i32(drafts if drafts is not None else [])
            st = self._L.pp_shard_forward_hidden(
                self._h, pos, m, hid.ctypes.data,
                d.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) if d.size else None, d.size, hp, vp)
        if st not in (_lib.PP_OK, _lib.PP_E_NONFINITE):
            check(st, self._h, f"forward(pos={pos}, m={m})")
        if self.last:
            return self._result(m, logits)
        return out_h

    def forward_tokens(self, pos: int, tokens: Sequence[int]) -> np.ndarray:
        """First shard (src/node.rs:70): the residual stream ``[s, hidden]``, or the
        ``[s, vocab]`` logits when this shard is also the last."""
        out = self._run(pos, tokens, None, None, want_logits=True)
        return out.logits if self.last else out

    def forward_hidden(self, pos: int, s: int, hidden) -> np.ndarray:
        """Non-first shard (src/node.rs:73): ``[s, hidden]`` in, ``[s, hidden]`` or logits out."""
        hid = np.asarray(hidden, dtype=np.float32).reshape(s, self.cfg.hidden)
        out = self._run(pos, None, hid, None, want_logits=True)
        return out.logits if self.last else out

    def verify_tokens(self, pos: int, tokens: Sequence[int], logits: bool = False) -> VerifyResult:
        """First+last shard: on-device greedy pick for every row of the chunk and the accept
        compare of drafts = tokens[1:] (src/specdecode.rs:92-98)."""
        return self._run(pos, tokens, None, None, want_logits=logits)

    def verify_hidden(self, pos: int, hidden, drafts: Sequence[int] = (),
                      logits: bool = False) -> VerifyResult:
        return self._run(pos, None, hidden, drafts, want_logits=logits)

    # ---- device-resident stage path (in-box pipeline) ----
    def buffers(self) -> tuple:
        """Device pointers (hidden, header, result) of the shard's resident buffers."""
        h, d, r = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        check(self._L.pp_shard_buffers(self._h, ctypes.byref(h), ctypes.byref(d), ctypes.byref(r)),
              self._h)
        return h.value, d.value, r.value

    def set_step(self, pos: int, m: int, tokens=None, drafts=(), want_logits=False,
                 stream: int = 0, flags: int = 0) -> None:
        """Enqueue the step header. flags bit 0 (or want_logits) also writes the logits; other
        bits travel with the header to the next stages."""
        self._last_m = m
        t = _i32(tokens) if tokens is not None else None
        d = _i32(drafts)
        check(self._L.pp_shard_set_step(
            self._h, pos, m, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) if t is not None else None,
            d.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) if d.size else None, d.size,
            int(flags) | int(bool(want_logits)), stream or None), self._h, "set_step")

    def step_device(self, max_rows: int, stream: int = 0) -> None:
        check(self._L.pp_shard_step_device(self._h, max_rows, stream or None), self._h, "step")

    def handoff_from(self, prev: "Shard", m: int) -> None:
        """Enqueue the copy of ``prev``'s output rows into this shard's input (peer copy over
        NVLink across devices), ordered after ``prev``'s enqueued work."""
        check(self._L.pp_shard_handoff(prev._h, self._h, m), self._h, "handoff")

    def result_enqueue(self, slot: int) -> None:
        check(self._L.pp_shard_result_enqueue(self._h, slot), self._h, "result_enqueue")

    def result_wait(self, slot: int, m: int) -> VerifyResult:
        vo = self._verify_struct(None)
        st = self._L.pp_shard_result_wait(self._h, slot, m, ctypes.byref(vo))
        if st not in (_lib.PP_OK, _lib.PP_E_NONFINITE):
            check(st, self._h, "result_wait")
        return self._result(m, None)

    # ---- cross-process link (pipeline stages in different processes of one box) ----
    def inbox_export(self, slots: int) -> bytes:
        """Allocate this stage's inbox of `slots` chunk slots; its CUDA IPC handle (64 bytes)."""
        h = ctypes.create_string_buffer(64)
        check(self._L.pp_shard_inbox_export(self._h, slots, h), self._h, "inbox_export")
        return h.raw

    def outbox_open(self, handle: bytes, slots: int) -> None:
        """Open the next stage's inbox (its IPC handle) as this stage's outbox."""
        buf = ctypes.create_string_buffer(bytes(handle), 64)
        check(self._L.pp_shard_outbox_open(self._h, buf, slots), self._h, "outbox_open")

    def send(self, seq: int, m: int, mail_ptr: int, info: int) -> None:
        """Enqueue: the chunk's header and m hidden rows into slot seq of the next stage's inbox,
        then mail[1] = info and mail[0] = seq + 1 (mail_ptr: registered host memory)."""
        check(self._L.pp_shard_send(self._h, seq, m, mail_ptr, info), self._h, "send")

    def recv(self, seq: int, m: int) -> None:
        """Enqueue: slot seq of this stage's inbox into its input and header buffers."""
        check(self._L.pp_shard_recv(self._h, seq, m), self._h, "recv")

    def send_result(self, host_ptr: int, mail_ptr: int, value: int) -> None:
        """Enqueue: the step result into host memory at host_ptr, then *mail = value."""
        check(self._L.pp_shard_send_result(self._h, host_ptr, mail_ptr, value), self._h,
              "send_result")

    def read_result(self, m: int, stream: int = 0, logits: bool = False) -> VerifyResult:
        lg = np.empty((m, self.cfg.vocab_size), np.float32) if logits else None
        vo = self._verify_struct(lg)
        st = self._L.pp_shard_read_result(self._h, m, ctypes.byref(vo), stream or None)
        if st not in (_lib.PP_OK, _lib.PP_E_NONFINITE):
            check(st, self._h, "read_result")
        return self._result(m, lg)
