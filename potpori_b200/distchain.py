"""Pipeline stages in separate processes, one per GPU, joined by CUDA IPC copies on the copy
engines and mailbox words in host memory that the processes share.

This replaces the reference's chain over QUIC (head ChainLink::send_chunk -> relay_middle ->
serve_tail -> VerifyResult back, src/node.rs:242-342,466-535, src/transport.rs:425-489):
 * rank 0 (the head) runs the draft model, stage 0 and the driver; every chunk it submits
   travels as the step header (position, rows, tokens, drafts) and the chunk's F32 hidden rows
   from rank r to rank r+1: after its step, rank r's stream copies them into slot k of rank
   r+1's inbox (device memory opened through CUDA IPC; the copy engines move it over NVLink)
   and then writes the slot's two mailbox words (info, then k + 1) into the shared host
   memory with stream-ordered writes;
 * every other rank loops: wait on the host for chunk k's mailbox word, copy the inbox slot
   into its shard's input and header buffers (stream-ordered), run the step (graph replay)
   and send it on;
 * the last rank computes the greedy picks and the accept compare on the device and copies
   the 208-byte result straight into the head's result ring in the shared host memory (a
   direct return instead of the reference's relay), then its mailbox word.
No SM takes part in a transfer: the copies run on the copy engines and the mailbox words are
stream memory writes, so the stages' kernels, and the draft's cooperative decode kernel on
rank 0, keep every SM. torch.distributed carries only the setup (the handshake of
src/transport.rs:299-358, the IPC handles and the shared memory's name) and the final timing
reduction. A chunk with m = 0 ends the session; flag bits mark the benchmark's timed window.

The protocol (run_stage, DistChain) talks to its stage through a small I/O object:
CudaStageIO (a Shard's device buffers and stream: the product path) or HostStageIO, a
host-memory stand-in whose inbox lives in the shared memory too, so the protocol runs under
gloo on CPU.
"""
from __future__ import annotations

import ctypes
import mmap
import os
import time
import uuid
from collections import deque
from typing import List, Tuple

import numpy as np
import torch
import torch.distributed as dist

from .chain import HandshakeError, check_link
from .config import is_eos
from .target import NonFiniteLogits

HDR_INTS = 36   # StepDesc: pos, m, n_drafts, flags, tokens[16], drafts[16]
RES_INTS = 52   # StepResult: argmax[16], top1[16], top2[16], nonfinite_rows, n_acc, corr, status
RES_NONFINITE, RES_STATUS = 48, 51
RES_SLOT = 256  # bytes per result slot
RING = 64       # chunk slots of every inbox and of the result ring
FLAG_WINDOW_START = 2
FLAG_WINDOW_END = 4
FLAG_PREFILL = 8  # the message is a prompt prefill: (pos, rows) in the link's parameter slot
FLAG_MARKS = 16   # the message has no rows and carries only its flags (timed-window marks)
PREFILL_MAX = 2048  # rows of one prefill message
WAIT_S = 120.0  # a stage that hears nothing for this long ends the session with an error


class ChainError(RuntimeError):
    pass


class ChainMemory:
    """The chain's shared host memory, one file in /dev/shm made by rank 0: for every link
    r -> r+1 a ring of RING mailbox word pairs (k + 1, info), the result ring (a word pair and
    a result slot per chunk) and, when `data_bytes` is given, the inbox data of host stand-ins
    (RING slots of data_bytes per link). info = rows | flags << 8."""

    def __init__(self, world: int, path: str, create: bool, data_bytes: int = 0,
                 extra_bytes: int = 0):
        self.world, self.path, self.data_bytes = world, path, data_bytes
        self.n_words = world * RING * 2  # world - 1 links + the result ring
        self.res_off = self.n_words * 4
        self.par_off = self.res_off + RING * RES_SLOT  # (pos, rows) of prefill messages
        self.data_off = self.par_off + world * RING * 8
        self.size = self.data_off + (world - 1) * RING * data_bytes + extra_bytes
        fd = os.open(path, os.O_RDWR | (os.O_CREAT if create else 0), 0o600)
        try:
            if create:
                os.ftruncate(fd, self.size)
            self.mm = mmap.mmap(fd, self.size)
        finally:
            os.close(fd)
        self.words = np.ndarray((self.n_words,), np.uint32, self.mm)
        if create:
            self.words[:] = 0
        self._anchor = ctypes.c_char.from_buffer(self.mm)
        self.base = ctypes.addressof(self._anchor)
        self.registered = False

    def mail(self, link: int, k: int) -> int:
        """Word index of chunk k's mailbox on link `link` (link world - 1: the results)."""
        return (link * RING + k % RING) * 2

    def params(self, link: int, k: int) -> np.ndarray:
        """The (pos, rows) words of prefill message k on `link`, written by the sender's host
        before it enqueues the message (so before its mailbox word can be seen)."""
        return np.ndarray((2,), np.uint32, self.mm, self.par_off + (link * RING + k % RING) * 8)

    def result_ints(self, k: int) -> np.ndarray:
        return np.ndarray((RES_INTS,), np.int32, self.mm, self.res_off + (k % RING) * RES_SLOT)

    def wait(self, link: int, k: int, timeout: float = WAIT_S) -> int:
        """Wait for chunk k on `link`; its info word."""
        i = self.mail(link, k)
        want = (k + 1) & 0xFFFFFFFF
        t0 = time.monotonic()
        n = 0
        while int(self.words[i]) != want:
            n += 1
            if (n & 1023) == 0:
                if time.monotonic() - t0 > timeout:
                    raise ChainError(f"no chunk {k} on link {link} within {timeout:.0f} s")
                time.sleep(0)
        return int(self.words[i + 1])

    def register(self, lib) -> None:
        from ._lib import check
        check(lib.pp_host_register(self.base, self.size), None, "register the chain memory")
        self.registered = True

    def close(self, lib=None) -> None:
        if self.registered and lib is not None:
            lib.pp_host_unregister(self.base)
            self.registered = False
        self.words = None
        self._anchor = None
        self.base = 0
        try:
            self.mm.close()
        except BufferError:  # a view still alive: the mapping goes with the process
            pass


class CudaStageIO:
    """A shard's resident buffers and stream, the inbox it exports and the outbox it opened;
    events for the timed window."""

    def __init__(self, shard, width: int):
        self.shard, self.width, self.device = shard, width, shard.device
        self.first, self.last = shard.first, shard.last
        self.stream = torch.cuda.ExternalStream(shard.stream(),
                                                device=torch.device("cuda", self.device))
        self._t0 = torch.cuda.Event(enable_timing=True)
        self._t1 = torch.cuda.Event(enable_timing=True)
        self.mem = None
        self.rank = 0

    def data_bytes(self) -> int:
        return 0

    def export_inbox(self) -> bytes:
        return self.shard.inbox_export(RING)

    def open_outbox(self, handle: bytes) -> None:
        self.shard.outbox_open(handle, RING)

    def attach(self, mem: ChainMemory) -> None:
        from . import _lib
        self.mem = mem
        mem.register(_lib.load())

    def detach(self) -> None:
        from . import _lib
        self.mem.close(_lib.load())

    def set_step(self, pos: int, m: int, tokens, drafts, flags: int) -> None:
        self.shard.set_step(pos, m, tokens=tokens, drafts=drafts, flags=flags)

    def step(self) -> None:
        self.shard.step_device(self.width)

    def recv(self, k: int, m: int) -> None:
        self.shard.recv(k, m)

    def send(self, link: int, k: int, m: int, info: int) -> None:
        mem = self.mem
        self.shard.send(k, m, mem.base + mem.mail(link, k) * 4, info)

    def send_result(self, k: int) -> None:
        mem = self.mem
        self.shard.send_result(mem.base + mem.res_off + (k % RING) * RES_SLOT,
                               mem.base + mem.mail(mem.world - 1, k) * 4, k + 1)

    def can_prefill(self) -> bool:
        return self.shard.can_prefill()

    def export_prefill(self) -> bytes:
        return self.shard.prefill_export()

    def open_prefill(self, handle: bytes) -> None:
        self.shard.prefill_open(handle)

    def prefill_first(self, pos: int, tokens) -> None:
        self.shard.prefill(pos, tokens)

    def prefill_rows(self, pos: int, t: int) -> None:
        self.shard.prefill_hidden(pos, t)

    def prefill_send(self, link: int, k: int, t: int, info: int) -> None:
        mem = self.mem
        self.shard.prefill_send(k, t, mem.base + mem.mail(link, k) * 4, info)

    def mark_start(self) -> None:
        self._t0.record(self.stream)

    def mark_end(self) -> None:
        self._t1.record(self.stream)

    def elapsed_ms(self) -> float:
        return self._t0.elapsed_time(self._t1)

    def finish(self) -> None:
        torch.cuda.synchronize(self.device)

    def capacity(self) -> int:
        return self.shard.capacity()

    def chunk_size(self) -> int:
        return self.shard.chunk_size()

    def range(self) -> Tuple[int, int]:
        return self.shard.range()

    def model_layers(self) -> int:
        return self.shard.model_layers()

    def hello(self, next_layer: int) -> dict:
        return self.shard.hello(next_layer)


class HostStageIO:
    """The same interface over host tensors and a host `stage` object with `step(hdr, hid,
    res)`; its inbox is a region of the shared memory. Runs the protocol under gloo without a
    GPU (tests of the multi-process logic)."""

    def __init__(self, stage, width: int, hidden: int, first: bool, last: bool,
                 capacity: int = 4096, chunk: int = 8, layer_range=(0, 1), model_layers=1,
                 model: str = "host-stand-in"):
        self.stage, self.width, self.hidden = stage, width, hidden
        self.first, self.last = first, last
        self._range, self._layers, self._model = tuple(layer_range), model_layers, model
        self.hid = torch.zeros(width * hidden, dtype=torch.float32)
        self.hdr = torch.zeros(HDR_INTS, dtype=torch.int32)
        self.res = torch.zeros(RES_INTS, dtype=torch.int32)
        self._cap, self._chunk = capacity, chunk
        self._t0 = self._t1 = 0.0
        self.mem = None
        self.rank = 0

    def data_bytes(self) -> int:
        return HDR_INTS * 4 + self.width * self.hidden * 4

    def export_inbox(self) -> bytes:
        return b""

    def open_outbox(self, handle: bytes) -> None:
        pass

    def attach(self, mem: ChainMemory) -> None:
        self.mem = mem

    def detach(self) -> None:
        self.mem.close()

    def _slot(self, link: int, k: int) -> Tuple[np.ndarray, np.ndarray]:
        mem = self.mem
        off = mem.data_off + (link * RING + k % RING) * mem.data_bytes
        hdr = np.ndarray((HDR_INTS,), np.int32, mem.mm, off)
        hid = np.ndarray((self.width * self.hidden,), np.float32, mem.mm, off + HDR_INTS * 4)
        return hdr, hid

    def set_step(self, pos: int, m: int, tokens, drafts, flags: int) -> None:
        self.hdr.zero_()
        self.hdr[0], self.hdr[1], self.hdr[2], self.hdr[3] = pos, m, len(drafts), flags
        self.hdr[4:4 + m] = torch.tensor(tokens, dtype=torch.int32)
        if drafts:
            self.hdr[20:20 + len(drafts)] = torch.tensor(drafts, dtype=torch.int32)

    def step(self) -> None:
        self.stage.step(self.hdr, self.hid, self.res)

    def recv(self, k: int, m: int) -> None:
        hdr, hid = self._slot(self.rank - 1, k)
        self.hdr.copy_(torch.from_numpy(hdr.copy()))
        self.hid.copy_(torch.from_numpy(hid.copy()))

    def send(self, link: int, k: int, m: int, info: int) -> None:
        mem = self.mem
        if m:
            hdr, hid = self._slot(link, k)
            hdr[:] = self.hdr.numpy()
            hid[:] = self.hid.numpy()
        i = mem.mail(link, k)
        mem.words[i + 1] = info
        mem.words[i] = (k + 1) & 0xFFFFFFFF

    def send_result(self, k: int) -> None:
        mem = self.mem
        mem.result_ints(k)[:] = self.res.numpy()
        mem.words[mem.mail(mem.world - 1, k)] = (k + 1) & 0xFFFFFFFF

    def can_prefill(self) -> bool:
        return hasattr(self.stage, "prefill")

    def export_prefill(self) -> bytes:
        return b""

    def open_prefill(self, handle: bytes) -> None:
        pass

    def _rows(self, rank: int) -> np.ndarray:
        mem = self.mem
        off = mem.data_off + (mem.world - 1) * RING * mem.data_bytes + rank * self._pf_bytes()
        return np.ndarray((PREFILL_MAX, self.hidden), np.float32, mem.mm, off)

    def _pf_bytes(self) -> int:
        return PREFILL_MAX * self.hidden * 4

    def extra_bytes(self, world: int) -> int:
        return world * self._pf_bytes()

    def prefill_first(self, pos: int, tokens) -> None:
        self.stage.prefill(pos, np.asarray(tokens), self._rows(self.rank))

    def prefill_rows(self, pos: int, t: int) -> None:
        self.stage.prefill(pos, None, self._rows(self.rank)[:t])

    def prefill_send(self, link: int, k: int, t: int, info: int) -> None:
        mem = self.mem
        self._rows(self.rank + 1)[:t] = self._rows(self.rank)[:t]
        i = mem.mail(link, k)
        mem.words[i + 1] = info
        mem.words[i] = (k + 1) & 0xFFFFFFFF

    def mark_start(self) -> None:
        self._t0 = time.perf_counter()

    def mark_end(self) -> None:
        self._t1 = time.perf_counter()

    def elapsed_ms(self) -> float:
        return (self._t1 - self._t0) * 1e3

    def finish(self) -> None:
        pass

    def capacity(self) -> int:
        return self._cap

    def chunk_size(self) -> int:
        return self._chunk

    def range(self) -> Tuple[int, int]:
        return self._range

    def model_layers(self) -> int:
        return self._layers

    def hello(self, next_layer: int) -> dict:
        return {"model": self._model, "next_layer": next_layer, "max_seq": self._cap,
                "chunk": self._chunk, "taps": []}


def negotiate(io, rank: int, world: int) -> None:
    """The session handshake (src/transport.rs:299-358) before any frame moves: every rank
    publishes the hello it sends downstream (its range end) and the one it expects from
    upstream (its range start); every link is checked, and the chain must end at the model's
    last layer (the head's Ready check). All ranks take this one collective step and raise the
    same HandshakeError, so a mismatched session ends everywhere before the first chunk."""
    a, b = io.range()
    mine = {"range": (a, b), "down": io.hello(b), "up": io.hello(a),
            "layers": io.model_layers()}
    every = [None] * world
    dist.all_gather_object(every, mine)
    # Each hello carries the session's tapped layers: every stage's own, ascending.
    taps = sorted({l for v in every for l in v["up"]["taps"]})
    errors = []
    for r in range(1, world):
        try:
            check_link(every[r - 1]["range"], dict(every[r - 1]["down"], taps=taps),
                       every[r]["range"], dict(every[r]["up"], taps=taps))
        except HandshakeError as e:
            errors.append(str(e))
    end, layers = every[-1]["range"][1], every[-1]["layers"]
    if end != layers:
        errors.append(f"the chain ends at layer {end}, but the model has {layers}")
    if errors:
        raise HandshakeError("; ".join(errors))


def connect(io, rank: int, world: int) -> ChainMemory:
    """Set up the links (collective: every rank, in the same order): the handshake, the shared
    memory (made by rank 0; its name and the inbox handles gathered), and each stage's outbox
    opened on the next stage's inbox."""
    negotiate(io, rank, world)
    io.rank = rank
    can = io.can_prefill()
    mine = {"inbox": io.export_inbox() if rank > 0 else b"", "data": io.data_bytes(),
            "extra": io.extra_bytes(world) if hasattr(io, "extra_bytes") else 0,
            "prefill": io.export_prefill() if rank > 0 and can else b"", "can": can,
            "path": f"/dev/shm/potpori_chain_{uuid.uuid4().hex}" if rank == 0 else ""}
    every = [None] * world
    dist.all_gather_object(every, mine)
    path = every[0]["path"]
    data = max(v["data"] for v in every)
    extra = max(v["extra"] for v in every)
    mem = ChainMemory(world, path, True, data, extra) if rank == 0 else None
    dist.barrier()
    if rank != 0:
        mem = ChainMemory(world, path, False, data, extra)
    io.attach(mem)
    mem.can_prefill = all(v["can"] for v in every)
    if rank + 1 < world:
        io.open_outbox(every[rank + 1]["inbox"])
        if mem.can_prefill:
            io.open_prefill(every[rank + 1]["prefill"])
    dist.barrier()
    if rank == 0:  # every rank has mapped it: the name can go
        os.unlink(path)
    return mem


def run_stage(shard, rank: int, world: int, width: int, io=None) -> float:
    """Serve as stage `rank` (1 <= rank < world) until the session ends. Returns the time (ms)
    between the timed-window marks, measured on this stage's stream (0 without both marks)."""
    io = io or CudaStageIO(shard, width)
    mem = connect(io, rank, world)
    started = ended = False
    k = 0
    try:
        while True:
            info = mem.wait(rank - 1, k)
            m, flags = info & 0xFF, info >> 8
            if flags & FLAG_PREFILL:
                # The prompt's rows through this stage in one pass, then on to the next
                # (src/node.rs:538-566 streams them in chunk-sized frames instead).
                pos, t = (int(v) for v in mem.params(rank - 1, k))
                io.prefill_rows(pos, t)
                if not io.last:
                    mem.params(rank, k)[:] = (pos, t)
                    io.prefill_send(rank, k, t, info)
                k += 1
                continue
            if flags & FLAG_WINDOW_START and not started:
                io.mark_start()
                started = True
            if flags & FLAG_WINDOW_END and started and not ended:
                io.mark_end()
                ended = True
            if m == 0:
                if not io.last:
                    io.send(rank, k, 0, info)
                if flags & FLAG_MARKS:
                    k += 1
                    continue
                break
            io.recv(k, m)
            io.step()
            if io.last:
                io.send_result(k)
            else:
                io.send(rank, k, m, info)
            k += 1
        io.finish()
    finally:
        io.detach()
    return io.elapsed_ms() if (started and ended) else 0.0


class DistChain:
    """The head's view of the multi-process chain (PipelinedChain / TargetChain)."""

    def __init__(self, stage0, world: int, width: int, io=None):
        self.io = io or CudaStageIO(stage0, width)
        assert self.io.first and not self.io.last and world > 1
        self.world, self.width = world, width
        self.mem = connect(self.io, 0, world)
        self.inflight: deque = deque()
        self.seq = 0    # next chunk to send
        self.done = 0   # next chunk whose result is read
        self.capacity_ = self.io.capacity()
        self.chunk = self.io.chunk_size() or width
        self.pending_flags = 0
        self.submitted = 0
        self.closed = False

    def capacity(self) -> int:
        return self.capacity_

    def mark(self, flags: int) -> None:
        """Put flag bits on the next chunk sent (timed-window marks)."""
        self.pending_flags |= flags

    def send_marks(self) -> None:
        """Send the pending flag bits now, in a message without rows that every stage passes
        on after the chunks sent before it (so a stage's timed window ends with its share of
        those chunks, not with the next chunk)."""
        if self.pending_flags:
            self.io.send(0, self.seq, 0, (self.pending_flags | FLAG_MARKS) << 8)
            self.pending_flags = 0
            self.seq += 1

    def submit(self, pos: int, cur: int, drafts: List[int]) -> None:
        # A slot of every inbox is reused RING chunks later; with at most RING / 2 chunks
        # between the head and its results, every stage has long read it by then.
        if self.seq - self.done >= RING // 2:
            raise ChainError("too many chunks in flight")
        tokens = [cur] + list(drafts)
        m = len(tokens)
        io = self.io
        io.set_step(pos, m, tokens, list(drafts), self.pending_flags)
        io.step()
        io.send(0, self.seq, m, m | (self.pending_flags << 8))
        self.pending_flags = 0
        self.inflight.append((self.seq, m))
        self.seq += 1
        self.submitted += 1

    def poll(self) -> List[int]:
        k, m = self.inflight.popleft()
        self.mem.wait(self.world - 1, k)
        r = self.mem.result_ints(k).tolist()
        self.done = k + 1
        if r[RES_NONFINITE] or r[RES_STATUS] & 8:
            raise NonFiniteLogits("the shard produced missing or non-finite logits")
        if r[RES_STATUS] & 5:
            raise RuntimeError(f"chain step failed (status {r[RES_STATUS]})")
        return r[:m]

    def prefill(self, prompt: List[int], one_pass: bool = True) -> int:
        """The greedy pick after the prompt. When every stage can (Shard.can_prefill) and the
        prompt has at most 2049 tokens, each stage writes the K/V rows of all but the last token
        in one pass and sends its output rows on (one prefill message per link); the last token
        is then submitted as the step that yields the pick. Otherwise, or with one_pass=False,
        the prompt goes in chunk-sized steps, as the reference streams it
        (src/node.rs:538-566)."""
        n = len(prompt) - 1
        if one_pass and 0 < n <= PREFILL_MAX and self.mem.can_prefill:
            while self.inflight:
                self.poll()
            self.io.prefill_first(0, prompt[:-1])
            self.mem.params(0, self.seq)[:] = (0, n)
            self.io.prefill_send(0, self.seq, n, FLAG_PREFILL << 8)
            self.seq += 1
            self.submit(n, prompt[-1], [])
            return self.poll()[-1]
        pos = 0
        while pos < len(prompt):
            take = self.chunk if len(prompt) - pos >= self.chunk else 1
            piece = prompt[pos:pos + take]
            self.submit(pos, piece[0], piece[1:])
            pos += take
            while len(self.inflight) >= RING // 2:
                self.poll()
        last = 0
        while self.inflight:
            last = self.poll()[-1]
        return last

    def verify(self, pos: int, cur: int, drafts: List[int]) -> List[int]:
        self.submit(pos, cur, drafts)
        return self.poll()

    def is_eos(self, t: int) -> bool:
        return is_eos(t)

    def stop(self) -> None:
        """End the session on every stage (a chunk with m = 0 carries any pending marks)."""
        if self.closed:
            return
        while self.inflight:
            self.poll()
        self.io.send(0, self.seq, 0, self.pending_flags << 8)
        self.pending_flags = 0
        self.io.finish()
        self.io.detach()
        self.closed = True
