"""Pipeline stages in separate processes, one per GPU, joined by NCCL point-to-point transfers
of the shards' own device buffers (torch.distributed is the plumbing).

This replaces the reference's chain over QUIC (head ChainLink::send_chunk -> relay_middle ->
serve_tail -> VerifyResult back, src/node.rs:242-342,466-535, src/transport.rs:425-489):
 * rank 0 (the head) runs the draft model, stage 0 and the driver; every chunk it submits
   travels as two messages, the 144-byte step header (position, rows, tokens, drafts) and
   the chunk's F32 hidden rows, from rank r to rank r+1, device buffer to device buffer;
 * every other rank loops: receive header + hidden into its shard's input buffers, run the
   step (graph replay, no host involvement), forward to the next rank;
 * the last rank computes the greedy picks and the accept compare on the device and sends
   the 208-byte result straight back to rank 0 (a direct return instead of a relay).
Ordering is by streams only: NCCL transfers are enqueued on each shard's stream (via
torch.cuda.ExternalStream), so nothing waits on the host except the head's poll and each
stage's look at the header it just received (to notice the end of the session).
A header with m = 0 ends the session; flag bits mark the benchmark's timed window.

The protocol (run_stage, DistChain) talks to its stage through a small I/O object:
CudaStageIO (a Shard's device buffers and stream: the product path) or any object with the
same methods, such as a host-memory stand-in that lets the protocol run under gloo on CPU.
"""
from __future__ import annotations

import contextlib
import time
from collections import deque
from typing import List, Tuple

import torch
import torch.distributed as dist

from .chain import HandshakeError, check_link
from .config import is_eos
from .target import NonFiniteLogits

HDR_INTS = 36   # StepDesc: pos, m, n_drafts, flags, tokens[16], drafts[16]
RES_INTS = 52   # StepResult: argmax[16], top1[16], top2[16], nonfinite_rows, n_acc, corr, status
RES_NONFINITE, RES_STATUS = 48, 51
RING = 64
FLAG_WINDOW_START = 2
FLAG_WINDOW_END = 4


class Links:
    """One process group per link, so transfers on different links never queue behind each
    other: NCCL runs the ops of one communicator in order, so with a single group the head's
    receive of chunk k's result (posted first, completing only after the whole traversal)
    would hold back the send of chunk k+1, and the chunks could not overlap in the pipeline.
    fwd[r]: rank r -> r + 1; ret: the last rank -> rank 0. Every rank must build it, in the
    same order (dist.new_group is collective)."""

    def __init__(self, world: int):
        self.fwd = [dist.new_group([r, r + 1]) for r in range(world - 1)]
        self.ret = dist.new_group([0, world - 1])


class _DevArray:
    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


def device_tensor(ptr: int, n: int, dtype, device: int) -> torch.Tensor:
    ts = {torch.float32: "<f4", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_DevArray(ptr, n, ts), device=torch.device("cuda", device))


class CudaStageIO:
    """A shard's resident buffers (hidden rows, step header, step result) as tensors, its
    stream as the ordering of every transfer, and events for the timed window."""

    def __init__(self, shard, width: int):
        hid, hdr, res = shard.buffers()
        dev = shard.device
        self.shard, self.width, self.device = shard, width, dev
        self.first, self.last = shard.first, shard.last
        self.hid = device_tensor(hid, width * shard.cfg.hidden, torch.float32, dev)
        self.hdr = device_tensor(hdr, HDR_INTS, torch.int32, dev)
        self.res = device_tensor(res, RES_INTS, torch.int32, dev)
        self.stream = torch.cuda.ExternalStream(shard.stream(), device=torch.device("cuda", dev))
        self._host_hdr = torch.empty(HDR_INTS, dtype=torch.int32, pin_memory=True)
        self._host_res = torch.empty(RES_INTS, dtype=torch.int32, pin_memory=True)
        self._seen = torch.cuda.Event()
        self._t0 = torch.cuda.Event(enable_timing=True)
        self._t1 = torch.cuda.Event(enable_timing=True)

    def ordered(self):
        return torch.cuda.stream(self.stream)

    def read_header(self) -> Tuple[int, int]:
        """(rows, flags) of the header that just arrived (waits for it on the host)."""
        self._host_hdr.copy_(self.hdr, non_blocking=True)
        self._seen.record(self.stream)
        self._seen.synchronize()
        return int(self._host_hdr[1]), int(self._host_hdr[3])

    def set_step(self, pos: int, m: int, tokens, drafts, flags: int) -> None:
        self.shard.set_step(pos, m, tokens=tokens, drafts=drafts, flags=flags)

    def step(self) -> None:
        self.shard.step_device(self.width, stream=self.shard.stream())

    def mark_start(self) -> None:
        self._t0.record(self.stream)

    def mark_end(self) -> None:
        self._t1.record(self.stream)

    def elapsed_ms(self) -> float:
        return self._t0.elapsed_time(self._t1)

    def finish(self) -> None:
        torch.cuda.synchronize(self.device)

    def result_slots(self, n: int) -> torch.Tensor:
        return torch.zeros((n, RES_INTS), dtype=torch.int32, device=torch.device("cuda", self.device))

    def fetch(self, slot_row: torch.Tensor) -> List[int]:
        self._host_res.copy_(slot_row, non_blocking=True)
        self.stream.synchronize()
        return self._host_res.tolist()

    def stop_header(self, flags: int) -> torch.Tensor:
        stop = torch.zeros(HDR_INTS, dtype=torch.int32, device=torch.device("cuda", self.device))
        stop[3] = flags
        return stop

    def drain(self) -> None:
        self.stream.synchronize()

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
    res)`: runs the protocol under gloo without a GPU (tests of the multi-process logic)."""

    def __init__(self, stage, width: int, hidden: int, first: bool, last: bool,
                 capacity: int = 4096, chunk: int = 8, layer_range=(0, 1), model_layers=1,
                 model: str = "host-stand-in"):
        self.stage, self.width = stage, width
        self.first, self.last = first, last
        self._range, self._layers, self._model = tuple(layer_range), model_layers, model
        self.hid = torch.zeros(width * hidden, dtype=torch.float32)
        self.hdr = torch.zeros(HDR_INTS, dtype=torch.int32)
        self.res = torch.zeros(RES_INTS, dtype=torch.int32)
        self._cap, self._chunk = capacity, chunk
        self._t0 = self._t1 = 0.0

    def ordered(self):
        return contextlib.nullcontext()

    def read_header(self) -> Tuple[int, int]:
        return int(self.hdr[1]), int(self.hdr[3])

    def set_step(self, pos: int, m: int, tokens, drafts, flags: int) -> None:
        self.hdr.zero_()
        self.hdr[0], self.hdr[1], self.hdr[2], self.hdr[3] = pos, m, len(drafts), flags
        self.hdr[4:4 + m] = torch.tensor(tokens, dtype=torch.int32)
        if drafts:
            self.hdr[20:20 + len(drafts)] = torch.tensor(drafts, dtype=torch.int32)

    def step(self) -> None:
        self.stage.step(self.hdr, self.hid, self.res)

    def mark_start(self) -> None:
        self._t0 = time.perf_counter()

    def mark_end(self) -> None:
        self._t1 = time.perf_counter()

    def elapsed_ms(self) -> float:
        return (self._t1 - self._t0) * 1e3

    def finish(self) -> None:
        pass

    def result_slots(self, n: int) -> torch.Tensor:
        return torch.zeros((n, RES_INTS), dtype=torch.int32)

    def fetch(self, slot_row: torch.Tensor) -> List[int]:
        return slot_row.tolist()

    def stop_header(self, flags: int) -> torch.Tensor:
        stop = torch.zeros(HDR_INTS, dtype=torch.int32)
        stop[3] = flags
        return stop

    def drain(self) -> None:
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


def run_stage(shard, rank: int, world: int, width: int, links: Links, io=None) -> float:
    """Serve as stage `rank` (1 <= rank < world) until the session ends. Returns the time (ms)
    between the timed-window marks, measured on this stage's stream (0 without both marks)."""
    io = io or CudaStageIO(shard, width)
    negotiate(io, rank, world)
    started = ended = False
    with io.ordered():
        while True:
            w1 = dist.irecv(io.hdr, rank - 1, group=links.fwd[rank - 1])
            w2 = dist.irecv(io.hid, rank - 1, group=links.fwd[rank - 1])
            w1.wait()
            w2.wait()
            m, flags = io.read_header()
            if flags & FLAG_WINDOW_START and not started:
                io.mark_start()
                started = True
            if flags & FLAG_WINDOW_END and started and not ended:
                io.mark_end()
                ended = True
            if m > 0:
                io.step()
            if io.last:
                if m == 0:
                    break
                w = dist.isend(io.res, 0, group=links.ret)
                w.wait()
            else:
                w1 = dist.isend(io.hdr, rank + 1, group=links.fwd[rank])
                w2 = dist.isend(io.hid, rank + 1, group=links.fwd[rank])
                w1.wait()
                w2.wait()
                if m == 0:
                    break
    io.finish()
    return io.elapsed_ms() if (started and ended) else 0.0


class DistChain:
    """The head's view of the multi-process chain (PipelinedChain / TargetChain)."""

    def __init__(self, stage0, world: int, width: int, links: Links, io=None):
        self.io = io or CudaStageIO(stage0, width)
        assert self.io.first and not self.io.last and world > 1
        negotiate(self.io, 0, world)
        self.world, self.width, self.links = world, width, links
        self.slots = self.io.result_slots(RING)
        self.inflight: deque = deque()
        self.slot = 0
        self.capacity_ = self.io.capacity()
        self.chunk = self.io.chunk_size() or width
        self.pending_flags = 0
        self.submitted = 0

    def capacity(self) -> int:
        return self.capacity_

    def mark(self, flags: int) -> None:
        """Put flag bits on the next header sent (timed-window marks)."""
        self.pending_flags |= flags

    def submit(self, pos: int, cur: int, drafts: List[int]) -> None:
        tokens = [cur] + list(drafts)
        m = len(tokens)
        io = self.io
        with io.ordered():
            io.set_step(pos, m, tokens, list(drafts), self.pending_flags)
            self.pending_flags = 0
            io.step()
            w1 = dist.isend(io.hdr, 1, group=self.links.fwd[0])
            w2 = dist.isend(io.hid, 1, group=self.links.fwd[0])
            w1.wait()
            w2.wait()
            wr = dist.irecv(self.slots[self.slot], self.world - 1, group=self.links.ret)
        self.inflight.append((self.slot, m, wr))
        self.slot = (self.slot + 1) % RING
        self.submitted += 1

    def poll(self) -> List[int]:
        slot, m, wr = self.inflight.popleft()
        with self.io.ordered():
            wr.wait()
            r = self.io.fetch(self.slots[slot])
        if r[RES_NONFINITE] or r[RES_STATUS] & 8:
            raise NonFiniteLogits("the shard produced missing or non-finite logits")
        if r[RES_STATUS] & 5:
            raise RuntimeError(f"chain step failed (status {r[RES_STATUS]})")
        return r[:m]

    def prefill(self, prompt: List[int]) -> int:
        pos = 0
        while pos < len(prompt):
            take = self.chunk if len(prompt) - pos >= self.chunk else 1
            piece = prompt[pos:pos + take]
            self.submit(pos, piece[0], piece[1:])
            pos += take
            while len(self.inflight) > RING // 2:
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
        """End the session on every stage (a header with m = 0 carries any pending marks)."""
        while self.inflight:
            slot, m, wr = self.inflight.popleft()
            with self.io.ordered():
                wr.wait()
        stop = self.io.stop_header(self.pending_flags)
        with self.io.ordered():
            w1 = dist.isend(stop, 1, group=self.links.fwd[0])
            w2 = dist.isend(self.io.hid, 1, group=self.links.fwd[0])
            w1.wait()
            w2.wait()
        self.io.drain()
