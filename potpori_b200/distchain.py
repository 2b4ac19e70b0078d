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
"""
from __future__ import annotations

from collections import deque
from typing import List

import torch
import torch.distributed as dist

from .config import is_eos
from .shard import Shard
from .target import NonFiniteLogits

HDR_INTS = 36   # StepDesc: pos, m, n_drafts, flags, tokens[16], drafts[16]
RES_INTS = 52   # StepResult: argmax[16], top1[16], top2[16], nonfinite_rows, n_acc, corr, status
RING = 64
FLAG_WINDOW_START = 2
FLAG_WINDOW_END = 4


class _DevArray:
    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


def device_tensor(ptr: int, n: int, dtype, device: int) -> torch.Tensor:
    ts = {torch.float32: "<f4", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_DevArray(ptr, n, ts), device=torch.device("cuda", device))


class _Bufs:
    def __init__(self, shard: Shard, width: int):
        hid, hdr, res = shard.buffers()
        dev = shard.device
        self.hid = device_tensor(hid, width * shard.cfg.hidden, torch.float32, dev)
        self.hdr = device_tensor(hdr, HDR_INTS, torch.int32, dev)
        self.res = device_tensor(res, RES_INTS, torch.int32, dev)
        self.stream = torch.cuda.ExternalStream(shard.stream(), device=torch.device("cuda", dev))


def run_stage(shard: Shard, rank: int, world: int, width: int) -> float:
    """Serve as stage `rank` until the session ends. Returns the device time (ms) between the
    timed-window marks, measured with events on this stage's stream."""
    b = _Bufs(shard, width)
    host_hdr = torch.empty(HDR_INTS, dtype=torch.int32, pin_memory=True)
    seen = torch.cuda.Event()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    started = ended = False
    with torch.cuda.stream(b.stream):
        while True:
            w1 = dist.irecv(b.hdr, rank - 1)
            w2 = dist.irecv(b.hid, rank - 1)
            w1.wait()
            w2.wait()
            host_hdr.copy_(b.hdr, non_blocking=True)
            seen.record(b.stream)
            seen.synchronize()
            m, flags = int(host_hdr[1]), int(host_hdr[3])
            if flags & FLAG_WINDOW_START and not started:
                t_start.record(b.stream)
                started = True
            if flags & FLAG_WINDOW_END and started and not ended:
                t_end.record(b.stream)
                ended = True
            if m > 0:
                shard.step_device(width, stream=shard.stream())
            if shard.last:
                if m == 0:
                    break
                w = dist.isend(b.res, 0)
                w.wait()
            else:
                w1 = dist.isend(b.hdr, rank + 1)
                w2 = dist.isend(b.hid, rank + 1)
                w1.wait()
                w2.wait()
                if m == 0:
                    break
    torch.cuda.synchronize(shard.device)
    return t_start.elapsed_time(t_end) if (started and ended) else 0.0


class DistChain:
    """The head's view of the multi-process chain (PipelinedChain / TargetChain)."""

    def __init__(self, stage0: Shard, world: int, width: int):
        assert stage0.first and not stage0.last and world > 1
        self.stage0, self.world, self.width = stage0, world, width
        self.b = _Bufs(stage0, width)
        dev = torch.device("cuda", stage0.device)
        self.slots = torch.zeros((RING, RES_INTS), dtype=torch.int32, device=dev)
        self.host = torch.empty((RING, RES_INTS), dtype=torch.int32, pin_memory=True)
        self.inflight: deque = deque()
        self.slot = 0
        self.capacity_ = stage0.capacity()
        self.chunk = stage0.chunk_size() or width
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
        s0 = self.stage0
        with torch.cuda.stream(self.b.stream):
            s0.set_step(pos, m, tokens=tokens, drafts=drafts, flags=self.pending_flags)
            self.pending_flags = 0
            s0.step_device(self.width)
            w1 = dist.isend(self.b.hdr, 1)
            w2 = dist.isend(self.b.hid, 1)
            w1.wait()
            w2.wait()
            wr = dist.irecv(self.slots[self.slot], self.world - 1)
        self.inflight.append((self.slot, m, wr))
        self.slot = (self.slot + 1) % RING
        self.submitted += 1

    def poll(self) -> List[int]:
        slot, m, wr = self.inflight.popleft()
        with torch.cuda.stream(self.b.stream):
            wr.wait()
            self.host[slot].copy_(self.slots[slot], non_blocking=True)
        self.b.stream.synchronize()
        r = self.host[slot]
        argmax = r[:m].tolist()
        nonfinite = int(r[48])
        if nonfinite or int(r[51]) & 8:
            raise NonFiniteLogits("the shard produced missing or non-finite logits")
        if int(r[51]) & 5:
            raise RuntimeError(f"chain step failed (status {int(r[51])})")
        return argmax

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
            with torch.cuda.stream(self.b.stream):
                wr.wait()
        stop = torch.zeros(HDR_INTS, dtype=torch.int32, device=self.slots.device)
        stop[3] = self.pending_flags
        with torch.cuda.stream(self.b.stream):
            w1 = dist.isend(stop, 1)
            w2 = dist.isend(self.b.hid, 1)
            w1.wait()
            w2.wait()
        self.b.stream.synchronize()
