"""The multi-process pipeline protocol (potpori_b200/distchain.py) on CPU: gloo ranks for the
setup, host stand-ins for the shards (HostStageIO) whose inboxes and mailboxes live in the
chain's shared memory, no GPU.

Checks what the chain of src/node.rs:242-342,466-535 must keep when its stages are separate
processes: every chunk's header and hidden rows go rank r -> r+1 in order, the last rank's
result comes straight back to rank 0, several chunks are in flight at once (the depth of
src/specpipe.rs:83-127), prefill feeds the prompt in 8-row chunks and single rows (or, when
every stage can, all but its last token as one prefill message per link), the timed window
marks ride on the headers to every stage, a non-finite result surfaces at the head as
NonFiniteLogits, and the stop header ends every rank.
"""
import multiprocessing as mp
import os
import socket

import pytest
import torch

HIDDEN = 16
WIDTH = 8


class FakeStage:
    """Stage r adds 1 to column 0 of every row; the first writes the tokens there first; the
    last returns column 0 as the picks. So a chunk's picks are its tokens + world; token 999
    makes the last stage report a non-finite row."""

    def __init__(self, first: bool, last: bool):
        self.first, self.last = first, last

    def step(self, hdr, hid, res):
        m = int(hdr[1])
        h = hid.view(-1, HIDDEN)
        toks = hdr[4:4 + m].float()
        if self.first:
            h[:m, 0] = toks
        h[:m, 0] += 1.0
        if self.last:
            res.zero_()
            res[:m] = h[:m, 0].to(torch.int32)
            if bool((res[:m] > 900).any()):
                res[48] = 1


class PrefillStage(FakeStage):
    """FakeStage that also takes a whole prompt in one pass: the first writes the tokens into
    column 0 of its output rows, every stage adds 1, and each records what it saw."""

    def __init__(self, first: bool, last: bool):
        super().__init__(first, last)
        self.prefilled = []

    def prefill(self, pos, tokens, rows):
        if self.first:
            t = len(tokens)
            rows[:t, 0] = tokens
        else:
            t = len(rows)
        rows[:t, 0] += 1.0
        self.prefilled.append((pos, t, rows[:t, 0].astype(int).tolist()))


def _worker(rank: int, world: int, port: int, one_pass: bool, q) -> None:
    import torch.distributed as dist
    from potpori_b200.distchain import (FLAG_WINDOW_END, FLAG_WINDOW_START, DistChain,
                                        HostStageIO, run_stage)
    from potpori_b200.target import NonFiniteLogits
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kind = PrefillStage if one_pass else FakeStage
        stage = kind(rank == 0, rank == world - 1)
        io = HostStageIO(stage, WIDTH, HIDDEN, first=rank == 0, last=rank == world - 1,
                         capacity=256, chunk=WIDTH, layer_range=(rank, rank + 1),
                         model_layers=world)
        if rank != 0:
            q.put((rank, "ms", run_stage(None, rank, world, WIDTH, io=io)))
            q.put((rank, "prefilled", getattr(stage, "prefilled", None)))
            return
        chain = DistChain(None, world, WIDTH, io=io)
        # 19 tokens: two 8-row chunks, then three single rows; or one prefill message of 18
        # rows, then the last token as a step
        prompt = list(range(10, 29))
        assert chain.mem.can_prefill == one_pass
        assert chain.prefill(prompt) == prompt[-1] + world
        # three chunks in flight, then read in order
        chunks = [(19, 40, [41, 42, 43]), (23, 50, []), (24, 60, [61, 62, 63, 64, 65, 66, 67])]
        chain.mark(FLAG_WINDOW_START)
        for pos, cur, ds in chunks:
            chain.submit(pos, cur, ds)
        chain.mark(FLAG_WINDOW_END)
        chain.send_marks()  # a message without rows: every stage ends its window on it
        chain.submit(32, 70, [71])
        for _, cur, ds in chunks + [(32, 70, [71])]:
            assert chain.poll() == [t + world for t in [cur] + ds]
        assert chain.verify(34, 80, [81, 82]) == [80 + world, 81 + world, 82 + world]
        try:
            chain.verify(37, 990, [])
            raise AssertionError("a non-finite result was not reported")
        except NonFiniteLogits:
            pass
        assert chain.submitted == (1 if one_pass else 2 + 3) + 3 + 1 + 1 + 1
        chain.stop()
        q.put((0, "ok", True))
    except BaseException as e:  # reported to the test process
        q.put((rank, "error", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("one_pass", [False, True])
@pytest.mark.parametrize("world", [2, 3])
def test_pipeline_protocol_over_gloo(world, one_pass):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, one_pass, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    got = {}
    while not q.empty():
        r, k, v = q.get()
        got[(r, k)] = v
    errors = {k: v for k, v in got.items() if k[1] == "error"}
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert got[(0, "ok")] is True
    # every stage saw both window marks
    for r in range(1, world):
        assert got[(r, "ms")] > 0.0
    # one prefill message of rows 0..17 through every stage, each adding 1 to column 0
    for r in range(1, world):
        want = [(0, 18, [t + r + 1 for t in range(10, 28)])] if one_pass else None
        assert got[(r, "prefilled")] == want, (r, got[(r, "prefilled")])


def _hello_worker(rank: int, world: int, port: int, bad: str, q) -> None:
    import torch.distributed as dist
    from potpori_b200.chain import HandshakeError
    from potpori_b200.distchain import DistChain, HostStageIO, run_stage
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cap, chunk, rng, layers = 256, WIDTH, (rank, rank + 1), world
        if rank == world - 1:  # the last stage is set up differently
            if bad == "chunk":
                chunk = 4
            elif bad == "max_seq":
                cap = 512
            elif bad == "boundary":
                rng = (rank + 1, rank + 2)
                layers = world + 1
            elif bad == "short":
                layers = world + 1
        io = HostStageIO(FakeStage(rank == 0, rank == world - 1), WIDTH, HIDDEN,
                         first=rank == 0, last=rank == world - 1, capacity=cap, chunk=chunk,
                         layer_range=rng, model_layers=layers)
        try:
            if rank == 0:
                DistChain(None, world, WIDTH, io=io)
            else:
                run_stage(None, rank, world, WIDTH, io=io)
            q.put((rank, "refused", None))
        except HandshakeError as e:
            q.put((rank, "refused", str(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bad,words", [("chunk", "chunk 8 (this node has 4)"),
                                       ("max_seq", "max_seq 256 (this node has 512)"),
                                       ("boundary", "next layer 2 (this node starts at 3)"),
                                       ("short", "the chain ends at layer 3, but the model has 4")])
def test_handshake_refuses_a_mismatched_session(bad, words):
    """src/transport.rs:299-358: before any frame moves, every link compares the upstream
    stage's hello with what the downstream stage serves, and a chain that stops short of the
    model's last layer is refused; every rank gets the same error, naming what differs."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_hello_worker, args=(r, world, port, bad, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    got = {}
    while not q.empty():
        r, k, v = q.get()
        got[r] = v
    assert sorted(got) == list(range(world)), got
    for r in range(world):
        assert got[r] is not None and words in got[r], (r, got[r])
