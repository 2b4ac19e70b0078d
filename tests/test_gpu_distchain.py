"""The multi-process chain on the device (potpori_b200/distchain.py): pipeline stages in
separate processes joined by CUDA IPC copies and mailboxes in shared host memory.

Two or three processes share one GPU here (with more GPUs each takes its own; the protocol
has no kernel that waits on another process, so the stages may share a device). The chain of
Qwen3-0.6B layer ranges (seed 0) must give the picks, top-1 logits and accept compare of one
whole-model shard for the prompt's chunks, and the depth-4 pipelined driver of
src/specpipe.rs over it, with the same weights as draft, the whole shard's committed stream
(src/node.rs:242-342,466-535 head/middle/tail, direct return of the result to the head).
A one-pass prefill (one prefill message per link) must then give the whole shard's picks for
the same chunks wherever its top-2 gap is at least 1e-3.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NEW = 16
TIE_GAP = 1e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, ranges, q) -> None:
    import torch
    import torch.distributed as dist

    import oracle
    from potpori_b200.config import QWEN3_0_6B
    from potpori_b200.distchain import DistChain, run_stage
    from potpori_b200.shard import Shard
    from potpori_b200.specdecode import SpecConfig
    from potpori_b200.specpipe import PipelinedDriver
    from potpori_b200.target import IncrementalDraft, QwenTarget

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg, cap = QWEN3_0_6B, 256
    try:
        stage = Shard.random(cfg, ranges[rank], cap, 8, seed=0, device=dev)
        if rank != 0:
            run_stage(stage, rank, world, 8)
            stage.close()
            q.put((rank, "ok", None))
            return
        whole = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=0, device=dev)
        chain = DistChain(stage, world, 8)
        prompt = np.random.default_rng(11).integers(0, cfg.vocab_size, 29).tolist()
        # The prompt in chunk-sized steps, then three chunks in flight at once.
        got_first = chain.prefill(prompt, one_pass=False)
        pos, want_first = 0, None
        while pos < len(prompt):
            take = 8 if len(prompt) - pos >= 8 else 1
            want_first = whole.verify_tokens(pos, prompt[pos:pos + take]).argmax[-1]
            pos += take
        assert got_first == want_first, (got_first, want_first)
        rng = np.random.default_rng(3)
        chunks = [(29 + 8 * i, [int(t) for t in rng.integers(0, cfg.vocab_size, 8)]) for i in range(3)]
        for p, toks in chunks:
            chain.submit(p, toks[0], toks[1:])
        for p, toks in chunks:
            got = chain.poll()
            want = whole.verify_tokens(p, toks)
            assert got == want.argmax, (p, got, want.argmax)
        # The pipelined driver over the chain, the whole shard's own weights as draft.
        whole.reset()
        draft = IncrementalDraft(QwenTarget(Shard.random(cfg, (0, cfg.layers), cap, 8, seed=0,
                                                         device=dev)), 8)
        drv = PipelinedDriver(draft, chain, prompt, SpecConfig(7, NEW), 4)
        drv.start()
        while drv.step():
            pass
        ref = QwenTarget(whole)
        cur = ref.prefill(prompt, one_pass=False)
        want, p = [cur], len(prompt)
        while len(want) < NEW:
            cur = ref.verify(p, cur, [])[0]
            want.append(cur)
            p += 1
        assert drv.out == want, (drv.out, want)
        assert drv.stats().toks_per_traversal() > 2  # the drafts were accepted
        # One pass per stage over the same cache rows (one prefill message per link), then the
        # three chunks: the whole shard's picks wherever its top-2 gap is at least 1e-3.
        assert chain.mem.can_prefill
        whole.reset()
        pos = 0
        while pos < len(prompt):
            take = 8 if len(prompt) - pos >= 8 else 1
            res = whole.verify_tokens(pos, prompt[pos:pos + take], logits=True)
            pos += take
        first = chain.prefill(prompt)
        t1, t2 = oracle.top2(res.logits[-1])
        if t1 - t2 >= TIE_GAP:
            assert first == res.argmax[-1]
        for p, toks in chunks:
            chain.submit(p, toks[0], toks[1:])
        for p, toks in chunks:
            got = chain.poll()
            want = whole.verify_tokens(p, toks, logits=True)
            for r in range(len(toks)):
                t1, t2 = oracle.top2(want.logits[r])
                if t1 - t2 >= TIE_GAP:
                    assert got[r] == want.argmax[r], (p, r)
        chain.stop()
        draft.model.shard.close()
        whole.close()
        stage.close()
        q.put((rank, "ok", None))
    except BaseException as e:  # reported to the test process
        q.put((rank, "error", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ranges", [[(0, 14), (14, 28)], [(0, 9), (9, 19), (19, 28)]])
def test_multiprocess_chain_matches_the_whole_model(gpu, ranges):
    world = len(ranges)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, ranges, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
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
    assert all((r, "ok") in got for r in range(world))
