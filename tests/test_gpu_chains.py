"""Multi-shard chains on the device against the oracle: the workloads of configs 1 and 2 as
in-box chains of stages (LocalChain: each stage's step runs from its device buffers, the
hidden rows move by pp_shard_handoff), all stages on one GPU.

The reference's chain (ChainLink::send_chunk -> serve_middle -> serve_tail,
src/node.rs:242-342,466-535) must compute the whole model's forward: the picks after the
prompt, then verify chunks whose logits match the oracle's whole model (rel-L2 <= 1e-3, the
same greedy pick wherever the oracle's top-2 gap is at least 1e-3), fed teacher-forced with
the oracle's picks. The depth-pipelined driver of src/specpipe.rs over the chain, with the
Qwen3-0.6B draft on the device, must then commit the oracle's greedy continuation up to its
first near tie (speculative greedy decoding is lossless, whatever the draft).
"""
import numpy as np
import pytest

import oracle
from helpers import rel_l2
from potpori_b200.chain import LocalChain
from potpori_b200.shard import Shard
from potpori_b200.specdecode import SpecConfig
from potpori_b200.specpipe import PipelinedDriver
from potpori_b200.target import IncrementalDraft, QwenTarget
from potpori_b200.workload import WORKLOADS

pytestmark = pytest.mark.gpu

TIE_GAP = 1e-3


def _chain_step_logits(chain, pos, tokens):
    """One chunk through every stage of a LocalChain on the device path (set_step, step_device,
    handoff), with the last stage's logits read back."""
    m = len(tokens)
    width = max(chain.chunk, m)
    first, last = chain.stages[0], chain.stages[-1]
    first.set_step(pos, m, tokens=tokens, drafts=tokens[1:] if first.last else ())
    first.step_device(width)
    for prev, st in zip(chain.stages, chain.stages[1:]):
        st.handoff_from(prev, m)
        st.set_step(pos, m, drafts=tokens[1:] if st.last else (), want_logits=st.last)
        st.step_device(width)
    return last.read_result(m, logits=True)


def _oracle_prefill(ref, prompt, chunk):
    pos, last = 0, None
    while pos < len(prompt):
        take = chunk if len(prompt) - pos >= chunk else 1
        last = ref.forward(pos, tokens=prompt[pos:pos + take])[-1]
        pos += take
    return last


@pytest.mark.parametrize("name,n_stages", [("qwen3-1.7b-2stage", 2), ("qwen3-4b-3stage", 3)])
def test_local_chain_matches_the_oracle(gpu, name, n_stages):
    wl = WORKLOADS[name]
    cfg = wl.target
    ranges = wl.split(n_stages)
    stages = [Shard.random(cfg, r, wl.max_seq, wl.chunk, seed=wl.target_seed) for r in ranges]
    chain = LocalChain(stages)
    ref = oracle.OracleShard(cfg, 0, cfg.layers, wl.max_seq, wl.chunk)
    ref.init_random(wl.target_seed)
    prompt = wl.prompt()

    # The prompt through the chain in chunk-sized steps (src/node.rs:538-566).
    got_first = chain.prefill(prompt)
    last = _oracle_prefill(ref, prompt, wl.chunk)
    t1, t2 = oracle.top2(last)
    if t1 - t2 >= TIE_GAP:
        assert got_first == oracle.argmax(last)
    # Teacher-forced verify chunks: the oracle's pick, then seven random drafts.
    rng = np.random.default_rng(7)
    pos, cur = len(prompt), oracle.argmax(last)
    for k in range(3):
        tokens = [cur] + rng.integers(0, cfg.vocab_size, wl.gamma).tolist()
        res = _chain_step_logits(chain, pos, tokens)
        want = ref.forward(pos, tokens=tokens)
        e = rel_l2(res.logits, want)
        assert e <= 1e-3, f"chunk {k}: logits rel-L2 {e:.2e}"
        for r in range(len(tokens)):
            a, b = oracle.top2(want[r])
            if a - b >= TIE_GAP:
                assert res.argmax[r] == oracle.argmax(want[r]), (k, r)
        n = 0
        while n < wl.gamma and tokens[1 + n] == res.argmax[n]:
            n += 1
        assert res.n_accepted == n and res.correction == res.argmax[n]
        # Commit the correction and roll back the rest of the chunk (src/specpipe.rs:165-180).
        cur = oracle.argmax(want[n])
        pos += n + 1

    # The pipelined driver from a fresh session, the Qwen3-0.6B draft on the device.
    new = 12
    chain.reset()
    ref.reset()
    draft = IncrementalDraft(QwenTarget.random(wl.draft, wl.max_seq, wl.chunk, wl.draft_seed), wl.chunk)
    drv = PipelinedDriver(draft, chain, prompt, SpecConfig(wl.gamma, new), wl.depth)
    drv.start()
    while drv.step():
        pass
    last = _oracle_prefill(ref, prompt, wl.chunk)
    want, pos = [], len(prompt)
    for i in range(new):
        a, b = oracle.top2(last)
        if a - b < TIE_GAP:
            break
        want.append(oracle.argmax(last))
        last = ref.forward(pos, tokens=[want[-1]])[0]
        pos += 1
    assert drv.out[:len(want)] == want
    assert len(drv.out) == new
    draft.model.shard.close()
    for s in stages:
        s.close()
    ref.close()


def _next_steps(chain, prompt, one_pass, chunks):
    """A fresh prefill of `prompt` through the chain (one pass per stage, or chunk-sized
    steps), then the teacher-forced `chunks`; the pick after the prompt and each chunk's
    logits."""
    chain.reset()
    first = chain.prefill(prompt, one_pass=one_pass)
    return first, [_chain_step_logits(chain, p, toks).logits for p, toks in chunks]


@pytest.mark.parametrize("name,n_stages,with_oracle", [("qwen3-1.7b-2stage", 2, True),
                                                       ("qwen3-4b-3stage", 3, True),
                                                       ("qwen3-4b-8stage", 4, False),
                                                       ("qwen3-4b-8stage", 8, False)])
def test_one_pass_prefill_across_stages(gpu, name, n_stages, with_oracle):
    """Every stage writes the K/V rows of all but the prompt's last token in one pass and
    hands its output rows to the next stage. The next steps must match those after the
    chunk-sized prefill of src/node.rs:538-566 (logits rel-L2 <= 2e-4) and the oracle's
    (rel-L2 <= 1e-3), with the pick after the prompt the same wherever the top-2 gap is at
    least 1e-3. The 2,048-token prompt of the Qwen3-4B seed-3 workload is checked against the
    chunked path only (the oracle cannot run 2,047 rows of a 4B model in a test's time)."""
    wl = WORKLOADS[name]
    cfg = wl.target
    stages = [Shard.random(cfg, r, wl.max_seq, wl.chunk, seed=wl.target_seed)
              for r in wl.split(n_stages)]
    chain = LocalChain(stages)
    assert all(s.can_prefill() for s in stages)
    prompt = wl.prompt()
    n = len(prompt)
    rng = np.random.default_rng(17)
    chunks = [(n, rng.integers(0, cfg.vocab_size, wl.chunk).tolist()),
              (n + wl.chunk, rng.integers(0, cfg.vocab_size, wl.chunk).tolist()),
              (n + 2 * wl.chunk, [int(rng.integers(0, cfg.vocab_size))])]
    first1, got = _next_steps(chain, prompt, True, chunks)
    first8, want = _next_steps(chain, prompt, False, chunks)
    for k, (a, b) in enumerate(zip(got, want)):
        e = rel_l2(a, b)
        assert e <= 2e-4, f"chunk {k}: one-pass vs chunked prefill rel-L2 {e:.2e}"
    if with_oracle:
        ref = oracle.OracleShard(cfg, 0, cfg.layers, wl.max_seq, wl.chunk)
        ref.init_random(wl.target_seed)
        last = _oracle_prefill(ref, prompt, wl.chunk)
        for k, (p, toks) in enumerate(chunks):
            e = rel_l2(got[k], ref.forward(p, tokens=toks))
            assert e <= 1e-3, f"chunk {k}: one-pass prefill vs oracle rel-L2 {e:.2e}"
        ref.close()
        t1, t2 = oracle.top2(last)
        if t1 - t2 >= TIE_GAP:
            assert first1 == first8 == oracle.argmax(last)
    else:
        # the logits of the prompt's last row, from the chunked session's cache
        last = _chain_step_logits(chain, n - 1, [prompt[-1]]).logits[0]
        t1, t2 = oracle.top2(last)
        if t1 - t2 >= TIE_GAP:
            assert first1 == first8 == oracle.argmax(last)
    for s in stages:
        s.close()
