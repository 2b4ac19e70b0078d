"""Parity of the benchmark's own workload on the device: the 36-layer Qwen3-4B target with
seed 3 (the qwen3-4b-8stage workload at one GPU), against the oracle.

Both sides hold the same seeded warm cache (fill_kv), then run 8-row verify chunks and 1-row
steps at about 2,048 cached positions and at the cache's end (4,088 + 8 = 4,096 positions,
the workload's max_seq). Every layer's output is compared through the shard's tapped layers
(rel-L2 <= 1e-3), the logits at rel-L2 <= 1e-3 and the greedy picks wherever the oracle's
top-2 gap is at least 1e-3 (the tolerances of the scope). A one-pass prefill of the
workload's 2,047 prompt rows must leave the K/V rows of the chunked verify path (the next
steps agree at rel-L2 <= 2e-4 and pick the same token), and a prefill of a 64-token prompt
the oracle's (the oracle cannot run 2,047 rows of a 4B model in a test's time).
"""
import numpy as np
import pytest

import oracle
from helpers import rel_l2
from potpori_b200.shard import Shard
from potpori_b200.workload import WORKLOADS

pytestmark = pytest.mark.gpu

TIE_GAP = 1e-3
WL = WORKLOADS["qwen3-4b-8stage"]


@pytest.fixture(scope="module")
def models(gpu):
    cfg = WL.target
    dev = Shard.random(cfg, (0, cfg.layers), WL.max_seq, WL.chunk, seed=WL.target_seed)
    dev.set_taps(list(range(cfg.layers - 1)))
    ref = oracle.OracleShard(cfg, 0, cfg.layers, WL.max_seq, WL.chunk)
    ref.init_random(WL.target_seed)
    yield cfg, dev, ref
    dev.close()
    ref.close()


def _check_step(cfg, dev, ref, pos, toks, what):
    want, taps = ref.forward(pos, tokens=toks, taps=True)
    res = dev.verify_tokens(pos, toks, logits=True)
    got_taps = dev.take_taps(len(toks))
    worst = 0.0
    for l in range(cfg.layers - 1):
        e = rel_l2(got_taps[l], taps[l])
        worst = max(worst, e)
        assert e <= 1e-3, f"{what}: layer {l} rel-L2 {e:.2e}"
    e = rel_l2(res.logits, want)
    assert e <= 1e-3, f"{what}: logits rel-L2 {e:.2e}"
    for r in range(len(toks)):
        t1, t2 = oracle.top2(want[r])
        if t1 - t2 >= TIE_GAP:
            assert res.argmax[r] == oracle.argmax(want[r]), f"{what}: row {r}"
    n = 0
    while n < len(toks) - 1 and toks[1 + n] == res.argmax[n]:
        n += 1
    assert res.n_accepted == n and res.correction == res.argmax[n]
    return max(worst, e)


@pytest.mark.parametrize("cached", [2047, 4088])
def test_qwen3_4b_seed3_whole_model_parity(models, cached):
    cfg, dev, ref = models
    dev.fill_kv(11, cached)
    ref.fill_kv(11, cached)
    rng = np.random.default_rng(cached)
    toks = rng.integers(0, cfg.vocab_size, 8).tolist()
    worst = _check_step(cfg, dev, ref, cached, toks, f"8 rows at {cached}")
    # The next chunk, whose first token is the device's pick after the first chunk (as the
    # driver feeds it), then a 1-row step, over the rows the earlier steps wrote.
    if cached + 16 <= WL.max_seq:
        r0 = dev.verify_tokens(cached, toks).argmax
        toks2 = [r0[-1], *rng.integers(0, cfg.vocab_size, 7).tolist()]
        worst = max(worst, _check_step(cfg, dev, ref, cached + 8, toks2, f"8 rows at {cached + 8}"))
        worst = max(worst, _check_step(cfg, dev, ref, cached + 16, [toks2[3]], f"1 row at {cached + 16}"))
    else:
        # The cache's last positions: a rolled-back 1-row step inside the chunk just written.
        worst = max(worst, _check_step(cfg, dev, ref, cached + 3, [toks[5]], f"1 row at {cached + 3}"))
    print(f"cached {cached}: worst rel-L2 {worst:.2e}")


def test_qwen3_4b_seed3_after_one_pass_prefill(models):
    cfg, dev, ref = models
    # 64-token prompt: one-pass prefill on the device, chunked verify steps in the oracle.
    prompt = np.random.default_rng(64).integers(0, cfg.vocab_size, 64).tolist()
    dev.set_taps([])
    dev.reset()
    ref.reset()
    dev.prefill(0, prompt[:-1])
    pos = 0
    while pos < 63:
        take = 8 if 63 - pos >= 8 else 1
        ref.forward(pos, tokens=prompt[pos:pos + take])
        pos += take
    cur = prompt[-1]
    for step in range(2):
        got = dev.forward_tokens(63 + step, [cur])[0]
        want = ref.forward(63 + step, tokens=[cur])[0]
        e = rel_l2(got, want)
        assert e <= 1e-3, f"step {step}: rel-L2 {e:.2e}"
        t1, t2 = oracle.top2(want)
        if t1 - t2 >= TIE_GAP:
            assert int(np.argmax(got)) == oracle.argmax(want)
        cur = oracle.argmax(want)
    dev.set_taps(list(range(cfg.layers - 1)))


def test_qwen3_4b_seed3_workload_prefill_matches_the_chunked_path(gpu):
    """The workload's own prompt (2,048 ids, seed 103): the one-pass prefill of its first
    2,047 rows against 8-row verify steps of the same rows on a second device shard."""
    cfg = WL.target
    prompt = WL.prompt()
    pre = Shard.random(cfg, (0, cfg.layers), WL.max_seq, WL.chunk, seed=WL.target_seed)
    chk = Shard.random(cfg, (0, cfg.layers), WL.max_seq, WL.chunk, seed=WL.target_seed)
    end = len(prompt) - 1
    pre.prefill(0, prompt[:end])
    pos = 0
    while pos < end:
        take = 8 if end - pos >= 8 else 1
        chk.forward_tokens(pos, prompt[pos:pos + take])
        pos += take
    cur = prompt[end]
    for step in range(3):
        got = pre.forward_tokens(end + step, [cur])[0]
        other = chk.forward_tokens(end + step, [cur])[0]
        e = rel_l2(got, other)
        assert e <= 2e-4, f"step {step}: {e:.2e} against the chunked path"
        top = np.sort(other)[-2:]
        if top[1] - top[0] >= TIE_GAP:
            assert int(np.argmax(got)) == int(np.argmax(other))
        cur = int(np.argmax(other))
    pre.close()
    chk.close()
