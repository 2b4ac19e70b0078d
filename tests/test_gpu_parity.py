"""Parity of the sm_100a verify pass with the oracle and the reference's golden vectors.

Every test here runs the CUDA path through the C ABI (potpori_b200/libpotpori_b200.so) and
checks it against the oracle (a CPU restatement of the reference math) or the reference's own
fixtures. Tolerances: the reference's own bounds where it has them (2e-4 for the tiny model,
src/qwen/tiny.rs:225; 2e-3 against transformers, src/qwen/cpu_check.rs:268-270); per-layer
hidden states rel-L2 <= 1e-3 and token identity except where the oracle's top-2 logit gap is
below 1e-3 for the Qwen3 geometries.
"""
import numpy as np
import pytest

import oracle
from helpers import load_fixture, rel_l2, tiny_weights
from potpori_b200._lib import PP_E_INVALID, PP_E_NONFINITE, PP_E_UNSUPPORTED, PPError
from potpori_b200.config import QWEN3_0_6B, QWEN3_4B, TINY
from potpori_b200.shard import Shard

pytestmark = pytest.mark.gpu

TIE_GAP = 1e-3


def test_tiny_shards_and_rollback(gpu):
    """src/qwen/tiny.rs:136-249 on the device: the whole model against the oracle, a 2-shard
    cut against the whole model, and a rolled-back cache against a fresh one (2e-4)."""
    cfg, W = TINY, tiny_weights()
    full, head, tail = (Shard(cfg, r, 8, 2) for r in [(0, 2), (0, 1), (1, 2)])
    for s in (full, head, tail):
        s.load(W)
        assert not s.missing()
    ref = oracle.OracleShard(cfg, 0, 2, 8, 2)
    ref.load(W)
    rollback = None
    for pos, toks in [(0, [1]), (1, [2, 3]), (1, [4, 5]), (3, [6])]:
        got = full.forward_tokens(pos, toks)
        want = ref.forward(pos, tokens=toks)
        assert got.shape == (len(toks), cfg.vocab_size)
        assert np.isfinite(got).all()
        assert np.abs(got - want).max() < 2e-4
        hidden = head.forward_tokens(pos, toks)
        cut = tail.forward_hidden(pos, len(toks), hidden)
        assert np.abs(cut - got).max() < 2e-4
        if pos == 3:
            rollback = got
    full.reset()
    full.forward_tokens(0, [1])
    full.forward_tokens(1, [4, 5])
    clean = full.forward_tokens(3, [6])
    assert np.abs(rollback - clean).max() < 2e-4


def test_fixture_cut_matches_transformers(gpu):
    """src/qwen/cpu_check.rs:244-275 on the device: the 6-layer fixture cut at the tapped
    layers into four shards reproduces transformers' logits and layer outputs (2e-3) and the
    greedy continuation."""
    cfg, meta, W, want_logits, want_feat = load_fixture()
    ranges = [(0, 1), (1, 3), (3, 5), (5, 6)]
    shards = [Shard(cfg, r, 64, 8) for r in ranges]
    for s in shards:
        s.load(W)
        assert not s.missing()
    seq = meta["sequence"]
    logits, feats, pos = [], [], 0
    while pos < len(seq):
        take = 8 if len(seq) - pos >= 8 else 1
        h = shards[0].forward_tokens(pos, seq[pos:pos + take])
        taps = [h]
        for s in shards[1:]:
            h = s.forward_hidden(pos, take, h)
            if not s.last:
                taps.append(h)
        logits.append(h)
        feats.append(np.concatenate(taps, axis=1))
        pos += take
    logits = np.concatenate(logits)
    feats = np.concatenate(feats)
    assert np.abs(logits - want_logits).max() < 2e-3
    assert np.abs(feats - want_feat).max() < 2e-3
    assert [int(np.argmax(r)) for r in logits] == meta["next_tokens"]


def _oracle_whole(cfg, seed, capacity, chunk):
    o = oracle.OracleShard(cfg, 0, cfg.layers, capacity, chunk)
    o.init_random(seed)
    return o


def test_qwen3_0_6b_per_layer_parity(gpu):
    """Qwen3-0.6B (seed 0): one device shard per layer, each layer's output against the
    oracle's (rel-L2 <= 1e-3), then the greedy picks of the last shard."""
    cfg, seed, cap = QWEN3_0_6B, 0, 128
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, cfg.vocab_size, 41).tolist()
    shards = [Shard.random(cfg, (l, l + 1), cap, 8, seed=seed) for l in range(cfg.layers)]
    ref = _oracle_whole(cfg, seed, cap, 8)
    pos = 0
    worst = 0.0
    while pos < len(prompt):
        take = 8 if len(prompt) - pos >= 8 else 1
        toks = prompt[pos:pos + take]
        want_logits, taps = ref.forward(pos, tokens=toks, taps=True)
        h = shards[0].forward_tokens(pos, toks)
        for l, s in enumerate(shards[1:], start=1):
            worst = max(worst, rel_l2(h, taps[l - 1]))
            assert rel_l2(h, taps[l - 1]) <= 1e-3, (pos, l)
            if s.last:
                res = s.verify_hidden(pos, h, drafts=toks[1:], logits=True)
            else:
                h = s.forward_hidden(pos, take, h)
        assert rel_l2(res.logits, want_logits) <= 1e-3
        for r in range(take):
            t1, t2 = oracle.top2(want_logits[r])
            want = oracle.argmax(want_logits[r])
            if t1 - t2 >= TIE_GAP:
                assert res.argmax[r] == want, (pos, r)
            assert res.argmax[r] == int(np.argmax(res.logits[r]))
            assert abs(res.top1[r] - float(res.logits[r].max())) == 0.0
        pos += take
    print(f"worst per-layer rel-L2 {worst:.3e}")


def test_qwen3_0_6b_whole_model_verify(gpu):
    """The production layout: all 28 layers in one shard; argmax, top-2 and the accept
    compare against the oracle."""
    cfg, seed, cap = QWEN3_0_6B, 0, 128
    rng = np.random.default_rng(1)
    toks_all = rng.integers(0, cfg.vocab_size, 24).tolist()
    dev = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=seed)
    ref = _oracle_whole(cfg, seed, cap, 8)
    for pos in range(0, 24, 8):
        toks = toks_all[pos:pos + 8]
        want = ref.forward(pos, tokens=toks)
        res = dev.verify_tokens(pos, toks, logits=True)
        assert rel_l2(res.logits, want) <= 1e-3
        picks = []
        for r in range(8):
            t1, t2 = oracle.top2(want[r])
            if t1 - t2 >= TIE_GAP:
                assert res.argmax[r] == oracle.argmax(want[r])
            picks.append(res.argmax[r])
        # accept compare: drafts = toks[1:] against the device's own picks
        n = 0
        while n < 7 and toks[1 + n] == picks[n]:
            n += 1
        assert res.n_accepted == n and res.correction == picks[n]


@pytest.mark.parametrize("m", [1, 4, 8, 16])
@pytest.mark.parametrize("kv_len", [128, 2048])
def test_qwen3_4b_layer_with_rollback(gpu, m, kv_len):
    """One Qwen3-4B decoder layer (seed 4) over a random warm cache: each step appends m
    rows and rolls back a random rejected suffix; output against the oracle."""
    cfg, seed = QWEN3_4B, 4
    lay = (5, 6)
    dev = Shard.random(cfg, lay, 4096, 0, seed=seed)
    ref = oracle.OracleShard(cfg, lay[0], lay[1], 4096, 0)
    ref.init_random(seed)
    dev.fill_kv(7, kv_len)
    ref.fill_kv(7, kv_len)
    rng = np.random.default_rng(kv_len + m)
    pos = kv_len
    for _ in range(3):
        hidden = rng.standard_normal((m, cfg.hidden)).astype(np.float32)
        got = dev.forward_hidden(pos, m, hidden)
        want = ref.forward(pos, hidden=hidden)
        assert rel_l2(got, want) <= 1e-3
        pos += m - int(rng.integers(0, m))  # keep a prefix, overwrite the rest next step


def test_rejects_invalid_steps(gpu):
    """src/qwen/model.rs:373-395: chunk size, capacity, token range, finite hidden."""
    cfg = TINY
    W = tiny_weights()
    full = Shard(cfg, (0, 2), 8, 2)
    full.load(W)
    tail = Shard(cfg, (1, 2), 8, 2)
    tail.load(W)
    for pos, toks in [(0, [1, 2, 3]), (7, [1, 2]), (0, [16]), (0, [-1])]:
        with pytest.raises(PPError) as e:
            full.forward_tokens(pos, toks)
        assert e.value.status == PP_E_INVALID
    bad = np.zeros((1, cfg.hidden), np.float32)
    bad[0, 3] = np.nan
    with pytest.raises(PPError) as e:
        tail.forward_hidden(0, 1, bad)
    assert e.value.status == PP_E_INVALID
    # the shard still works after the rejections
    assert np.isfinite(full.forward_tokens(0, [1])).all()


def test_nonfinite_logits_are_flagged(gpu):
    """A NaN weight reaches the logits: the tail reports the row as non-finite
    (src/engine.rs:14-17, src/node.rs:266-272) instead of a token."""
    cfg = TINY
    W = tiny_weights()
    W["model.norm.weight"] = np.full(cfg.hidden, np.nan, np.float32)
    full = Shard(cfg, (0, 2), 8, 2)
    full.load(W)
    res = full.verify_tokens(0, [1, 2])
    assert res.nonfinite_rows == 0b11
    assert res.argmax == [-1, -1]


@pytest.mark.parametrize("ctas", [8, 144])
def test_qwen3_4b_layer_under_an_sm_budget(gpu, ctas):
    """A shard whose kernels may use only `ctas` SMs (pp_shard_set_sm_limit: the multi-GPU
    ranks leave SMs to NCCL's transfer kernels) still matches the oracle; only the split-K and
    key-split partition, i.e. the summation order, changes."""
    cfg, seed = QWEN3_4B, 4
    lay = (5, 6)
    dev = Shard.random(cfg, lay, 4096, 0, seed=seed)
    dev.set_sm_limit(ctas)
    assert dev.sm_limit() == ctas
    ref = oracle.OracleShard(cfg, lay[0], lay[1], 4096, 0)
    ref.init_random(seed)
    dev.fill_kv(7, 2048)
    ref.fill_kv(7, 2048)
    rng = np.random.default_rng(ctas)
    pos = 2048
    for m in (8, 1):
        hidden = rng.standard_normal((m, cfg.hidden)).astype(np.float32)
        got = dev.forward_hidden(pos, m, hidden)
        want = ref.forward(pos, hidden=hidden)
        assert rel_l2(got, want) <= 1e-3
        pos += m
    with pytest.raises(PPError) as e:
        dev.set_sm_limit(cfg.n_kv_heads - 1)
    assert e.value.status == PP_E_INVALID


def test_greedy_decode_on_device_matches_the_host_loop(gpu):
    """pp_shard_decode_greedy (the draft's gamma loop, src/qwen/draft.rs:14-93, with each pick
    fed to the next step on the device) gives the same picks as one host round trip per
    token, and the oracle's greedy continuation where its top-2 gaps are clear."""
    cfg, seed, cap = QWEN3_0_6B, 0, 128
    a = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=seed)
    b = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=seed)
    ref = _oracle_whole(cfg, seed, cap, 8)
    prompt = np.random.default_rng(3).integers(0, cfg.vocab_size, 16).tolist()
    for s in (a, b):
        s.verify_tokens(0, prompt[:8])
        s.verify_tokens(8, prompt[8:])
    ref.forward(0, tokens=prompt[:8])
    ref.forward(8, tokens=prompt[8:])
    got = a.decode_greedy(16, prompt[-1], 6)
    host, cur = [], prompt[-1]
    for i in range(6):
        cur = b.verify_tokens(16 + i, [cur]).argmax[0]
        host.append(cur)
    assert got == host
    cur = prompt[-1]
    for i in range(6):
        want = ref.forward(16 + i, tokens=[cur])[0]
        t1, t2 = oracle.top2(want)
        if t1 - t2 < TIE_GAP:
            break
        assert got[i] == oracle.argmax(want)
        cur = got[i]
    part = Shard.random(cfg, (0, 2), cap, 8, seed=seed)
    with pytest.raises(PPError) as e:
        part.decode_greedy(0, 1, 2)
    assert e.value.status == PP_E_INVALID


def test_speculative_stream_equals_oracle_greedy(gpu):
    """Config 0 (Qwen3-0.6B seed 0, 41-id prompt, gamma 7, the draft a second copy of the same
    weights, so drafts are accepted): the committed stream of the one-chunk driver
    (src/specdecode.rs) and of the depth-4 pipelined driver (src/specpipe.rs) over the device
    shards equals the oracle's plain greedy continuation (speculative greedy decoding is
    lossless), up to the first position where the oracle's top-2 gap is below 1e-3."""
    from potpori_b200.chain import LocalChain
    from potpori_b200.specdecode import SpecConfig, run_spec_decode
    from potpori_b200.specpipe import PipelinedDriver
    from potpori_b200.target import IncrementalDraft, QwenTarget

    cfg, seed, cap, new = QWEN3_0_6B, 0, 128, 24
    prompt = np.random.default_rng(41).integers(0, cfg.vocab_size, 41).tolist()
    ref = _oracle_whole(cfg, seed, cap, 8)
    pos, last = 0, None
    while pos < len(prompt):
        take = 8 if len(prompt) - pos >= 8 else 1
        last = ref.forward(pos, tokens=prompt[pos:pos + take])[-1]
        pos += take
    want, gaps = [], []
    for i in range(new):
        t1, t2 = oracle.top2(last)
        gaps.append(t1 - t2)
        want.append(oracle.argmax(last))
        last = ref.forward(pos, tokens=[want[-1]])[0]
        pos += 1
    clear = next((i for i, g in enumerate(gaps) if g < TIE_GAP), new)

    def model():
        return QwenTarget(Shard.random(cfg, (0, cfg.layers), cap, 8, seed=seed))

    scfg = SpecConfig(7, new)
    out, stats = run_spec_decode(IncrementalDraft(model(), 8), model(), prompt, scfg)
    assert out[:clear] == want[:clear]
    assert stats.toks_per_traversal() > 4  # the same weights: drafts are accepted

    tgt = model()
    drv = PipelinedDriver(IncrementalDraft(model(), 8), LocalChain([tgt.shard]), prompt, scfg, 4)
    drv.start()
    while drv.step():
        pass
    assert drv.out[:clear] == want[:clear]


def _step_logits_agree(got, want, worst, name):
    """Logits of one 1-row step against the oracle: rel-L2 <= 1e-3 and the same greedy pick
    unless the oracle's top-2 gap is below 1e-3."""
    e = rel_l2(got, want)
    assert e <= 1e-3, f"{name}: rel-L2 {e:.2e}"
    t1, t2 = oracle.top2(want)
    if t1 - t2 >= TIE_GAP:
        assert int(np.argmax(got)) == oracle.argmax(want), name
    return max(worst, e)


def test_decode_kernel_matches_the_oracle_and_the_layer_kernels(gpu):
    """The persistent 1-row decode kernel (pp_shard_set_decode_kernel) on Qwen3-0.6B (seed 0):
    single-token steps at the first position (one key), after a chunked prefill, over a
    seeded 2048-position cache (114 keys per attention split), after a rolled-back position
    and under an SM budget give the oracle's logits (rel-L2 <= 1e-3, same pick unless the
    top-2 gap is below 1e-3) and the per-layer kernels' (rel-L2 <= 2e-4); the device decode
    loop gives the same picks as the per-layer kernels."""
    cfg, seed, cap = QWEN3_0_6B, 0, 2304
    dec = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=seed)
    lay = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=seed)
    dec.set_decode_kernel(True)
    assert dec.decode_kernel() and not lay.decode_kernel()
    ref = _oracle_whole(cfg, seed, cap, 8)
    rng = np.random.default_rng(7)
    toks = rng.integers(0, cfg.vocab_size, 24).tolist()
    worst, worst_lay = 0.0, 0.0

    def step(pos, tok, name):
        nonlocal worst, worst_lay
        got = dec.forward_tokens(pos, [tok])[0]
        other = lay.forward_tokens(pos, [tok])[0]
        want = ref.forward(pos, tokens=[tok])[0]
        worst = _step_logits_agree(got, want, worst, name)
        worst_lay = max(worst_lay, rel_l2(got, other))
        assert worst_lay <= 2e-4, f"{name}: {worst_lay:.2e} against the per-layer kernels"

    step(0, toks[0], "pos 0")
    for s in (dec, lay):
        s.forward_tokens(1, toks[1:9])
    ref.forward(1, tokens=toks[1:9])
    for i in range(3):
        step(9 + i, toks[9 + i], f"pos {9 + i}")
    step(10, toks[20], "rolled back to pos 10")
    step(11, toks[21], "pos 11 after the rollback")
    for s in (dec, lay, ref):
        s.fill_kv(5, 2048)
    for i in range(3):
        step(2048 + i, toks[12 + i], f"pos {2048 + i}")
    dec.set_sm_limit(64)
    step(2051, toks[15], "64-SM budget")
    dec.set_sm_limit(0)
    step(2052, toks[16], "all SMs again")
    got = dec.decode_greedy(2053, toks[17], 6)
    want = lay.decode_greedy(2053, toks[17], 6)
    assert got == want
    part = Shard.random(cfg, (0, 2), 64, 8, seed=seed)
    with pytest.raises(PPError) as e:
        part.set_decode_kernel(True)  # the kernel runs shards that hold every layer
    assert e.value.status == PP_E_UNSUPPORTED
    assert not part.decode_kernel()
    print(f"decode kernel: worst rel-L2 {worst:.2e} vs oracle, {worst_lay:.2e} vs layer kernels")


@pytest.mark.parametrize("H,I,nh,G", [(2048, 6144, 16, 2), (2560, 9728, 32, 4),
                                      (1024, 4608, 16, 2), (1024, 3072, 8, 1)])
def test_decode_kernel_row_layouts(gpu, H, I, nh, G):
    """The decode kernel's GEMV slots take R = 32, 16, 8, 4, 2 or 1 rows of the padded K at a
    time, with the lanes of a row either R apart (contiguous column slices) or adjacent (every
    lpr-th 16-byte unit); two-layer models of the Qwen3-1.7B and Qwen3-4B geometries, an
    intermediate size whose padded K (5120) splits 80 units over 16 lanes, and one query head
    per KV head: 1-row steps at 1 and at 300 cached positions give the oracle's logits
    (rel-L2 <= 1e-3) and the per-layer kernels' (rel-L2 <= 2e-4)."""
    from potpori_b200.config import QwenConfig
    cfg = QwenConfig(layers=2, hidden=H, intermediate=I, head_dim=128, n_heads=nh,
                     n_kv_heads=nh // G, vocab_size=1000, rms_norm_eps=1e-6, rope_theta=1e6)
    dec = Shard.random(cfg, (0, 2), 512, 8, seed=9)
    lay = Shard.random(cfg, (0, 2), 512, 8, seed=9)
    dec.set_decode_kernel(True)
    ref = _oracle_whole(cfg, 9, 512, 8)
    rng = np.random.default_rng(H + I)
    worst = 0.0
    for pos in (0, 1):
        t = int(rng.integers(0, cfg.vocab_size))
        got, other = dec.forward_tokens(pos, [t])[0], lay.forward_tokens(pos, [t])[0]
        worst = _step_logits_agree(got, ref.forward(pos, tokens=[t])[0], worst, f"pos {pos}")
        assert rel_l2(got, other) <= 2e-4
    for sh in (dec, lay, ref):
        sh.fill_kv(3, 300)
    for pos in (300, 301):
        t = int(rng.integers(0, cfg.vocab_size))
        got, other = dec.forward_tokens(pos, [t])[0], lay.forward_tokens(pos, [t])[0]
        worst = _step_logits_agree(got, ref.forward(pos, tokens=[t])[0], worst, f"pos {pos}")
        assert rel_l2(got, other) <= 2e-4
    for sh in (dec, lay, ref):
        sh.close()


def test_prefill_matches_the_chunked_path_and_the_oracle(gpu):
    """pp_shard_prefill (all layers over a prompt chunk at once: tensor-core projections,
    flash-style causal attention) leaves the K/V rows of the reference's chunked prefill
    (src/qwen/target.rs:62-84): after it, the next steps give the logits of the chunked verify
    path (rel-L2 <= 2e-4) and of the oracle (rel-L2 <= 1e-3, same pick unless the top-2 gap is
    below 1e-3). Config 0 (Qwen3-0.6B seed 0, 41-token prompt from position 0) and a 2-layer
    model of Qwen3-4B geometry (G = 4) over 173 tokens from position 5 (a ragged last block)."""
    from potpori_b200.config import QwenConfig

    cases = [(QWEN3_0_6B, 0, 0, 41),
             (QwenConfig(2, 2560, 9728, 128, 32, 8, 151936, 1e-6, 1e6), 4, 5, 173)]
    for cfg, seed, pos0, n in cases:
        cap = 256
        rng = np.random.default_rng(seed + 100)
        prompt = rng.integers(0, cfg.vocab_size, pos0 + n).tolist()
        pre = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=seed)
        chk = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=seed)
        ref = _oracle_whole(cfg, seed, cap, 8)
        assert pre.can_prefill()
        end = pos0 + n - 1  # every prompt token but the last
        # The first pos0 positions go the chunked way on every side, then the prefill.
        pos = 0
        while pos < end:
            take = 8 if end - pos >= 8 else 1
            if pos < pos0:
                take = 8 if pos0 - pos >= 8 else 1
                pre.forward_tokens(pos, prompt[pos:pos + take])
            chk.forward_tokens(pos, prompt[pos:pos + take])
            ref.forward(pos, tokens=prompt[pos:pos + take])
            pos += take
        pre.prefill(pos0, prompt[pos0:end])
        cur = prompt[end]
        for step in range(2):
            got = pre.forward_tokens(end + step, [cur])[0]
            other = chk.forward_tokens(end + step, [cur])[0]
            want = ref.forward(end + step, tokens=[cur])[0]
            _step_logits_agree(got, want, 0.0, f"{cfg.layers}-layer model, step {step}")
            e = rel_l2(got, other)
            assert e <= 2e-4, f"{cfg.layers}-layer model, step {step}: {e:.2e} against the chunked path"
            cur = int(np.argmax(want))
    later = Shard.random(QWEN3_0_6B, (2, 4), 64, 8, seed=0)
    with pytest.raises(PPError) as e:
        later.prefill(0, [1, 2, 3])  # token input on a later stage
    assert e.value.status == PP_E_INVALID
    tiny = Shard(TINY, (0, 2), 8, 2)
    tiny.load(tiny_weights())
    assert not tiny.can_prefill()
    with pytest.raises(PPError) as e:
        tiny.prefill(0, [1, 2, 3])  # head size 4
    assert e.value.status == PP_E_UNSUPPORTED


@pytest.mark.gpu
def test_prefill_past_2048_keys_matches_the_chunked_path(gpu):
    """Two prefill calls over a 2199-token prompt (2048 rows from position 0, then 151 rows
    from position 2048, whose rows see more than 2048 keys) leave the K/V rows of the chunked
    verify path: the next two steps agree within rel-L2 2e-4 and pick the same token unless
    its top-2 gap is below 1e-3. A 2-layer model of Qwen3-0.6B geometry."""
    from potpori_b200.config import QwenConfig

    cfg = QwenConfig(2, 1024, 3072, 128, 16, 8, 151936, 1e-6, 1e6)
    cap, n = 2304, 2200
    prompt = np.random.default_rng(7).integers(0, cfg.vocab_size, n).tolist()
    pre = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=1)
    chk = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=1)
    end = n - 1
    pre.prefill(0, prompt[:2048])
    pre.prefill(2048, prompt[2048:end])
    pos = 0
    while pos < end:
        take = 8 if end - pos >= 8 else 1
        chk.forward_tokens(pos, prompt[pos:pos + take])
        pos += take
    cur = prompt[end]
    for step in range(2):
        got = pre.forward_tokens(end + step, [cur])[0]
        other = chk.forward_tokens(end + step, [cur])[0]
        e = rel_l2(got, other)
        assert e <= 2e-4, f"step {step}: {e:.2e} against the chunked path"
        top2 = np.sort(other)[-2:]
        if top2[1] - top2[0] > 1e-3 * abs(top2[1]):
            assert int(np.argmax(got)) == int(np.argmax(other))
        cur = int(np.argmax(other))
    pre.close()
    chk.close()


def test_bounded_wait_times_out_and_the_shard_recovers(gpu):
    """A device wait that nothing can end (the decode kernel's first grid barrier made to
    wait for one CTA more than the grid has, pp_shard_set_wait_test) runs out after its time
    limit: the step returns PP_E_TIMEOUT instead of hanging, the GPU and the shard stay
    usable, and the next normal steps match the oracle (the reference bounds its waits too,
    src/node.rs:47-50)."""
    from potpori_b200._lib import PP_E_TIMEOUT

    cfg, seed, cap = QWEN3_0_6B, 0, 64
    dev = Shard.random(cfg, (0, cfg.layers), cap, 8, seed=seed)
    dev.set_decode_kernel(True)
    ref = _oracle_whole(cfg, seed, cap, 8)
    dev.set_wait_test(limit_us=5000, unreachable=True)
    for _ in range(2):
        with pytest.raises(PPError) as e:
            dev.forward_tokens(0, [7])
        assert e.value.status == PP_E_TIMEOUT
    dev.set_wait_test(0, False)
    for pos, tok in enumerate([7, 8, 9]):
        got = dev.forward_tokens(pos, [tok])[0]
        want = ref.forward(pos, tokens=[tok])[0]
        _step_logits_agree(got, want, 0.0, f"pos {pos} after the timeouts")
    dev.close()
