"""The oracle against the reference's golden vectors and its own invariants (no GPU)."""
import numpy as np
import pytest

import oracle
from helpers import load_fixture, rel_l2, tiny_weights
from potpori_b200.config import TINY, QwenConfig
from potpori_b200.engine import argmax as host_argmax


def test_argmax_rejects_non_finite_rows():
    """src/engine.rs:68-75, for both the oracle and the host mirror."""
    for f in (oracle.argmax, host_argmax):
        assert f(np.array([0.1, 2.0, -3.0], np.float32)) == 1
        assert f(np.array([-1.0, -2.0], np.float32)) == 0
        assert f(np.array([], np.float32)) is None
        assert f(np.array([0.0, np.nan], np.float32)) is None
        assert f(np.array([np.inf, 0.0], np.float32)) is None
        assert f(np.array([1.0, 3.0, 3.0], np.float32)) == 1  # first index of the maximum


def _feed(shards, seq, chunk):
    logits, feats, pos = [], [], 0
    while pos < len(seq):
        take = chunk if len(seq) - pos >= chunk else 1
        h = shards[0].forward(pos, tokens=seq[pos:pos + take])
        taps = [h]
        for s in shards[1:]:
            h = s.forward(pos, hidden=h)
            if not s.last:
                taps.append(h)
        logits.append(h)
        feats.append(np.concatenate(taps, axis=1))
        pos += take
    return np.concatenate(logits), np.concatenate(feats)


@pytest.mark.parametrize("rope_mode", [oracle.ROPE_F64, oracle.ROPE_F32])
def test_oracle_matches_reference_fixture(rope_mode):
    """The reference's golden vectors (transformers on the 6-layer fixture,
    src/qwen/cpu_check.rs:244-275): logits and tapped layer outputs within the reference's
    2e-3 (the oracle lands near 4e-6), greedy picks equal to next_tokens."""
    cfg, meta, W, want_logits, want_feat = load_fixture()
    shards = [oracle.OracleShard(cfg, a, b, 64, 8, rope_mode=rope_mode)
              for a, b in [(0, 1), (1, 3), (3, 5), (5, 6)]]
    for s in shards:
        s.load(W)
        assert not s.missing()
    logits, feats = _feed(shards, meta["sequence"], 8)
    assert np.abs(logits - want_logits).max() < 1e-4
    assert np.abs(feats - want_feat).max() < 1e-4
    assert [oracle.argmax(r) for r in logits] == meta["next_tokens"]
    # The prompt's greedy continuation (the fixture's `sequence`).
    p = len(meta["prompt"])
    assert [oracle.argmax(r) for r in logits[p - 1:-1]] == meta["sequence"][p:]


def test_oracle_tiny_cut_and_rollback():
    """src/qwen/tiny.rs:211-248 on the oracle: a fresh recompute of the whole prefix, a
    2-shard cut and a rolled-back cache all agree (2e-4)."""
    cfg, W = TINY, tiny_weights()
    full = oracle.OracleShard(cfg, 0, 2, 8, 2)
    head = oracle.OracleShard(cfg, 0, 1, 8, 2)
    tail = oracle.OracleShard(cfg, 1, 2, 8, 2)
    for s in (full, head, tail):
        s.load(W)
    prefix, rollback = [], None
    for pos, toks in [(0, [1]), (1, [2, 3]), (1, [4, 5]), (3, [6])]:
        got = full.forward(pos, tokens=toks)
        prefix = prefix[:pos] + toks
        fresh = oracle.OracleShard(cfg, 0, 2, 8, 0)
        fresh.load(W)
        want = fresh.forward(0, tokens=prefix)[pos:]
        assert np.abs(got - want).max() < 2e-4
        cut = tail.forward(pos, hidden=head.forward(pos, tokens=toks))
        assert np.abs(cut - got).max() < 2e-4
        if pos == 3:
            rollback = got
    full.reset()
    full.forward(0, tokens=[1])
    full.forward(1, tokens=[4, 5])
    assert np.abs(full.forward(3, tokens=[6]) - rollback).max() < 2e-4


def test_oracle_rejects_invalid_steps():
    """src/qwen/model.rs:373-395."""
    cfg, W = TINY, tiny_weights()
    full = oracle.OracleShard(cfg, 0, 2, 8, 2)
    full.load(W)
    for pos, toks in [(0, [1, 2, 3]), (7, [1, 2]), (0, [16]), (0, [-1])]:
        with pytest.raises(oracle.OracleError):
            full.forward(pos, tokens=toks)
    tail = oracle.OracleShard(cfg, 1, 2, 8, 2)
    tail.load(W)
    bad = np.zeros((1, cfg.hidden), np.float32)
    bad[0, 0] = np.inf
    with pytest.raises(oracle.OracleError):
        tail.forward(0, hidden=bad)


def test_oracle_matches_transformers_random_qwen3():
    """A random 2-layer Qwen3 with the real head width, run by transformers'
    Qwen3ForCausalLM in F32 and by the oracle on the same BF16 weights."""
    torch = pytest.importorskip("torch")
    tr = pytest.importorskip("transformers")
    cfg = QwenConfig(layers=2, hidden=256, intermediate=512, head_dim=128, n_heads=4,
                     n_kv_heads=2, vocab_size=512, rms_norm_eps=1e-6, rope_theta=1e6)
    hf = tr.Qwen3Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden,
                        intermediate_size=cfg.intermediate, num_hidden_layers=cfg.layers,
                        num_attention_heads=cfg.n_heads, num_key_value_heads=cfg.n_kv_heads,
                        head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_norm_eps,
                        rope_theta=cfg.rope_theta, tie_word_embeddings=True,
                        max_position_embeddings=256)
    torch.manual_seed(0)
    model = tr.Qwen3ForCausalLM(hf).eval().float()
    ora = oracle.OracleShard(cfg, 0, cfg.layers, 64, 0)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.copy_(1 + 0.3 * torch.randn(p.shape))
            else:
                p.copy_((0.05 * torch.randn(p.shape)).bfloat16().float())
        for name, p in model.named_parameters():
            if name == "lm_head.weight":
                continue
            v = p.detach().numpy().astype(np.float32).reshape(-1)
            ora.set_tensor(name, v)
        assert not ora.missing()
        toks = list(range(3, 40, 3))
        want = model(torch.tensor([toks])).logits[0].numpy()
    got = ora.forward(0, tokens=toks)
    assert rel_l2(got, want) < 1e-5


def test_generator_is_deterministic_and_normal():
    a = oracle.gen_bf16(3, "model.layers.0.mlp.up_proj.weight", 200000)
    b = oracle.gen_bf16(3, "model.layers.0.mlp.up_proj.weight", 1000, start=500)
    assert np.array_equal(a[500:1500], b)
    c = oracle.gen_bf16(4, "model.layers.0.mlp.up_proj.weight", 1000)
    assert not np.array_equal(a[:1000], c)
    v = (a.astype(np.uint32) << 16).view(np.float32)
    assert abs(float(v.mean())) < 2e-4 and abs(float(v.std()) - 0.02) < 2e-4
