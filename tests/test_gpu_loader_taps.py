"""Prepared-file loading and tapped-layer outputs on the device, through the C ABI.

The reference loads each shard's parameters from one prepared safetensors file
(src/qwen/hf.rs:160-272: matrices BF16, norms F32) and reports the outputs of tapped layers
with every result (TappedShards, src/node.rs:108-223; LayerTap, src/transport.rs:148-179).
Here a prepared file written by the test helper must give the same device weights as
set_tensor (identical logits for the whole model, the same to F32 rounding for a cut into two
shards), and a shard's tapped outputs must
be the oracle's per-layer outputs, with the wire form their BF16 rounding.
"""
import numpy as np
import pytest

import oracle
from helpers import bf16_bits_to_f32, f32_to_bf16_bits, random_weights, rel_l2, write_prepared
from potpori_b200._lib import PP_E_INVALID, PP_E_MISSING, PPError
from potpori_b200.config import QwenConfig
from potpori_b200.shard import Shard

pytestmark = pytest.mark.gpu

CFG = QwenConfig(layers=3, hidden=256, intermediate=512, head_dim=128, n_heads=4, n_kv_heads=2,
                 vocab_size=1000, rms_norm_eps=1e-6, rope_theta=1e6)


def _steps(shards, prompt):
    """Feed `prompt` through a chain of host-synchronous shards in 8-row and 1-row steps;
    the last step's logits."""
    pos, out = 0, None
    while pos < len(prompt):
        take = 8 if len(prompt) - pos >= 8 else 1
        h = shards[0].forward_tokens(pos, prompt[pos:pos + take])
        for s in shards[1:]:
            h = s.forward_hidden(pos, take, h)
        out = h
        pos += take
    return out


@pytest.mark.parametrize("matrix_dtype", ["bf16", "f32"])
def test_prepared_file_loads_like_set_tensor(gpu, tmp_path, matrix_dtype):
    W = random_weights(CFG, seed=21)
    path = str(tmp_path / "model_combined_bf16_v1.safetensors")
    write_prepared(path, CFG, W, matrix_dtype)
    prompt = np.random.default_rng(4).integers(0, CFG.vocab_size, 19).tolist()

    direct = Shard(CFG, (0, 3), 64, 8)
    direct.load(W)
    want = _steps([direct], prompt)
    whole = Shard.load_chunked(CFG, (0, 3), True, True, path, 64)
    assert not whole.missing()
    got = _steps([whole], prompt)
    assert np.array_equal(got, want)
    # Each cut takes only its own parameters from the same file (Shard::load_chunked). A cut
    # forms the next norm's sum of squares in its input kernel, not in the residual epilogue,
    # so it agrees to F32 rounding rather than bit for bit.
    cut = [Shard.load_chunked(CFG, r, r[0] == 0, r[1] == 3, path, 64) for r in [(0, 1), (1, 3)]]
    assert all(not s.missing() for s in cut)
    assert rel_l2(_steps(cut, prompt), want) <= 1e-5
    ref = oracle.OracleShard(CFG, 0, 3, 64, 8)
    ref.load(W)
    pos, last = 0, None
    while pos < len(prompt):
        take = 8 if len(prompt) - pos >= 8 else 1
        last = ref.forward(pos, tokens=prompt[pos:pos + take])
        pos += take
    assert rel_l2(got, last) <= 1e-3
    for s in [direct, whole] + cut:
        s.close()


def test_prepared_file_errors(gpu, tmp_path):
    """A file without some of the shard's parameters leaves them missing (the step is refused
    with PP_E_MISSING); a stored shape other than the parameter's is refused on load
    (src/qwen/hf.rs:235)."""
    W = random_weights(CFG, seed=22)
    partial = {k: v for k, v in W.items() if "layers.2." not in k}
    path = str(tmp_path / "partial.safetensors")
    write_prepared(path, CFG, partial)
    s = Shard(CFG, (0, 3), 64, 8)
    s.load_safetensors(path)
    assert any("model.layers.2." in n for n in s.missing())
    with pytest.raises(PPError) as e:
        s.forward_tokens(0, [1])
    assert e.value.status == PP_E_MISSING
    # o_proj stored transposed: the same element count, the wrong shape.
    import torch
    from safetensors.torch import save_file
    name = "model.layers.1.self_attn.o_proj.weight"
    o = W[name].reshape(CFG.hidden, CFG.q_dim).T.copy()
    bad = str(tmp_path / "bad.safetensors")
    save_file({name: torch.from_numpy(o.view(np.int16).copy()).view(torch.bfloat16)}, bad)
    with pytest.raises(PPError) as e:
        s.load_safetensors(bad)
    assert e.value.status == PP_E_INVALID and "shape mismatch" in str(e.value)
    s.close()


def test_tapped_layers_match_the_oracle(gpu):
    """Taps on layers 0 and 1 of a 3-layer model, on a head shard (0, 2) and on a whole-model
    shard: the kept outputs equal the oracle's per-layer outputs (rel-L2 <= 1e-3), the wire
    form is their BF16 rounding, the hello carries them, and tapping the model's last layer
    or a layer outside the shard is refused. A shard with the 1-row decode kernel keeps its
    taps too (its 1-row steps run on the per-layer kernels while it taps)."""
    W = random_weights(CFG, seed=23)
    ref = oracle.OracleShard(CFG, 0, 3, 64, 8)
    ref.load(W)
    head, whole = Shard(CFG, (0, 2), 64, 8), Shard(CFG, (0, 3), 64, 8)
    for s in (head, whole):
        s.load(W)
        s.set_taps([1, 0, 1])
        assert s.tap_layers() == [0, 1]
        assert s.hello(s.range()[1])["taps"] == [0, 1]
    prompt = np.random.default_rng(5).integers(0, CFG.vocab_size, 17).tolist()
    pos = 0
    while pos < len(prompt):
        take = 8 if len(prompt) - pos >= 8 else 1
        toks = prompt[pos:pos + take]
        _, taps = ref.forward(pos, tokens=toks, taps=True)
        head.forward_tokens(pos, toks)
        whole.forward_tokens(pos, toks)
        for s in (head, whole):
            got = s.take_taps()
            assert len(got) == 2 and got[0].shape == (take, CFG.hidden)
            for l in range(2):
                assert rel_l2(got[l], taps[l]) <= 1e-3, (pos, l)
            wire = s.take_taps(bf16=True)
            for l in range(2):
                assert np.array_equal(wire[l], f32_to_bf16_bits(got[l]))
                assert np.allclose(bf16_bits_to_f32(wire[l]), got[l], rtol=1e-2, atol=1e-6)
        pos += take
    for bad in ([2], [3]):
        with pytest.raises(PPError) as e:
            whole.set_taps(bad)
        assert e.value.status == PP_E_INVALID
    with pytest.raises(PPError):
        head.set_taps([2])
    # The decode kernel leaves 1-row steps of a tapped shard to the per-layer kernels.
    big = QwenConfig(layers=2, hidden=1024, intermediate=3072, head_dim=128, n_heads=16,
                     n_kv_heads=8, vocab_size=1000, rms_norm_eps=1e-6, rope_theta=1e6)
    Wb = random_weights(big, seed=24)
    rb = oracle.OracleShard(big, 0, 2, 64, 8)
    rb.load(Wb)
    dec = Shard(big, (0, 2), 64, 8)
    dec.load(Wb)
    dec.set_decode_kernel(True)
    dec.set_taps([0])
    for p, t in enumerate([11, 12, 13]):
        _, taps = rb.forward(p, tokens=[t], taps=True)
        dec.forward_tokens(p, [t])
        assert rel_l2(dec.take_taps()[0], taps[0]) <= 1e-3
    dec.set_taps([])
    assert dec.take_taps() == []
    got = dec.forward_tokens(3, [14])
    assert rel_l2(got, rb.forward(3, tokens=[14])) <= 1e-3
    for s in (head, whole, dec):
        s.close()
