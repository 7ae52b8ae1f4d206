"""Parity at the contexts the larger configurations decode at, reached by
writing the same seeded keys and values into the device's cache
(engine_kv_write) and the oracle's (orc_kv_write, the reference's run-state
layout [layer][position][kv_dim], src/gguf_forward.c:197-226), then decoding
from there on both sides:

  * Llama-2-7B shape at a 1024-position context and Llama-3-8B shape at a
    4096-position context, 16 greedy steps of engine_forward (the decode
    step's attention splits positions over CTAs and merges the splits);
  * TinyLlama shape, 64 batched sequences after 512 positions each,
    8 steps of engine_forward_batch, 8 of the sequences checked;
  * a model whose output matrix is tied to the embedding table
    (src/gguf_model.c:257-266).

Bars: logits within 1e-3 max-abs of the oracle at every checked step, and
the same greedy tokens.
"""
import numpy as np
import pytest

import pk_b200
import pk_synth

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


def kv_rows(seed, layer, npos, kvd, scale=0.5):
    """Seeded keys and values for positions 0 .. npos - 1 of one layer."""
    k = pk_synth.gaussian(seed * 1000 + 2 * layer, npos * kvd, std=scale).reshape(npos, kvd)
    v = pk_synth.gaussian(seed * 1000 + 2 * layer + 1, npos * kvd, std=scale).reshape(npos, kvd)
    return k, v


def fill_context(e, o, cfg, ctx, seed, seq=-1, oracles=()):
    kvd = cfg["dim"] // cfg["n_heads"] * cfg["n_kv_heads"]
    for layer in range(cfg["n_layers"]):
        k, v = kv_rows(seed, layer, ctx, kvd)
        e.kv_write(layer, 0, k, v, seq=seq)
        for m in ([o] if o is not None else []) + list(oracles):
            for p in range(ctx):
                assert m.kv_write(layer, p, k[p], v[p]) == 1


@pytest.mark.slow
@pytest.mark.parametrize("preset,ctx", [("llama2-7b-q4km", 1024), ("llama3-8b-q5k", 4096)])
def test_decode_after_long_context(orc, synth_model, preset, ctx):
    path = synth_model(preset, seed=1234)
    steps = 16
    e, o = pk_b200.Engine(path, ctx + steps + 8), orc.open(path, ctx + steps + 8)
    fill_context(e, o, e.config, ctx, seed=7)
    tok, worst = 17, 0.0
    for i in range(steps):
        a, b = e.forward(tok, ctx + i), o.forward(tok, ctx + i)
        worst = max(worst, float(np.abs(a - b).max()))
        tok = o.greedy(b)
        assert int(np.argmax(a)) == tok, (preset, i)
    assert worst < LOGIT_TOL, (preset, worst)
    e.close()
    o.close()


@pytest.mark.slow
def test_batched_decode_after_512_positions(orc, synth_model):
    path = synth_model("tinyllama-1.1b-q4km", seed=1234)
    ctx, steps, B = 512, 8, 64
    e = pk_b200.Engine(path, ctx + steps + 8)
    e.batch_open(B)
    cfg = e.config
    checked = list(range(0, B, 9))  # 8 sequences
    oracles = {s: orc.open(path, ctx + steps + 8) for s in checked}
    for s in range(B):
        fill_context(e, None, cfg, ctx, seed=100 + s, seq=s, oracles=[oracles[s]] if s in oracles else [])
    toks = pk_synth.uniform_ints(77, B, 3, cfg["vocab_size"])
    seq = np.arange(B, dtype=np.int32)
    worst = 0.0
    for i in range(steps):
        nxt, lg = e.forward_batch(toks, np.full(B, ctx + i), seq, logits=True)
        for s in checked:
            want = oracles[s].forward(int(toks[s]), ctx + i)
            worst = max(worst, float(np.abs(lg[s] - want).max()))
            assert int(nxt[s]) == oracles[s].greedy(want), (s, i)
        toks = nxt
    assert worst < LOGIT_TOL, worst
    for m in oracles.values():
        m.close()
    e.close()


def test_batched_rows_need_their_earlier_positions(synth_model):
    """engine_forward_batch refuses a row whose earlier positions hold no
    K/V (neither earlier steps, engine_kv_write, nor rows of the call), and
    the handle stays usable."""
    path = synth_model("tiny-q4km")
    e = pk_b200.Engine(path, 64)
    e.batch_open(2)
    assert e.forward_batch([5], [3], [0]) is None  # positions 0..2 of sequence 0 were never filled
    assert "no K/V" in e.last_error()
    assert e.forward_batch([5, 6, 7], [0, 1, 2], [0, 0, 0]) is not None  # a prompt chunk fills 0..2
    assert e.forward_batch([8], [3], [0]) is not None
    assert e.forward_batch([8], [1], [1]) is None  # sequence 1 is still empty
    kvd = e.config["dim"] // e.config["n_heads"] * e.config["n_kv_heads"]
    for layer in range(e.config["n_layers"]):
        k, v = kv_rows(3, layer, 1, kvd)
        e.kv_write(layer, 0, k, v, seq=1)
    assert e.forward_batch([8], [1], [1]) is not None  # position 0 was written directly
    with pytest.raises(RuntimeError):
        e.kv_write(0, 5, k, v, seq=1)  # would leave a gap at 2..4
    e.close()


def test_tied_output_matches_oracle(orc, synth_model):
    """A file without output.weight decodes through the embedding table
    (src/gguf_model.c:257-266) on the device as in the oracle."""
    path = synth_model("tiny-q4km", seed=9, tied_output=1)
    e, o = pk_b200.Engine(path, 64), orc.open(path, 64)
    toks = pk_synth.uniform_ints(19, 6, 3, o.vocab_size)
    worst = 0.0
    for pos, t in enumerate(toks):
        a, b = e.forward(int(t), pos), o.forward(int(t), pos)
        worst = max(worst, float(np.abs(a - b).max()))
    tok = o.greedy(b)
    for pos in range(len(toks), len(toks) + 20):
        a, b = e.forward(tok, pos), o.forward(tok, pos)
        worst = max(worst, float(np.abs(a - b).max()))
        assert int(np.argmax(a)) == o.greedy(b), pos
        tok = o.greedy(b)
    assert worst < LOGIT_TOL, worst
    e.close()
    o.close()
