"""engine.h on the device against the oracle and the reference's golden
outputs, called through the C ABI with host buffers.

Bars (from the hot path's parity criteria): logits within 1e-3 max-abs of the
reference at every checked position, and greedy token sequences identical to
the reference's.
"""
import hashlib
import os

import numpy as np
import pytest

import pk_b200
import pk_synth
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


def test_golden_forward_and_greedy(tmp_path):
    g = np.load(os.path.join(GOLDEN, "forward_tiny.npz"))
    path = str(tmp_path / "tiny.gguf")
    pk_synth.write_model(path, "tiny-q4km", seed=int(g["seed"]))
    assert hashlib.sha256(open(path, "rb").read()).hexdigest() == str(g["sha256"])
    e = pk_b200.Engine(path, int(g["max_context"]))
    for pos, tok in enumerate(g["prompt"]):
        got = e.forward(int(tok), pos)
        assert np.abs(got - g["logits"][pos]).max() < LOGIT_TOL, pos
    n0 = len(g["prompt"])
    # 1) host argmax over engine_forward logits (the reference's own loop)
    tok, greedy = int(np.argmax(g["logits"][-1])), []
    for step in range(len(g["greedy"])):
        greedy.append(tok)
        tok = int(np.argmax(e.forward(tok, n0 + step)))
    assert greedy == [int(t) for t in g["greedy"]]
    # 2) device argmax, one call per token
    for pos, tok in enumerate(g["prompt"]):
        e.forward(int(tok), pos)
    tok, greedy = int(np.argmax(g["logits"][-1])), []
    for step in range(len(g["greedy"])):
        greedy.append(tok)
        tok = e.forward_greedy(tok, n0 + step)
    assert greedy == [int(t) for t in g["greedy"]]
    # 3) device-resident loop
    for pos, tok in enumerate(g["prompt"]):
        e.forward(int(tok), pos)
    first = int(np.argmax(g["logits"][-1]))
    toks, ms = e.generate_greedy(first, n0, len(g["greedy"]) - 1)
    assert [first] + [int(t) for t in toks] == [int(t) for t in g["greedy"]]
    assert ms > 0
    e.close()


@pytest.mark.parametrize("preset", ["tiny-q4km", "tiny-q5k", "tiny-legacy", "tiny-float"])
def test_engine_matches_oracle(orc, synth_model, preset):
    path = synth_model(preset)
    e = pk_b200.Engine(path, 128)
    o = orc.open(path, 128)
    assert e.config["seq_len"] == o.seq_len == 128
    toks = pk_synth.uniform_ints(5, 10, 3, o.vocab_size)
    worst = 0.0
    for pos, t in enumerate(toks):
        a, b = e.forward(int(t), pos), o.forward(int(t), pos)
        worst = max(worst, float(np.abs(a - b).max()))
    tok = int(np.argmax(b))
    for pos in range(len(toks), len(toks) + 40):
        a, b = e.forward(tok, pos), o.forward(tok, pos)
        worst = max(worst, float(np.abs(a - b).max()))
        assert int(np.argmax(a)) == o.greedy(b), (preset, pos)
        tok = o.greedy(b)
    assert worst < LOGIT_TOL, worst
    e.close()
    o.close()


def test_long_context_attention(orc, synth_model):
    """Positions well past one attention split per CTA (and the engine's
    256-position mark) against the oracle."""
    path = synth_model("tiny-q4km")
    e, o = pk_b200.Engine(path, 512), orc.open(path, 512)
    toks = pk_synth.uniform_ints(21, 400, 3, o.vocab_size)
    for pos, t in enumerate(toks):
        a, b = e.forward(int(t), pos), o.forward(int(t), pos)
        if pos % 50 == 49 or pos == len(toks) - 1:
            assert np.abs(a - b).max() < LOGIT_TOL, pos
    e.close()
    o.close()


def test_api_contracts(synth_model, ref):
    path = synth_model("tiny-q4km")
    e = pk_b200.Engine(path, 0)
    r = ref.open(path, 0)
    assert e.config == r.config
    assert e.file_context() == 512 and e.seq_len == 512
    assert e.kv_cache_bytes() == r.kv_cache_bytes()
    assert e.description() == r.description()
    assert e.format() == 2
    tk = e.tokenizer()
    assert tk.vocab_size == e.vocab_size and tk.bos_id == 1 and tk.eos_id == 2
    assert tk.byte_ids[0] == 3 and tk.byte_ids[255] == 258
    assert tk.vocab[300] == b" t300"
    assert e.is_stop(2) == 1 and e.is_stop(1) == 0
    # invalid inputs return NULL and leave the handle usable
    a = e.forward(1, 0)
    assert e.forward(-1, 0) is None and e.forward(e.vocab_size, 0) is None
    assert e.forward(1, -1) is None and e.forward(1, e.seq_len) is None
    assert e.forward_greedy(-1, 0) == -2
    assert np.array_equal(e.forward(1, 0), a)  # pos 0 restarts and overwrites
    # max_context caps, 0 means min(file, 4096)
    e2 = pk_b200.Engine(path, 100)
    assert e2.seq_len == 100 and e2.kv_cache_bytes() == e.kv_cache_bytes() * 100 // 512
    # two handles at once give the same answers
    for pos, t in enumerate([5, 6, 7]):
        assert np.array_equal(e.forward(t, pos), e2.forward(t, pos))
    with pytest.raises(RuntimeError):
        e.generate_greedy(1, 510, 5)  # runs past seq_len
    e.close()
    e2.close()
    r.close()


def test_open_close_cycles(synth_model):
    path = synth_model("tiny-legacy")
    first = None
    for _ in range(25):
        e = pk_b200.Engine(path, 32)
        y = e.forward(3, 0)
        if first is None:
            first = y
        assert np.array_equal(y, first)
        e.close()


@pytest.mark.slow
def test_tinyllama_shape_greedy_128_steps(orc, synth_model):
    """TinyLlama-1.1B shape, Q4_K_M mix: 32 seeded prompt ids, then 128
    greedy steps on the device identical to the oracle's; then the same 128
    steps again through engine_forward with the logits of every step within
    1e-3 of the oracle's."""
    path = synth_model("tinyllama-1.1b-q4km", seed=1234)
    e, o = pk_b200.Engine(path, 2048), orc.open(path, 2048)
    prompt = pk_synth.uniform_ints(42, 32, 3, o.vocab_size)
    worst = 0.0
    for pos, t in enumerate(prompt):
        a = e.forward(int(t), pos)
        b = o.forward(int(t), pos)
        worst = max(worst, float(np.abs(a - b).max()))
    tok = o.greedy(b)
    assert int(np.argmax(a)) == tok
    dev_tokens, _ = e.generate_greedy(tok, 32, 128)
    ref_tokens = []
    for step in range(128):
        a = e.forward(tok, 32 + step)  # rewrites the position generate_greedy filled
        b = o.forward(tok, 32 + step)
        worst = max(worst, float(np.abs(a - b).max()))
        tok = o.greedy(b)
        assert int(np.argmax(a)) == tok, step
        ref_tokens.append(tok)
    assert [int(t) for t in dev_tokens] == ref_tokens
    assert worst < LOGIT_TOL, worst
    e.close()
    o.close()


@pytest.mark.slow
@pytest.mark.parametrize("preset", ["llama2-7b-q4km", "llama3-8b-q5k"])
def test_7b_8b_shapes_match_oracle(orc, synth_model, preset):
    """Llama-2-7B and Llama-3-8B shapes (ffn_down rows longer than a ring
    stage, streamed in column chunks): 4 prompt ids and 4 greedy steps against
    the oracle, logits within 1e-3."""
    path = synth_model(preset, seed=1234)
    e, o = pk_b200.Engine(path, 64), orc.open(path, 64)
    assert e.launches_per_step() == 2  # the single cooperative step kernel
    prompt = pk_synth.uniform_ints(43, 4, 3, o.vocab_size)
    worst = 0.0
    for pos, t in enumerate(prompt):
        a = e.forward(int(t), pos)
        b = o.forward(int(t), pos)
        worst = max(worst, float(np.abs(a - b).max()))
    tok = o.greedy(b)
    dev_tokens, _ = e.generate_greedy(tok, 4, 4)
    ref_tokens = []
    for step in range(4):
        tok = o.greedy(o.forward(tok, 4 + step))
        ref_tokens.append(tok)
    assert [int(t) for t in dev_tokens] == ref_tokens
    assert worst < LOGIT_TOL, worst
    e.close()
    o.close()
