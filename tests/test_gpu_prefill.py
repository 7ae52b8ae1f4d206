"""engine_prefill (include/engine_ext.h): a prompt through the batched step,
in chunks of up to 64 rows, into the cache engine_forward uses. The
reference feeds prompts one token at a time (src/pocket.c:294-301), so the
oracle is its forward over the same tokens: the logits of the prompt's last
position within 1e-3 max-abs, the same greedy token, and the same logits and
greedy tokens for the decode steps that follow through engine_forward.
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


def check(orc, path, ctx, lead, n, steps, seed):
    """`lead` tokens through engine_forward, then n through engine_prefill,
    then `steps` greedy decode steps through engine_forward."""
    e, o = pk_b200.Engine(path, ctx), orc.open(path, ctx)
    toks = pk_synth.uniform_ints(seed, lead + n, 3, o.vocab_size)
    worst = 0.0
    for pos in range(lead):
        a, b = e.forward(int(toks[pos]), pos), o.forward(int(toks[pos]), pos)
        worst = max(worst, float(np.abs(a - b).max()))
    tok, lg = e.prefill(toks[lead:], pos0=lead, logits=True)
    for pos in range(lead, lead + n):
        b = o.forward(int(toks[pos]), pos)
    worst = max(worst, float(np.abs(lg - b).max()))
    assert tok == o.greedy(b)
    for pos in range(lead + n, lead + n + steps):
        a, b = e.forward(tok, pos), o.forward(tok, pos)
        worst = max(worst, float(np.abs(a - b).max()))
        assert int(np.argmax(a)) == o.greedy(b), pos
        tok = o.greedy(b)
    e.close()
    o.close()
    return worst


@pytest.mark.parametrize("preset", ["tiny-q4km", "tiny-q5k", "tiny-legacy"])
def test_prefill_then_decode_matches_oracle(orc, synth_model, preset):
    path = synth_model(preset)
    assert check(orc, path, 256, lead=0, n=150, steps=20, seed=3) < LOGIT_TOL  # chunks of 64, 64, 22
    assert check(orc, path, 256, lead=10, n=70, steps=10, seed=4) < LOGIT_TOL  # after engine_forward calls


@pytest.mark.slow
def test_prefill_tinyllama_shape(orc, synth_model):
    path = synth_model("tinyllama-1.1b-q4km", seed=1234)
    assert check(orc, path, 512, lead=0, n=96, steps=8, seed=5) < LOGIT_TOL


def test_prefill_rejects_bad_arguments(synth_model):
    path = synth_model("tiny-q4km")
    e = pk_b200.Engine(path, 64)
    with pytest.raises(RuntimeError):
        e.prefill([], 0)
    with pytest.raises(RuntimeError):
        e.prefill([1] * 10, 60)  # past the context
    with pytest.raises(RuntimeError):
        e.prefill([1, e.vocab_size], 0)  # token outside the vocabulary
    tok, _ = e.prefill([1, 2, 3], 0)  # the handle stays usable
    assert tok >= 0 and e.forward(tok, 3) is not None
    e.close()
