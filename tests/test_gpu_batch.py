"""Batched decode (engine_batch_open / engine_forward_batch) against the
oracle's single-sequence forward, through the C ABI.

Every sequence of a batched step must get the logits the oracle gives that
sequence alone (within 1e-3 max-abs) and the same greedy token, whatever the
other sequences in the batch, their positions and the order of seq_ids.
"""
import numpy as np
import pytest

import pk_b200

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def prompts(nseq, vocab, seed):
    rng = np.random.default_rng(seed)
    return [list(rng.integers(0, vocab, size=int(rng.integers(2, 7)))) for _ in range(nseq)]


def run_batched(orc, path, nseq, steps, seq_ids, seed, ctx=128, stagger=True, check=None):
    """Feed each sequence its prompt then its own greedy tokens; sequence s
    joins at step s when staggered. Compares every produced row with the
    oracle's forward of that sequence."""
    e = pk_b200.Engine(path, ctx, device=0)
    e.batch_open(max(seq_ids) + 1)
    vocab = e.vocab_size
    ps = prompts(nseq, vocab, seed)
    refs = {s: orc.open(path, ctx) for s in (check if check is not None else range(nseq))}
    feed = [list(p) for p in ps]  # tokens still to feed per sequence
    pos = [0] * nseq
    worst = 0.0
    checked = 0
    for step in range(steps):
        active = [s for s in range(nseq) if (not stagger or s <= step) and pos[s] < ctx - 1]
        if not active:
            break
        toks = [feed[s][0] for s in active]
        out = e.forward_batch(toks, [pos[s] for s in active], [seq_ids[s] for s in active], logits=True)
        assert out is not None, e.last_error()
        nxt, lg = out
        for i, s in enumerate(active):
            if s in refs:
                want = np.asarray(refs[s].forward(toks[i], pos[s])).copy()
                worst = max(worst, float(np.max(np.abs(lg[i] - want))))
                assert int(nxt[i]) == int(np.argmax(want)), (step, s)
                checked += 1
            feed[s].pop(0)
            if not feed[s]:
                feed[s].append(int(nxt[i]))
            pos[s] += 1
    for r in refs.values():
        r.close()
    e.close()
    assert checked > 0
    return worst


def test_batch_matches_oracle_staggered(orc, synth_model):
    path = synth_model("tiny-q4km")
    worst = run_batched(orc, path, nseq=6, steps=24, seq_ids=[5, 0, 7, 2, 3, 6], seed=11)
    assert worst <= LOGIT_TOL, worst


def test_batch_of_64_matches_oracle(orc, synth_model):
    path = synth_model("tp-q4km")
    worst = run_batched(orc, path, nseq=64, steps=5, seq_ids=list(range(64))[::-1], seed=3, stagger=False)
    assert worst <= LOGIT_TOL, worst


def test_batch_legacy_formats(orc, synth_model):
    # Q4_0 / Q8_0 weights: the CUDA-core path for every matrix
    path = synth_model("tiny-legacy")
    worst = run_batched(orc, path, nseq=5, steps=10, seq_ids=[0, 1, 2, 3, 4], seed=5)
    assert worst <= LOGIT_TOL, worst


def test_batch_prefill_chunks_match_oracle(orc, synth_model):
    # one call carries a whole prompt of sequence 0 (positions 0..39), a
    # chunk of sequence 2's prompt and a decode row of sequence 1
    path = synth_model("tiny-q4km")
    e = pk_b200.Engine(path, 128, device=0)
    e.batch_open(3)
    rng = np.random.default_rng(21)
    p0 = list(rng.integers(0, e.vocab_size, size=40))
    p1 = list(rng.integers(0, e.vocab_size, size=3))
    p2 = list(rng.integers(0, e.vocab_size, size=20))
    refs = [orc.open(path, 128) for _ in range(3)]
    worst = 0.0
    # sequence 1 first decodes its first two tokens alone
    for pos, t in enumerate(p1[:2]):
        nxt, lg = e.forward_batch([t], [pos], [1], logits=True)
        want = refs[1].forward(int(t), pos)
        worst = max(worst, float(np.max(np.abs(lg[0] - want))))
    toks = p0 + p2[:10] + [p1[2]]
    poss = list(range(40)) + list(range(10)) + [2]
    seqs = [0] * 40 + [2] * 10 + [1]
    nxt, lg = e.forward_batch(toks, poss, seqs, logits=True)
    for i, (t, p, s_) in enumerate(zip(toks, poss, seqs)):
        want = refs[s_].forward(int(t), p)
        worst = max(worst, float(np.max(np.abs(lg[i] - want))))
        assert int(nxt[i]) == int(np.argmax(want)), i
    # the rest of sequence 2's prompt in a second chunk
    nxt, lg = e.forward_batch(p2[10:], list(range(10, 20)), [2] * 10, logits=True)
    for i, t in enumerate(p2[10:]):
        want = refs[2].forward(int(t), 10 + i)
        worst = max(worst, float(np.max(np.abs(lg[i] - want))))
        assert int(nxt[i]) == int(np.argmax(want)), i
    for r in refs:
        r.close()
    e.close()
    assert worst <= LOGIT_TOL, worst


def test_batch_refuses_bad_arguments(synth_model):
    path = synth_model("tiny-q4km")
    e = pk_b200.Engine(path, 64, device=0)
    assert e.forward_batch([1], [0], [0]) is None  # before engine_batch_open
    e.batch_open(4)
    assert e.forward_batch([1, 2], [0, 0], [1, 1]) is None          # repeated (sequence, position)
    assert e.forward_batch([1], [64], [0]) is None                  # position past the context
    assert e.forward_batch([e.vocab_size], [0], [0]) is None        # token outside the vocabulary
    assert e.forward_batch([1], [0], [4]) is None                   # sequence id past max_seqs
    assert e.forward_batch([1] * 65, list(range(65)), [0] * 65) is None  # more than 64 rows
    out = e.forward_batch([1, 2], [0, 0], [2, 0])
    assert out is not None and out[1] is None
    # the single-sequence path is independent of the batched state
    assert e.forward(1, 0) is not None
    e.close()


@pytest.mark.slow
def test_batch_tinyllama_shape(orc, synth_model):
    path = synth_model("tinyllama-1.1b-q4km")
    worst = run_batched(orc, path, nseq=64, steps=3, seq_ids=list(range(64)), seed=9, ctx=64, stagger=False,
                        check={0, 17, 63})
    assert worst <= LOGIT_TOL, worst


def test_batch_q5k_model_matches_oracle(orc, synth_model):
    """Q5_K attention and gate/up matrices on the tensor-core matmul, Q6_K
    ffn_down and Q8_0 output on the tile kernel (the Llama-3-8B mix)."""
    path = synth_model("tiny-q5k")
    worst = run_batched(orc, path, nseq=8, steps=12, seq_ids=list(range(8)), seed=21)
    assert worst <= LOGIT_TOL, worst
