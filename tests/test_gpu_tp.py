"""Tensor-parallel decode (engine_open_tp / engine_tp_connect) on 2, 4 and 8
GPUs against the oracle's single-process forward of the same model (at 4
and 8 ranks there are more ranks than KV heads, so ranks share KV heads).

One spawned process per GPU; the ranks exchange their 64-byte handles over
gloo on the host, then decode the same token sequence. Every rank's
engine_forward must return the full logits within 1e-3 max-abs of the
oracle, and the greedy tokens (device argmax across the ranks) must be the
oracle's. The same holds for the batched step on the group
(engine_forward_batch: a prompt chunk, single rows, a late-joining
sequence, with and without logits) and for engine_prefill followed by
engine_forward. Skipped when the machine has fewer GPUs than ranks.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import pk_b200

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
PROMPT = [5, 17, 300, 41, 7, 1999, 2, 64]
STEPS = 40


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, path, out_dir):
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=120))
    try:
        e = pk_b200.Engine(path, 128, device=rank, rank=rank, world=world)
        e.tp_connect(pk_b200.tp_exchange(e.tp_handle(), world))
        logits = [e.forward(t, pos) for pos, t in enumerate(PROMPT)]
        assert all(lg is not None for lg in logits), e.last_error()
        first = int(np.argmax(logits[-1]))
        toks, _ = e.generate_greedy(first, len(PROMPT), STEPS)
        single = e.forward_greedy(int(toks[-1]), len(PROMPT) + STEPS)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), logits=np.stack(logits), toks=np.asarray(toks),
                 first=first, single=single)
        e.close()
    finally:
        dist.destroy_process_group()


def _oracle(orc, path):
    m = orc.open(path, 128)
    logits = [np.asarray(m.forward(t, pos)).copy() for pos, t in enumerate(PROMPT)]
    tok, toks = int(np.argmax(logits[-1])), []
    for i in range(STEPS + 1):
        tok = int(np.argmax(m.forward(tok, len(PROMPT) + i)))
        toks.append(tok)
    m.close()
    return np.stack(logits), toks


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_decode_matches_oracle(orc, synth_model, tmp_path, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    path = synth_model("tp8-q4km" if world == 8 else "tp-q4km")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, path, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    want_logits, want_toks = _oracle(orc, path)
    for r in range(world):
        got = np.load(os.path.join(str(tmp_path), f"rank{r}.npz"))
        err = float(np.max(np.abs(got["logits"] - want_logits)))
        assert err <= LOGIT_TOL, (r, err)
        assert int(got["first"]) == int(np.argmax(want_logits[-1]))
        assert list(got["toks"]) == want_toks[:STEPS], r
        assert int(got["single"]) == want_toks[STEPS], r


def _batch_schedule():
    """The rows of each batched step: (tokens, positions, sequence ids, with
    logits). Sequence 0 starts with its prompt as one chunk, sequence 2 with
    one token, sequence 1 joins at the second step; later steps feed back
    the greedy tokens (None: the previous step's token of that sequence)."""
    steps = [(list(PROMPT) + [3], list(range(len(PROMPT))) + [0], [0] * len(PROMPT) + [2], True)]
    for i in range(6):
        seqs = [0, 2] if i == 0 else [2, 0, 1]
        toks = [None] * len(seqs)
        if i == 0:
            seqs, toks = [0, 2, 1], [None, None, 100]
        steps.append((toks, None, seqs, i != 3))  # step 4: greedy tokens only
    return steps


def _batch_rank(rank, world, port, path, out_dir):
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=120))
    try:
        e = pk_b200.Engine(path, 128, device=rank, rank=rank, world=world)
        e.tp_connect(pk_b200.tp_exchange(e.tp_handle(), world))
        e.batch_open(4)
        nxt_of, pos_of = {}, {}
        rec_seq, rec_pos, rec_tok, rec_logits, rec_next = [], [], [], [], []
        for toks, poss, seqs, with_logits in _batch_schedule():
            if poss is None:
                poss = [pos_of.get(s, 0) for s in seqs]
                toks = [nxt_of[s] if t is None else t for t, s in zip(toks, seqs)]
            out = e.forward_batch(toks, poss, seqs, logits=with_logits)
            assert out is not None, e.last_error()
            nxt, lg = out
            for i, s in enumerate(seqs):
                nxt_of[s], pos_of[s] = int(nxt[i]), poss[i] + 1
                rec_seq.append(s)
                rec_pos.append(poss[i])
                rec_tok.append(toks[i])
                rec_next.append(int(nxt[i]))
                rec_logits.append(lg[i] if with_logits else np.full(e.vocab_size, np.nan, dtype=np.float32))
        np.savez(os.path.join(out_dir, f"brank{rank}.npz"), seq=np.asarray(rec_seq), pos=np.asarray(rec_pos),
                 tok=np.asarray(rec_tok), nxt=np.asarray(rec_next), logits=np.stack(rec_logits))
        e.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_batched_decode_matches_oracle(orc, synth_model, tmp_path, world):
    """engine_forward_batch on a tensor-parallel group: three sequences at
    different positions (a prompt chunk, single rows, a late joiner), with and
    without logits; every rank's rows against the oracle's single-sequence
    forward of the same tokens at the same positions."""
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    path = synth_model("tp8-q4km" if world == 8 else "tp-q4km")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_batch_rank, args=(r, world, port, path, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ref = np.load(os.path.join(str(tmp_path), "brank0.npz"))
    want = {}
    for s in sorted(set(int(v) for v in ref["seq"])):
        rows = sorted((int(p), int(t)) for q, p, t in zip(ref["seq"], ref["pos"], ref["tok"]) if int(q) == s)
        assert [p for p, _ in rows] == list(range(len(rows)))
        m = orc.open(path, 128)
        for p, t in rows:
            want[(s, p)] = np.asarray(m.forward(t, p)).copy()
        m.close()
    for r in range(world):
        got = np.load(os.path.join(str(tmp_path), f"brank{r}.npz"))
        for i in range(len(got["seq"])):
            w = want[(int(got["seq"][i]), int(got["pos"][i]))]
            assert int(got["nxt"][i]) == int(np.argmax(w)), (r, i)
            if not np.isnan(got["logits"][i][0]):
                err = float(np.max(np.abs(got["logits"][i] - w)))
                assert err <= LOGIT_TOL, (r, i, err)


def _prefill_rank(rank, world, port, path, out_dir):
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=120))
    try:
        e = pk_b200.Engine(path, 128, device=rank, rank=rank, world=world)
        e.tp_connect(pk_b200.tp_exchange(e.tp_handle(), world))
        prompt = [(37 * i + 11) % e.vocab_size for i in range(70)]  # two chunks: 64 + 6
        tok, last = e.prefill(prompt, 0, logits=True)
        after = []
        for i in range(4):
            lg = e.forward(tok, len(prompt) + i)
            assert lg is not None, e.last_error()
            after.append(np.asarray(lg).copy())
            tok = int(np.argmax(lg))
        np.savez(os.path.join(out_dir, f"prank{rank}.npz"), prompt=np.asarray(prompt), final=tok, last=last,
                 after=np.stack(after))
        e.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_prefill_matches_oracle(orc, synth_model, tmp_path, world):
    """engine_prefill on a tensor-parallel group (70 tokens: a 64-row chunk
    and a 6-row chunk through the tensor-parallel batched step into the
    decode step's cache), then engine_forward continuing after it: the last
    prompt position's logits and four decode steps against the oracle."""
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    path = synth_model("tp8-q4km" if world == 8 else "tp-q4km")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_prefill_rank, args=(r, world, port, path, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got0 = np.load(os.path.join(str(tmp_path), "prank0.npz"))
    prompt = [int(t) for t in got0["prompt"]]
    m = orc.open(path, 128)
    lg = None
    for pos, t in enumerate(prompt):
        lg = np.asarray(m.forward(t, pos)).copy()
    want_last, tok, want_after = lg, int(np.argmax(lg)), []
    for i in range(4):
        lg = np.asarray(m.forward(tok, len(prompt) + i)).copy()
        want_after.append(lg)
        tok = int(np.argmax(lg))
    m.close()
    for r in range(world):
        got = np.load(os.path.join(str(tmp_path), f"prank{r}.npz"))
        assert float(np.max(np.abs(got["last"] - want_last))) <= LOGIT_TOL, r
        assert float(np.max(np.abs(got["after"] - np.stack(want_after)))) <= LOGIT_TOL, r
        assert int(got["final"]) == tok, r
