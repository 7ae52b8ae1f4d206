"""Tensor-parallel decode (engine_open_tp / engine_tp_connect) on 2, 4 and 8
GPUs against the oracle's single-process forward of the same model (at 4
and 8 ranks there are more ranks than KV heads, so ranks share KV heads).

One spawned process per GPU; the ranks exchange their 64-byte handles over
gloo on the host, then decode the same token sequence. Every rank's
engine_forward must return the full logits within 1e-3 max-abs of the
oracle, and the greedy tokens (device argmax across the ranks) must be the
oracle's. Skipped when the machine has fewer GPUs than ranks.
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
