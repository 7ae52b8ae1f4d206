"""Tensor-parallel placement (engine_tp_plan, include/engine_ext.h) and the
host-side handle exchange, on the CPU.

The plan must give every query head, KV head, hidden quant block, output row
and residual-stream element to the ranks exactly as the split rules say:
heads by rank, KV heads by rank or shared when ranks outnumber them, hidden
slices on whole blocks of ffn_down, attn_output columns on whole blocks.
"""
import multiprocessing as mp
import os
import socket

import pytest

import pk_b200

MODELS = {
    # name: (dim, hidden, heads, kv_heads, vocab, wo_block, down_block)
    "tinyllama": (2048, 5632, 32, 4, 32000, 256, 256),
    "llama2-7b": (4096, 11008, 32, 32, 32000, 256, 256),
    "llama3-8b": (4096, 14336, 32, 8, 128256, 256, 256),
    "tp-q4km": (1024, 2048, 8, 2, 2048, 256, 256),
    "legacy": (1024, 2048, 8, 8, 1000, 32, 32),
}


@pytest.mark.parametrize("name", list(MODELS))
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_everything_once(name, world):
    dim, hid, nh, nkv, voc, wo_bw, dn_bw = MODELS[name]
    hs = dim // nh
    try:
        plans = [pk_b200.tp_plan(dim, hid, nh, nkv, voc, wo_bw, dn_bw, r, world) for r in range(world)]
    except ValueError:
        # the only refusals: Wo blocks straddling the head split
        assert (nh // world * hs) % wo_bw != 0
        return
    q = sorted(h for p in plans for h in range(p["q_head0"], p["q_head0"] + p["q_heads"]))
    assert q == list(range(nh))
    hidden = sorted(i for p in plans for i in range(p["hid0"], p["hid0"] + p["hid"]))
    assert hidden == list(range(hid))
    assert all(p["hid0"] % dn_bw == 0 and p["hid"] % dn_bw == 0 and p["hid"] > 0 for p in plans)
    vocab = [i for p in plans for i in range(p["voc0"], p["voc0"] + p["voc"])]
    assert vocab == list(range(voc))
    own = [i for p in plans for i in range(p["own0"], p["own0"] + p["own"])]
    assert own == list(range(dim))
    kvm = nh // nkv
    for p in plans:
        assert (p["q_heads"] * hs) % wo_bw == 0
        for h in range(p["q_head0"], p["q_head0"] + p["q_heads"]):
            assert p["kv_head0"] <= h // kvm < p["kv_head0"] + p["kv_heads"]
    if nkv % world == 0:
        kv = sorted(g for p in plans for g in range(p["kv_head0"], p["kv_head0"] + p["kv_heads"]))
        assert kv == list(range(nkv))


def test_plan_refusals_carry_a_message():
    with pytest.raises(ValueError, match="attention heads"):
        pk_b200.tp_plan(2048, 5632, 32, 4, 32000, 256, 256, 0, 3)
    with pytest.raises(ValueError, match="attn_output"):
        pk_b200.tp_plan(1024, 2048, 8, 2, 2048, 256, 256, 0, 8)
    with pytest.raises(ValueError, match="ffn_down"):
        pk_b200.tp_plan(1024, 512, 8, 8, 2048, 32, 256, 0, 4)
    with pytest.raises(ValueError, match="world"):
        pk_b200.tp_plan(1024, 2048, 8, 2, 2048, 256, 256, 2, 2)
    with pytest.raises(ValueError, match="KV heads"):
        pk_b200.tp_plan(1536, 3072, 12, 3, 2048, 32, 256, 0, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
    try:
        mine = bytes([rank]) * 64
        q.put((rank, pk_b200.tp_exchange(mine, world)))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_over_gloo_in_rank_order():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = b"".join(bytes([r]) * 64 for r in range(world))
    assert got[0] == want and got[1] == want


def _absent_peer_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        q.put((rank, "left"))  # leaves between steps: never joins the exchange
        return
    try:
        pk_b200.tp_exchange(bytes([rank]) * 64, world)
        q.put((rank, "no error"))
    except Exception as e:  # the process group's timeout ends the collective
        q.put((rank, "error: " + type(e).__name__))


def test_exchange_with_an_absent_rank_ends_in_an_error_not_a_hang():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "left"
    assert got[0].startswith("error"), got[0]
