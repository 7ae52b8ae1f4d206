"""Benchmark: greedy decode tokens/s of the GGUF quantized decode path.

Default workload: TinyLlama-1.1B architecture, Q4_K_M mix (synthetic
random-init weights), batch 1: a 32-id seeded prompt, then W warm-up and K
timed greedy decode steps; one step = one decoded token.

  value  device-timed tokens/s of K greedy steps run back to back on the
         device (engine_generate_greedy: CUDA events on the engine's stream),
         weights resident in HBM.
  e2e    the same K steps through the reference-facing C ABI with host
         buffers: engine_forward() (token/pos up, logits down) + host argmax.

Under torchrun (N > 1), on the TinyLlama shape every GPU decodes its own
independent sequence (data parallel, weak scaling, no collective on the
data path; value = N x the tokens / the slowest rank's time; the B=64 line
likewise runs 64 sequences per GPU). The 7B/8B shapes (and --tp) decode ONE
sequence tensor-parallel (strong scaling): each GPU holds its attention
heads, FFN hidden slice and vocabulary rows, and the decode kernels
all-reduce the partial sums over NVLink peer memory; value = the sequence's
tokens / the slowest rank's time. The roofline peak is N x the HBM figure.

Extra objects of the default line:
  b64     64 independent sequences after a 512-token context, 128 greedy
          steps through engine_forward_batch.
  matvec  (N = 1) the isolated fused dequant-matvec sweep, 8 shapes x 5
          formats through gguf_cuda_matvec, GB/s of packed weights and the
          fraction of the measured HBM peak, beside the reference's own
          gguf_matvec on the same blocks (all host threads) and the relative
          L2 distance of the outputs.
  llama2_7b_b16  (N = 1) Llama-2-7B shape, 16 sequences after a 1024-position
          context, batched decode.
  llama3_8b      (N = 1) Llama-3-8B shape: 2048-token prefill, 512 decode
          steps, and decode at the end of an 8192 context.
  tp7b    the Llama-2-7B shape decoded tensor-parallel over the run's N GPUs
          (N = 1: one GPU): tok/s, e2e, roofline against N x the HBM peak,
          and whether the greedy tokens match a 1-GPU run of the same prompt.

  --impl reference   times the reference's own CPU engine (compiled from its
                     sources into oracle/_ref) on the same model file, with
                     the same `config`; the model file, if missing, is
                     written by the pk_synth_cli command.
  --workload matvec  the isolated fused dequant-matvec sweep (GB/s per type
                     and shape), printed as extra lines for profiling.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llm-inference-c_b200"))
import pk_synth  # noqa: E402

WORKLOADS = {
    "tinyllama": dict(preset="tinyllama-1.1b-q4km", name="TinyLlama-1.1B-arch Q4_K_M, B=1 greedy decode",
                      prompt=32, context=2048),
    "llama2-7b": dict(preset="llama2-7b-q4km", name="Llama-2-7B-arch Q4_K_M, B=1 greedy decode",
                      prompt=32, context=4096),
    "llama3-8b": dict(preset="llama3-8b-q5k", name="Llama-3-8B-arch Q5_K/Q6_K/Q8_0, B=1 greedy decode",
                      prompt=32, context=8192),
}
PUBLISHED_TOKS = 8.03  # reference, TinyLlama-1.1B-Chat Q4_K_M, 8 threads (documentation/PERFORMANCE.md:60)
VS_BASELINE_NOTE = "published 8.03 tok/s: reference on 8 laptop cores, real TinyLlama Q4_K_M file"

# DRAM bytes (read + write) of one decode-step launch of phase_kernel, from
# one ncu capture of that launch (the phase_kernel summary under profiles/:
# dram__bytes_read.sum + dram__bytes_write.sum); None for workloads without
# a capture.
NCU_TRAFFIC = {"tinyllama-1.1b-q4km": 639016192 + 6886400}
FALLBACK_HBM_GBS = 6650.0
MODEL_SEED = 1234


_T0 = time.perf_counter()


def note(msg):
    """Progress on stderr (the JSON line is the only stdout)."""
    print(f"[bench {time.perf_counter() - _T0:7.1f}s] {msg}", file=sys.stderr, flush=True)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def model_path(preset):
    d = os.environ.get("PK_BENCH_DIR", "/tmp/pk_bench")
    os.makedirs(d, exist_ok=True)
    return os.path.join(d, f"{preset}-{MODEL_SEED}.gguf")


def ensure_model(preset, rank, barrier, via_cli=False):
    """The seeded synthetic GGUF file of `preset` (written once per box by
    rank 0). via_cli: written by the pk_synth_cli command in a child process,
    so that the caller never loads the writer library (the reference arm)."""
    path = model_path(preset)
    if rank == 0 and not os.path.exists(path):
        tmp = path + ".tmp"
        if via_cli:
            pk_synth.write_model_cli(tmp, preset, seed=MODEL_SEED)
        else:
            pk_synth.write_model(tmp, preset, seed=MODEL_SEED)
        os.replace(tmp, path)
    barrier()
    return path


def kv_bytes_per_step(cfg, positions, entry_bytes=4):
    kvd = cfg["dim"] // cfg["n_heads"] * cfg["n_kv_heads"]
    # K and V read for positions 0..pos, plus the K/V row written
    return sum(2 * cfg["n_layers"] * (p + 2) * kvd * entry_bytes for p in positions) / len(positions)


def kv_entry_bytes():
    return 2 if os.environ.get("POCKET_CUDA_KV") == "f16" else 4


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a moment to start: wait for its first sample so
            # that a short timed region still has samples around it
            t0 = time.perf_counter()
            while not self.rows and time.perf_counter() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.02)
            self.first = len(self.rows)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            # one sample taken after the region ends (at least 100 ms apart)
            n, t0 = len(self.rows), time.perf_counter()
            while len(self.rows) <= n and time.perf_counter() - t0 < 1.0 and self.proc.poll() is None:
                time.sleep(0.02)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def reference_decode(path, prompt, steps, warmup, budget_s):
    """The reference engine (its own C sources, OpenMP over all host cores):
    prompt, warm-up, then up to `steps` timed greedy tokens within budget_s."""
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    if not oracle.ref_available():
        return None
    ref = oracle.Reference()
    m = ref.open(path, prompt + warmup + steps + 1)
    tok = 1
    for pos, t in enumerate(prompt_ids(prompt, m.vocab_size, 0)):
        m.forward_ptr(int(t), pos)
    pos = prompt
    for _ in range(warmup):
        tok = m.greedy_ptr(m.forward_ptr(tok, pos))
        pos += 1
    done, t0 = 0, time.perf_counter()
    while done < steps:
        tok = m.greedy_ptr(m.forward_ptr(tok, pos))
        pos += 1
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    m.close()
    return {"value": done / dt, "unit": "tok/s", "cores": cores, "kind": "reference",
            "sample": f"{done} greedy decode tokens at positions {prompt + warmup}..{pos - 1} after a "
                      f"{prompt}-id prompt, same model file, OMP_NUM_THREADS={cores}"}


def _mix64(z):
    """SplitMix64's output function on uint64 arrays (wrapping arithmetic),
    as pks_uniform_ints in synth/gguf_synth.c computes it."""
    z = z + np.uint64(0x9E3779B97F4A7C15)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def uniform_ints(seed, n, lo, hi):
    """pk_synth.uniform_ints without the writer library: lo + (mix64(seed ^
    mix64(i)) mod (hi - lo)) for i < n."""
    with np.errstate(over="ignore"):
        i = np.arange(n, dtype=np.uint64)
        r = _mix64(np.uint64(seed) ^ _mix64(i))
    return (lo + (r % np.uint64(hi - lo)).astype(np.int64)).astype(np.int32)


def prompt_ids(n, vocab, rank):
    return uniform_ints(4242 + rank, n, 3, vocab)


def workload_config(wl, path, args, world, tp):
    """The `config` of the B=1 line, identical in both arms."""
    pos0 = wl["prompt"] + args.warmup
    return {"workload": wl["name"], "model_file": os.path.basename(path), "batch_per_gpu": 1,
            "prompt": wl["prompt"], "positions": [pos0, pos0 + args.steps - 1], "kv_cache": args.kv,
            "parallelism": f"tensor parallel over {world} GPUs (one sequence)" if tp
            else (f"data parallel: {world} GPUs, one independent sequence each" if world > 1 else "1 GPU"),
            "l2": "weights streamed per step exceed the 126 MB L2 (no flush needed)"}


def run_reference_arm(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    path = ensure_model(wl["preset"], 0, lambda: None, via_cli=True)
    base = reference_decode(path, wl["prompt"], args.steps, args.warmup, budget_s=150.0)
    if base is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref.so was not built"}))
        return 0
    tp = world > 1 and (args.tp or args.workload != "tinyllama")
    line = {"metric": "decode tok/s (B=1)", "value": base["value"], "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / base["value"],
            "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": base["value"] / PUBLISHED_TOKS,
            "dtype": "f32 (packed Q4_K/Q6_K weights)", "data": "synthetic random-init weights N(0,0.02), seeded prompt ids",
            "vs_baseline_note": VS_BASELINE_NOTE,
            "config": workload_config(wl, path, args, world, tp), "impl": "reference", "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def run_matvec_sweep(args):
    import torch
    import pk_b200
    torch.cuda.set_device(0)
    hbm, _ = peaks()
    shapes = [(2048, 2048), (256, 2048), (5632, 2048), (2048, 5632), (32000, 2048), (4096, 4096),
              (14336, 4096), (128256, 4096)]
    only = None
    if args.only:  # e.g. "Q4_K:128256x4096"
        t, shp = args.only.split(":")
        only = (t, tuple(int(v) for v in shp.split("x")))
    for name, qt in (("Q4_0", 2), ("Q8_0", 8), ("Q4_K", 12), ("Q5_K", 13), ("Q6_K", 14)):
        for rows, cols in shapes:
            if only is not None and (name, (rows, cols)) != only:
                continue
            rb = pk_b200.row_bytes(qt, cols)
            nbytes = rows * rb
            copies = max(1, min(8, (512 << 20) // nbytes))  # rotate > 2x L2 of weight copies
            wb = pk_synth.random_matrix(qt, rows, cols, seed=rows + qt)
            ws = [torch.from_numpy(wb).cuda() for _ in range(copies)]
            x = torch.from_numpy(pk_synth.gaussian(1, cols)).cuda()
            y = torch.empty(rows, device="cuda")
            wts = [pk_b200.make_weight(w.data_ptr(), qt, rows, cols) for w in ws]
            st = torch.cuda.current_stream().cuda_stream
            for i in range(3):
                pk_b200.matvec(wts[i % copies], x.data_ptr(), y.data_ptr(), st)
            reps = max(args.steps, 20)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for i in range(reps):
                pk_b200.matvec(wts[i % copies], x.data_ptr(), y.data_ptr(), st)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            gbs = nbytes / (ms * 1e-3) / 1e9
            print(json.dumps({"matvec": name, "rows": rows, "cols": cols, "bytes": nbytes, "us": ms * 1e3,
                              "GB/s": gbs, "frac_of_hbm": gbs / hbm}))
            del ws
    return 0


MATVEC_TYPES = (("Q4_0", 2), ("Q8_0", 8), ("Q4_K", 12), ("Q5_K", 13), ("Q6_K", 14))
MATVEC_SHAPES = ((2048, 2048), (256, 2048), (5632, 2048), (2048, 5632), (32000, 2048), (4096, 4096),
                 (14336, 4096), (128256, 4096))


def run_matvec_object(args):
    """The isolated fused dequant-matvec sweep (8 shapes x 5 formats, x ~
    N(0,1), weights N(0,0.02) quantized, one seed per shape) through
    gguf_cuda_matvec: GB/s of packed weight bytes with CUDA events over
    max(steps, 20) calls, rotating weight copies so that every call streams
    from HBM (> 2x the L2 together); beside it the reference's own
    gguf_matvec (src/gguf_model.c:693-771, OpenMP over all host threads) on
    the same blocks and x, and the relative L2 distance of the two outputs."""
    import torch
    import pk_b200
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    ref = oracle.Reference() if oracle.ref_available() else None
    hbm, peak_kind = peaks()
    st = torch.cuda.current_stream().cuda_stream
    entries = []
    for name, qt in MATVEC_TYPES:
        for rows, cols in MATVEC_SHAPES:
            rb = pk_b200.row_bytes(qt, cols)
            nbytes = rows * rb
            copies = max(1, min(8, (512 << 20) // nbytes))
            wb = pk_synth.random_matrix(qt, rows, cols, seed=rows + qt)
            xh = pk_synth.gaussian(1, cols)
            ws = [torch.from_numpy(wb).cuda() for _ in range(copies)]
            x = torch.from_numpy(xh).cuda()
            y = torch.empty(rows, device="cuda")
            wts = [pk_b200.make_weight(w.data_ptr(), qt, rows, cols) for w in ws]
            for i in range(3):
                pk_b200.matvec(wts[i % copies], x.data_ptr(), y.data_ptr(), st)
            reps = max(args.steps, 20)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for i in range(reps):
                pk_b200.matvec(wts[i % copies], x.data_ptr(), y.data_ptr(), st)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / reps
            gbs = nbytes / (us * 1e-6) / 1e9
            ent = {"type": name, "rows": rows, "cols": cols, "bytes": nbytes, "us": round(us, 2),
                   "GB/s": round(gbs, 1), "frac": round(gbs / hbm, 4)}
            if ref is not None:
                got = y.cpu().numpy()
                t0, n = time.perf_counter(), 0
                while n < 3 and (n == 0 or time.perf_counter() - t0 < 0.3):
                    want = ref.matvec(qt, wb, rows, cols, xh)
                    n += 1
                cpu_s = (time.perf_counter() - t0) / n
                ent["cpu_GB/s"] = round(nbytes / cpu_s / 1e9, 2)
                ent["vs_cpu"] = round(gbs / ent["cpu_GB/s"], 1)
                ent["rel_l2_vs_reference"] = float(np.linalg.norm(got - want) / np.linalg.norm(want))
            entries.append(ent)
            del ws, wts
    fr = np.array([e["frac"] for e in entries])
    return {"metric": "fused dequant-matvec GB/s of packed weights (gguf_cuda_matvec)", "unit": "GB/s",
            "peak": hbm, "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs",
            "geomean_frac": float(np.exp(np.log(fr).mean())), "max_frac": float(fr.max()),
            "cpu": None if ref is None else {"kind": "reference", "function": "gguf_matvec",
                                             "cores": os.cpu_count(),
                                             "threads": int(os.environ.get("OMP_NUM_THREADS", "0") or 0)},
            "l2": "weight copies rotated so that consecutive calls read > 2x the 126 MB L2",
            "entries": entries}


def run_tp7b(args, world, rank, local, barrier, allmax):
    """Llama-2-7B shape, Q4_K_M mix, one sequence decoded tensor-parallel over
    the N GPUs of the run (N = 1: the single-GPU engine): a 32-id prompt,
    W warm-up steps, then K timed greedy steps (CUDA events around the
    device-resident loop, slowest rank), and the same steps through
    engine_forward with host logits (e2e). At N > 1, rank 0 first decodes
    the same prompt on one GPU; tokens_match_n1 says whether the N-GPU run
    produced the same greedy tokens."""
    import torch
    import pk_b200
    wl = WORKLOADS["llama2-7b"]
    path = ensure_model(wl["preset"], rank, barrier)
    note("7B model ready")
    P, W, K = wl["prompt"], args.warmup, args.steps
    ctx = P + W + K + 16
    prompt = prompt_ids(P, 32000, 0)

    def feed(e):
        lg = None
        for pos, t in enumerate(prompt):
            lg = e.forward(int(t), pos)
        return int(np.argmax(lg))

    ref_toks = None
    if world > 1 and rank == 0:
        e1 = pk_b200.Engine(path, ctx, device=local)
        first = feed(e1)
        wt, _ = e1.generate_greedy(first, P, W)
        t1, _ = e1.generate_greedy(int(wt[-1]), P + W, K)
        ref_toks = [first] + [int(t) for t in wt] + [int(t) for t in t1]
        e1.close()
    barrier()
    if world > 1:
        e = pk_b200.Engine(path, ctx, device=local, rank=rank, world=world)
        e.tp_connect(pk_b200.tp_exchange(e.tp_handle(), world))
    else:
        e = pk_b200.Engine(path, ctx, device=local)
    cfg = e.config
    first = feed(e)
    wt, _ = e.generate_greedy(first, P, W)
    barrier()
    torch.cuda.synchronize()
    toks, ms = e.generate_greedy(int(wt[-1]), P + W, K)
    torch.cuda.synchronize()
    barrier()
    mine = [first] + [int(t) for t in wt] + [int(t) for t in toks]
    # e2e: the same positions through engine_forward, host logits, host argmax
    feed(e)
    for i in range(W):
        e.forward(first if i == 0 else mine[i], P + i)
    L = pk_b200.lib()
    tok = mine[W]
    barrier()
    t0 = time.perf_counter()
    for i in range(K):
        p = L.engine_forward(e.h, tok, P + W + i)
        tok = int(np.argmax(np.ctypeslib.as_array(p, shape=(e.vocab_size,))))
    e2e_s = time.perf_counter() - t0
    barrier()
    launches = e.launches_per_step()
    e.close()
    ms_max, e2e_max = allmax([ms, e2e_s * 1000.0])
    if rank != 0:
        return None
    hbm, peak_kind = peaks()
    wbytes = pk_synth.weight_bytes_per_token(wl["preset"])
    kvb = kv_bytes_per_step(cfg, list(range(P + W, P + W + K)), kv_entry_bytes())
    step_s = ms_max / 1000.0 / K
    achieved = (wbytes + kvb) / step_s / 1e9
    return {"metric": "decode tok/s (B=1), Llama-2-7B arch Q4_K_M", "value": K / (ms_max / 1000.0),
            "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms_max / K,
            "config": {"workload": wl["name"], "model_file": os.path.basename(path), "prompt": P,
                       "positions": [P + W, P + W + K - 1],
                       "parallelism": f"tensor parallel over {world} GPUs" if world > 1 else "1 GPU"},
            "tokens_match_n1": (ref_toks == mine) if world > 1 else True,
            "e2e": {"value": K / (e2e_max / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": 12,
                    "d2h_bytes_per_step": 4 * cfg["vocab_size"] + 20,
                    "path": "engine_forward (host logits) + host argmax, every rank"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm * world, "unit": "GB/s",
                         "frac": achieved / (hbm * world), "algorithmic_bytes_per_step": wbytes + kvb,
                         "weight_bytes_per_step": wbytes,
                         "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs x {world} GPUs"},
            "gpu_launches_per_step": launches}


def run_cfg4(args):
    """Llama-3-8B shape, Q5_K/Q6_K/Q8_0 mix, one sequence at an 8192-token
    context: a seeded 2048-token prompt through engine_prefill (chunks of 64
    rows on the batched tensor-core step), then 512 greedy decode steps
    (engine_generate_greedy, the persistent decode kernel) at positions
    2048..2559; and 64 decode steps after position 8128, the first 8128
    positions written with seeded keys and values (engine_kv_write)."""
    import torch
    import pk_b200
    wl = WORKLOADS["llama3-8b"]
    path = ensure_model(wl["preset"], 0, lambda: None)
    note("8B model ready")
    P, D, LONG, LSTEPS = 2048, 512, 8128, 64
    e = pk_b200.Engine(path, 8192, device=0)
    cfg = e.config
    prompt = prompt_ids(P, cfg["vocab_size"], 0)
    e.prefill(prompt[:64], 0)  # builds the 64-row step's graph
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tok, _ = e.prefill(prompt, 0)
    prefill_s = time.perf_counter() - t0
    wt, _ = e.generate_greedy(tok, P, 4)
    toks, ms = e.generate_greedy(tok, P, D)
    kvd = cfg["dim"] // cfg["n_heads"] * cfg["n_kv_heads"]
    for layer in range(cfg["n_layers"]):
        k = pk_synth.gaussian(9000 + 2 * layer, LONG * kvd, std=0.5).reshape(LONG, kvd)
        v = pk_synth.gaussian(9001 + 2 * layer, LONG * kvd, std=0.5).reshape(LONG, kvd)
        e.kv_write(layer, 0, k, v)
    e.generate_greedy(int(toks[-1]), LONG, 4)
    ltoks, lms = e.generate_greedy(int(toks[-1]), LONG, LSTEPS)
    e.close()
    note("8B config done")
    hbm, peak_kind = peaks()
    wbytes = pk_synth.weight_bytes_per_token(wl["preset"])
    dim, hid, L, V = cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["vocab_size"]
    mparams = L * (2 * dim * dim + 2 * dim * kvd + 3 * dim * hid) + V * dim
    attn = 4 * cfg["n_heads"] * (dim // cfg["n_heads"]) * L * sum(range(1, P + 1))
    flops = 2.0 * mparams * P + attn
    step = ms / 1000.0 / D
    kv_d = kv_bytes_per_step(cfg, list(range(P, P + D)), kv_entry_bytes())
    step_l = lms / 1000.0 / LSTEPS
    kv_l = kv_bytes_per_step(cfg, list(range(LONG, LONG + LSTEPS)), kv_entry_bytes())
    return {"workload": "Llama-3-8B-arch Q5_K/Q6_K/Q8_0, one sequence, context 8192",
            "model_file": os.path.basename(path),
            "prefill": {"tokens": P, "seconds": prefill_s, "value": P / prefill_s, "unit": "tok/s",
                        "path": "engine_prefill: 32 chunks of 64 rows; Q5_K and Q6_K matrices on the tcgen05 matmul, "
                                "Q8_0 output on the CUDA-core tile kernel; host time around the synchronous call",
                        "roofline": {"bound": "tensor", "flops": flops, "achieved_tflops": flops / prefill_s / 1e12,
                                     "peak_tflops": 1655.5, "frac": flops / prefill_s / 1e12 / 1655.5,
                                     "peak_source": "measured MEASURED_PEAKS.json bf16_tflops (burst)"}},
            "decode": {"steps": D, "positions": [P, P + D - 1], "value": D / (ms / 1000.0), "unit": "tok/s",
                       "ms_per_step": step * 1e3,
                       "roofline": {"bound": "hbm", "achieved": (wbytes + kv_d) / step / 1e9, "peak": hbm,
                                    "frac": (wbytes + kv_d) / step / 1e9 / hbm, "weight_bytes_per_step": wbytes}},
            "decode_at_8k": {"steps": LSTEPS, "positions": [LONG, LONG + LSTEPS - 1],
                             "value": LSTEPS / (lms / 1000.0), "unit": "tok/s", "ms_per_step": step_l * 1e3,
                             "roofline": {"bound": "hbm", "achieved": (wbytes + kv_l) / step_l / 1e9, "peak": hbm,
                                          "frac": (wbytes + kv_l) / step_l / 1e9 / hbm,
                                          "kv_bytes_per_step": kv_l}},
            "peak_source": f"{peak_kind} MEASURED_PEAKS.json"}


def run_cfg3(args, world=1, rank=0, local=0, barrier=lambda: None, allmax=lambda v: v):
    """Llama-2-7B shape, Q4_K_M mix, 16 independent sequences after a
    1024-position context (written with seeded keys and values through
    engine_kv_write), 32 greedy steps of engine_forward_batch; at N > 1 the
    N ranks run the batched step tensor-parallel (every rank the same
    calls), timed on each rank's host around its synchronous steps, the
    slowest rank's time."""
    import pk_b200
    wl = WORKLOADS["llama2-7b"]
    path = ensure_model(wl["preset"], rank, barrier)
    B, C, K = 16, 1024, 32
    if world > 1:
        e = pk_b200.Engine(path, C + K + 16, device=local, rank=rank, world=world)
        e.tp_connect(pk_b200.tp_exchange(e.tp_handle(), world))
    else:
        e = pk_b200.Engine(path, C + K + 16, device=local)
    e.batch_open(B)
    cfg = e.config
    kvd = cfg["dim"] // cfg["n_heads"] * cfg["n_kv_heads"]
    for layer in range(cfg["n_layers"]):
        k = pk_synth.gaussian(7000 + 2 * layer, C * kvd, std=0.5).reshape(C, kvd)
        v = pk_synth.gaussian(7001 + 2 * layer, C * kvd, std=0.5).reshape(C, kvd)
        for sq in range(B):
            e.kv_write(layer, 0, k, v, seq=sq)
    toks = prompt_ids(B, cfg["vocab_size"], 1)
    seq = np.arange(B, dtype=np.int32)
    for i in range(args.warmup):
        toks, _ = e.forward_batch(toks, np.full(B, C + i), seq)
    barrier()
    t0 = time.perf_counter()
    for i in range(K):
        toks, _ = e.forward_batch(toks, np.full(B, C + args.warmup + i), seq)
    dt = time.perf_counter() - t0
    barrier()
    e.close()
    dt = allmax([dt])[0]
    if rank != 0:
        return None
    hbm, peak_kind = peaks()
    hbm_all = hbm * world
    wbytes = pk_synth.weight_bytes_per_token(wl["preset"])
    kvb = kv_bytes_per_step(cfg, list(range(C + args.warmup, C + args.warmup + K)), kv_entry_bytes()) * B
    step = dt / K
    return {"workload": "Llama-2-7B-arch Q4_K_M, 16 sequences after a 1024-position context", "n_gpus": world,
            "steps": K, "value": B * K / dt, "unit": "tok/s", "ms_per_step": step * 1e3,
            "parallelism": f"tensor parallel over {world} GPUs" if world > 1 else "1 GPU",
            "path": "engine_forward_batch (tcgen05 matmuls), one graph per step, host time around synchronous "
                    "steps" + ("; the ranks all-reduce the Wo and ffn_down partial sums over NVLink" if world > 1
                               else ""),
            "roofline": {"bound": "hbm", "achieved": (wbytes + kvb) / step / 1e9, "peak": hbm_all,
                         "frac": (wbytes + kvb) / step / 1e9 / hbm_all, "weight_bytes_per_step": wbytes,
                         "kv_bytes_per_step": kvb,
                         "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs" +
                                        (f" x {world} GPUs" if world > 1 else "")}}


def run_matmul_sweep(args):
    """The batched Q4_K matmul (gguf_cuda_matmul) alone: n activation
    vectors against one weight matrix, graph-replayed, inputs resident; one
    JSON line per (shape, n) with the time, the weight-stream GB/s and the
    tensor FLOP/s (2 * rows * cols * N, N = 2n rounded up to 16: the hi and
    lo fp16 halves of every vector)."""
    import torch
    import pk_b200
    torch.cuda.set_device(0)
    hbm, _ = peaks()
    shapes = [(2048, 2048), (5632, 2048), (2048, 5632), (4096, 4096), (11008, 4096), (32000, 4096)]
    ns = (1, 8, 16, 32, 64)
    only = None
    if args.only:  # e.g. "32000x4096:64"
        shp, n = args.only.split(":")
        only = (tuple(int(v) for v in shp.split("x")), int(n))
    for rows, cols in shapes:
        if only is not None and (rows, cols) != only[0]:
            continue
        wb = pk_synth.random_matrix(pk_b200.Q4_K, rows, cols, seed=rows + cols)
        nbytes = wb.size
        copies = max(1, min(8, (512 << 20) // nbytes))  # rotate > 2x L2 of weight copies
        ws = [torch.from_numpy(wb).cuda() for _ in range(copies)]
        wts = [pk_b200.make_weight(w.data_ptr(), pk_b200.Q4_K, rows, cols) for w in ws]
        for n in ns:
            if only is not None and n != only[1]:
                continue
            x = torch.from_numpy(np.stack([pk_synth.gaussian(7 + b, cols) for b in range(n)])).cuda()
            y = torch.empty(n, rows, device="cuda")
            st = torch.cuda.Stream()
            with torch.cuda.stream(st):
                for i in range(3):
                    assert pk_b200.matmul(wts[i % copies], x.data_ptr(), n, y.data_ptr(), st.cuda_stream) == 1
                st.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=st):
                    for i in range(copies):
                        pk_b200.matmul(wts[i], x.data_ptr(), n, y.data_ptr(), st.cuda_stream)
                reps = max(1, max(args.steps, 20) // copies)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                g.replay()
                st.synchronize()
                e0.record(st)
                for i in range(reps):
                    g.replay()
                e1.record(st)
                st.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
            N = (2 * n + 15) // 16 * 16
            print(json.dumps({"matmul": "Q4_K", "rows": rows, "cols": cols, "n": n, "bytes": nbytes, "us": us,
                              "GB/s": nbytes / (us * 1e-6) / 1e9, "frac_of_hbm": nbytes / (us * 1e-6) / 1e9 / hbm,
                              "tensor_TFLOP/s": 2.0 * rows * cols * N / (us * 1e-6) / 1e12,
                              "matmul_error": pk_b200.matmul_error()}))
            del g
        del ws
    return 0


def run_b64(path, args, cfg, device=0, barrier=lambda: None):
    """Batched decode of 64 independent sequences (engine_forward_batch):
    each sequence first decodes a seeded random context (512 tokens by
    default, --b64-context) into its KV cache, then W warm-up and K timed
    greedy steps of all 64 together.
    Every step carries its token ids to the device and the greedy tokens
    back (synchronous), so the wall time per step is end to end."""
    import pk_b200
    B, W, K, C = 64, args.warmup, args.b64_steps, args.b64_context
    e = pk_b200.Engine(path, C + W + K + 8, device=device)
    e.batch_open(B)
    rng = np.random.default_rng(MODEL_SEED + 64)
    ctx = rng.integers(0, e.vocab_size, size=(B, C))
    seq = np.arange(B, dtype=np.int32)
    t0 = time.perf_counter()
    nxt = None
    for p in range(C):
        nxt, _ = e.forward_batch(ctx[:, p], np.full(B, p), seq)
    fill_s = time.perf_counter() - t0
    pos = C
    for i in range(W):
        nxt, _ = e.forward_batch(nxt, np.full(B, pos), seq)
        pos += 1
    barrier()
    t0 = time.perf_counter()
    for i in range(K):
        nxt, _ = e.forward_batch(nxt, np.full(B, pos), seq)
        pos += 1
    dt = time.perf_counter() - t0
    barrier()
    e.close()
    wbytes = pk_synth.weight_bytes_per_token(WORKLOADS["tinyllama"]["preset"])
    kvb = kv_bytes_per_step(cfg, list(range(C + W, C + W + K)), kv_entry_bytes()) * B
    step_s = dt / K
    hbm, peak_kind = peaks()
    achieved = (wbytes + kvb) / step_s / 1e9
    return {"metric": "decode tok/s (B=64)", "value": B * K / dt, "unit": "tok/s", "steps": K, "warmup": W,
            "seconds": dt,
            "ms_per_step": step_s * 1e3,
            "config": {"workload": "TinyLlama-1.1B-arch Q4_K_M, 64 independent sequences, greedy decode",
                       "context_per_sequence": [C + W, C + W + K - 1],
                       "kv_cache": "f16" if kv_entry_bytes() == 2 else "f32",
                       "context_fill": f"{C} seeded random tokens per sequence decoded through "
                                       f"engine_forward_batch ({fill_s:.1f} s, untimed)"},
            "path": "engine_forward_batch: Q4_K and Q6_K matrices on the tcgen05 tensor-core matmul (the Q6_K "
                    "attn_v of even layers on the CUDA-core tile kernel beside the Q/K launch), one CUDA graph "
                    "per step; token ids in and greedy tokens out every step (h2d 768 B, d2h 260 B), timed on the "
                    "host around synchronous steps",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "algorithmic_bytes_per_step": wbytes + kvb, "weight_bytes_per_step": wbytes,
                         "kv_bytes_per_step": kvb,
                         "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs" if peak_kind == "measured"
                         else "fallback 6.65 TB/s"}}


def run_step_trace(args, positions=130):
    """Per-phase critical path of one B=1 decode step on the TinyLlama
    shape (under torchrun with N > 1: the Llama-2-7B shape tensor-parallel
    over the N GPUs, rank 0's trace), from the step trace
    (POCKET_CUDA_TRACE=1: every CTA's %globaltimer stamps after staging its
    input and after its work, per phase). Decodes `positions` greedy steps,
    then reports per phase kind, averaged over the inner layers: the phase's
    length on the critical path (last CTA end minus the previous phase's
    last CTA end), the median time from that previous end until a CTA has
    staged its input, and the median and maximum work time of the CTAs with
    work. A diagnostic, not a bench line: the tracing itself adds a barrier
    per phase."""
    os.environ["POCKET_CUDA_TRACE"] = "1"
    import pk_b200
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
        path = ensure_model(WORKLOADS["llama2-7b"]["preset"], rank, dist.barrier)
        e = pk_b200.Engine(path, positions + 8, device=local, rank=rank, world=world)
        e.tp_connect(pk_b200.tp_exchange(e.tp_handle(), world))
    else:
        path = ensure_model(WORKLOADS["tinyllama"]["preset"], 0, lambda: None)
        e = pk_b200.Engine(path, positions + 8, device=0)
    tok = 1
    for pos in range(positions):
        tok = int(np.argmax(e.forward(tok, pos)))
    a = e.trace(all_ctas=True)  # [cta][phase][after staging, after work], us from CTA 0's start
    e.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
        if rank != 0:
            return 0
    stg, end = a[:, :, 0], a[:, :, 1]
    kinds = (["qkv", "attention", "wo", "wo_allreduce", "gate_up", "down", "down_allreduce"] if world > 1
             else ["qkv", "attention", "wo", "gate_up", "down"])
    per = len(kinds)
    out = {k: [] for k in kinds}
    nl = (a.shape[1] - 1) // per
    for layer in range(1, nl - 1):
        for i, k in enumerate(kinds):
            ph = per * layer + i
            prev = end[:, ph - 1].max()
            work = end[:, ph] - stg[:, ph]
            busy = work > 0.3
            if not busy.any():
                busy = work >= work.max()
            out[k].append((end[:, ph].max() - prev, np.median(stg[busy, ph] - prev), np.median(work[busy]),
                           work.max()))
    res = {"metric": "decode step trace (B=1)", "unit": "us", "position": positions, "n_gpus": world,
           "workload": "Llama-2-7B-arch Q4_K_M, tensor parallel" if world > 1 else "TinyLlama-1.1B-arch Q4_K_M",
           "step_us": float(end[:, -1].max()), "phases": {}}
    for k, v in out.items():
        v = np.array(v)
        res["phases"][k] = {"critical_us": round(float(v[:, 0].mean()), 2),
                            "staged_after_prev_us": round(float(v[:, 1].mean()), 2),
                            "work_median_us": round(float(v[:, 2].mean()), 2),
                            "work_max_us": round(float(v[:, 3].mean()), 2)}
    lg = a.shape[1] - 1
    res["phases"]["logits"] = {"critical_us": round(float(end[:, lg].max() - end[:, lg - 1].max()), 2)}
    print(json.dumps(res))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="tinyllama",
                    choices=list(WORKLOADS) + ["matvec", "matmul", "b64", "trace"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", default=None, help="matvec workload: one TYPE:ROWSxCOLS case")
    ap.add_argument("--b64-steps", type=int, default=128, help="timed steps of the B=64 batched decode (0: skip)")
    ap.add_argument("--b64-context", type=int, default=512, help="tokens decoded into each sequence's KV cache first")
    ap.add_argument("--kv", default="f32", choices=["f32", "f16"],
                    help="KV cache entries (f16: the half cache option, POCKET_CUDA_KV)")
    ap.add_argument("--tp", action="store_true",
                    help="N > 1 on the TinyLlama shape: one sequence tensor-parallel instead of one per GPU")
    ap.add_argument("--no-matvec", action="store_true", help="skip the matvec sweep object of the default line")
    ap.add_argument("--no-tp7b", action="store_true", help="skip the Llama-2-7B tensor-parallel object")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the Llama-2-7B B=16 and Llama-3-8B prefill/decode objects")
    ap.add_argument("--configs", default="both", choices=["both", "llama2_7b_b16", "llama3_8b"],
                    help="which of those two objects to run")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    os.environ["POCKET_CUDA_KV"] = args.kv
    # the synthetic-model writer and the reference's CPU kernels (OpenMP) use
    # every host thread
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))

    if args.workload == "matvec":
        return run_matvec_sweep(args)
    if args.workload == "matmul":
        return run_matmul_sweep(args)
    if args.workload == "trace":
        return run_step_trace(args)
    if args.workload == "b64":
        import torch
        import pk_b200
        torch.cuda.set_device(0)
        path = ensure_model(WORKLOADS["tinyllama"]["preset"], 0, lambda: None)
        e = pk_b200.Engine(path, 64, device=0)
        cfg = e.config
        e.close()
        print(json.dumps(run_b64(path, args, cfg)))
        return 0
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference_arm(args, wl)

    import torch
    import torch.distributed as dist
    import pk_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def allmax(vals):
        t = torch.tensor(vals, dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t]

    note("model file")
    path = ensure_model(wl["preset"], rank, barrier)
    note("model ready")
    need = wl["prompt"] + args.warmup + args.steps + 1
    # N > 1: the 7B/8B shapes (or --tp) decode one sequence tensor-parallel
    # over the N GPUs (each rank holds its heads, hidden slice and vocabulary
    # rows; the decode kernels all-reduce over NVLink peer memory). The
    # TinyLlama shape fits one GPU many times over, so by default every GPU
    # decodes its own independent sequence (data parallel, no collective on
    # the data path; weak scaling).
    tp = world > 1 and (args.tp or args.workload != "tinyllama")
    if tp:
        e = pk_b200.Engine(path, max(need, 64), device=local, rank=rank, world=world)
        e.tp_connect(pk_b200.tp_exchange(e.tp_handle(), world))
    else:
        e = pk_b200.Engine(path, max(need, 64), device=local)
    cfg = e.config
    if need > e.seq_len:
        raise SystemExit(f"prompt + warmup + steps = {need} exceeds the context {e.seq_len}")
    # tensor parallel: every rank feeds the same sequence; data parallel: its own
    prompt = prompt_ids(wl["prompt"], e.vocab_size, 0 if tp or world == 1 else rank)

    def feed_prompt():
        logits = None
        for pos, t in enumerate(prompt):
            logits = e.forward(int(t), pos)
        return int(np.argmax(logits))

    with ClockSampler(local) as clocks:
        # value: device-resident greedy loop
        tok = feed_prompt()
        wtoks, _ = e.generate_greedy(tok, wl["prompt"], args.warmup)
        barrier()
        torch.cuda.synchronize()
        toks, ms = e.generate_greedy(int(wtoks[-1]), wl["prompt"] + args.warmup, args.steps)
        torch.cuda.synchronize()
        barrier()
        # e2e: the same steps through engine_forward with host buffers
        tok0 = feed_prompt()
        L = pk_b200.lib()
        pos0 = wl["prompt"] + args.warmup
        for i in range(args.warmup):  # replay the warm-up positions
            e.forward(tok0 if i == 0 else int(wtoks[i - 1]), wl["prompt"] + i)
        tok = int(wtoks[-1])
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(args.steps):
            p = L.engine_forward(e.h, tok, pos0 + i)
            tok = int(np.argmax(np.ctypeslib.as_array(p, shape=(e.vocab_size,))))
        e2e_s = time.perf_counter() - t0
        torch.cuda.synchronize()
        barrier()
    e2e_tokens_match = tok == int(toks[-1])

    t = torch.tensor([ms, e2e_s * 1000.0], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, e2e_ms_max = float(t[0]), float(t[1])

    hbm1, peak_kind = peaks()
    hbm = hbm1 * world  # the N GPUs' HBM together
    wbytes = pk_synth.weight_bytes_per_token(wl["preset"])
    positions = list(range(pos0, pos0 + args.steps))
    kvb = kv_bytes_per_step(cfg, positions, kv_entry_bytes())
    step_s = ms_max / 1000.0 / args.steps
    replicas = 1 if tp else world  # sequences decoded at once, each streaming all weights
    achieved = replicas * (wbytes + kvb) / step_s / 1e9
    launches_per_step = e.launches_per_step()
    if launches_per_step == 2:
        per = 7 if tp else 5
        kernel = (f"phase_kernel (one cooperative launch per step per GPU: {per * cfg['n_layers'] + 1} phases, "
                  f"tagged-word hand-offs, no grid barrier) + finish_kernel (1 thread)")
    else:
        kernel = f"phase_kernel x{launches_per_step - 1} (one per phase) + finish_kernel"

    b64 = None
    if not tp and args.b64_steps > 0 and args.workload == "tinyllama":
        b64 = run_b64(path, args, cfg, device=local, barrier=barrier)
        tb = torch.tensor([b64["seconds"]], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(tb, op=dist.ReduceOp.MAX)
        b64["value"] = world * 64 * args.b64_steps / float(tb[0])  # all GPUs, slowest rank's time
        b64["ms_per_step"] = float(tb[0]) / args.b64_steps * 1e3
        b64["n_gpus"] = world
        b64["roofline"]["achieved"] *= world * b64["seconds"] / float(tb[0])
        b64["roofline"]["peak"] = hbm
        b64["roofline"]["frac"] = b64["roofline"]["achieved"] / hbm

    note("b=1 and b64 done")
    matvec = None
    if rank == 0 and world == 1 and not args.no_matvec and args.workload == "tinyllama":
        matvec = run_matvec_object(args)
        note("matvec sweep done")
    cfg3 = cfg4 = None
    if not args.no_configs and args.workload == "tinyllama" and args.configs in ("both", "llama2_7b_b16"):
        cfg3 = run_cfg3(args, world, rank, local, barrier, allmax)  # all ranks: tensor parallel at N > 1
        note("7B B=16 done")
    if rank == 0 and world == 1 and not args.no_configs and args.workload == "tinyllama":
        if args.configs in ("both", "llama3_8b"):
            cfg4 = run_cfg4(args)
    tp7b = None
    if not args.no_tp7b and args.workload == "tinyllama":
        tp7b = run_tp7b(args, world, rank, local, barrier, allmax)
        note("tp7b done")

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = reference_decode(path, wl["prompt"], 64, 2, budget_s=15.0)

    if rank == 0:
        value = replicas * args.steps / (ms_max / 1000.0)
        line = {
            "metric": "decode tok/s (B=1)", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": value / PUBLISHED_TOKS,
            "dtype": "f32 (packed Q4_K/Q6_K weights)",
            "data": "synthetic random-init weights N(0,0.02), seeded prompt ids",
            "vs_baseline_note": VS_BASELINE_NOTE,
            "config": workload_config(wl, path, args, world, tp),
            "e2e": {"value": replicas * args.steps / (e2e_ms_max / 1000.0), "unit": "tok/s",
                    "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 4 * e.vocab_size + 20,
                    "path": "engine_forward (host logits) + host argmax",
                    "same_tokens_as_device_loop": bool(e2e_tokens_match)},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": NCU_TRAFFIC.get(wl["preset"]) if world == 1 else None,
                         "kernel": kernel,
                         "duration": "CUDA events around the graph replays of the timed steps, per step",
                         "algorithmic_bytes_per_step": wbytes + kvb,
                         "weight_bytes_per_step": wbytes,
                         "weight_stream_frac": replicas * wbytes / step_s / 1e9 / hbm,
                         "peak_source": (f"{peak_kind} MEASURED_PEAKS.json hbm_gbs" if peak_kind == "measured"
                                         else "fallback 6.65 TB/s") + (f" x {world} GPUs" if world > 1 else "")},
            "cpu_baseline": base,
            "b64": b64,
            "matvec": matvec,
            "tp7b": tp7b,
            "llama2_7b_b16": cfg3,
            "llama3_8b": cfg4,
            "clocks": clocks.summary(),
            "gpu_launches": launches_per_step * args.steps,
        }
        print(json.dumps(line))
    e.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
