"""ctypes bindings for libpk_synth.so: seeded synthetic llama GGUF models and
the block quantizer (synth/gguf_synth.c).

Model presets carry the architectures the benchmark is quoted on:
TinyLlama-1.1B (Q4_K_M mix), Llama-2-7B (Q4_K_M mix) and Llama-3-8B
(Q5_K / Q6_K / Q8_0 mix). Weights are random-init N(0, 0.02).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SYNTH_SO = os.path.join(HERE, "lib", "libpk_synth.so")

F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 8, 12, 13, 14
_P = ctypes.c_void_p


class Spec(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("dim", "hidden_dim", "n_layers", "n_heads",
                                             "n_kv_heads", "vocab_size", "context_length")] + \
               [(n, ctypes.c_float) for n in ("rope_theta", "rms_eps", "weight_std")] + \
               [("seed", ctypes.c_uint64)] + \
               [(n, ctypes.c_uint32) for n in ("t_embd", "t_output", "t_q", "t_k", "t_v_even",
                                                "t_v_odd", "t_o", "t_gate", "t_up",
                                                "t_down_even", "t_down_odd")] + \
               [("tied_output", ctypes.c_int), ("space_piece", ctypes.c_int)]


def _q4km(**kw):
    """The Q4_K_M mix: Q4_K for q/k/o/gate/up, Q6_K for token_embd/output and
    for attn_v/ffn_down on even layers (Q4_K on odd layers)."""
    d = dict(t_embd=Q6_K, t_output=Q6_K, t_q=Q4_K, t_k=Q4_K, t_v_even=Q6_K, t_v_odd=Q4_K,
             t_o=Q4_K, t_gate=Q4_K, t_up=Q4_K, t_down_even=Q6_K, t_down_odd=Q4_K)
    d.update(kw)
    return d


PRESETS = {
    # TinyLlama-1.1B architecture.
    "tinyllama-1.1b-q4km": dict(dim=2048, hidden_dim=5632, n_layers=22, n_heads=32, n_kv_heads=4,
                                vocab_size=32000, context_length=2048, rope_theta=10000.0,
                                **_q4km()),
    # Llama-2-7B architecture.
    "llama2-7b-q4km": dict(dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, n_kv_heads=32,
                           vocab_size=32000, context_length=4096, rope_theta=10000.0, **_q4km()),
    # Llama-3-8B architecture: Q5_K attention and gate/up, Q6_K down, Q8_0 embd/output.
    "llama3-8b-q5k": dict(dim=4096, hidden_dim=14336, n_layers=32, n_heads=32, n_kv_heads=8,
                          vocab_size=128256, context_length=8192, rope_theta=500000.0,
                          t_embd=Q8_0, t_output=Q8_0, t_q=Q5_K, t_k=Q5_K, t_v_even=Q5_K,
                          t_v_odd=Q5_K, t_o=Q5_K, t_gate=Q5_K, t_up=Q5_K, t_down_even=Q6_K,
                          t_down_odd=Q6_K),
    # Small models for parity tests (same code paths, seconds on the CPU).
    "tiny-q4km": dict(dim=256, hidden_dim=768, n_layers=2, n_heads=8, n_kv_heads=2,
                      vocab_size=1024, context_length=512, rope_theta=10000.0, **_q4km()),
    "tiny-q5k": dict(dim=512, hidden_dim=1024, n_layers=2, n_heads=4, n_kv_heads=2,
                     vocab_size=1024, context_length=512, rope_theta=500000.0,
                     t_embd=Q8_0, t_output=Q8_0, t_q=Q5_K, t_k=Q5_K, t_v_even=Q5_K,
                     t_v_odd=Q5_K, t_o=Q5_K, t_gate=Q5_K, t_up=Q5_K, t_down_even=Q6_K,
                     t_down_odd=Q6_K),
    "tiny-legacy": dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, n_kv_heads=4,
                        vocab_size=512, context_length=256, rope_theta=10000.0,
                        t_embd=Q8_0, t_output=Q4_0, t_q=Q4_0, t_k=Q8_0, t_v_even=Q4_0,
                        t_v_odd=Q8_0, t_o=Q8_0, t_gate=Q4_0, t_up=Q8_0, t_down_even=Q4_0,
                        t_down_odd=Q8_0),
    # Tensor-parallel parity: head and hidden splits on whole Q4_K blocks
    # for 2 and 4 ranks (512 / 256 Wo columns, 8 hidden blocks), 3 layers.
    "tp-q4km": dict(dim=1024, hidden_dim=2048, n_layers=3, n_heads=8, n_kv_heads=2,
                    vocab_size=2048, context_length=512, rope_theta=10000.0, **_q4km()),
    # ... and for 8 ranks: 2 query heads of 128 (one Q4_K block of Wo columns)
    # per rank, 4 KV heads shared by pairs of ranks, 2 hidden blocks per rank.
    "tp8-q4km": dict(dim=2048, hidden_dim=4096, n_layers=2, n_heads=16, n_kv_heads=4,
                     vocab_size=4096, context_length=512, rope_theta=10000.0, **_q4km()),
    "tiny-float": dict(dim=128, hidden_dim=256, n_layers=2, n_heads=4, n_kv_heads=2,
                       vocab_size=300, context_length=128, rope_theta=10000.0,
                       t_embd=F16, t_output=F32, t_q=F32, t_k=F16, t_v_even=F32, t_v_odd=F16,
                       t_o=F16, t_gate=F32, t_up=F16, t_down_even=F32, t_down_odd=F16),
}


def build():
    os.makedirs(os.path.join(HERE, "lib"), exist_ok=True)
    subprocess.run(["gcc", "-std=c11", "-O2", "-fopenmp", "-fPIC", "-Wall", "-Wextra", "-shared",
                    os.path.join(HERE, "synth", "gguf_synth.c"), "-o", SYNTH_SO, "-lm"],
                   check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(SYNTH_SO):
            build()
        L = ctypes.CDLL(SYNTH_SO)
        L.pks_write_model.restype = ctypes.c_int
        L.pks_write_model.argtypes = [ctypes.c_char_p, ctypes.POINTER(Spec), ctypes.c_char_p,
                                      ctypes.c_size_t]
        L.pks_quantize.restype = ctypes.c_int
        L.pks_quantize.argtypes = [ctypes.c_uint32, _P, ctypes.c_uint64, _P]
        L.pks_type_bytes.restype = ctypes.c_uint64
        L.pks_type_bytes.argtypes = [ctypes.c_uint32, ctypes.c_uint64]
        L.pks_gaussian.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_size_t,
                                   ctypes.c_float, _P]
        L.pks_uniform_ints.argtypes = [ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int,
                                       ctypes.c_int, _P]
        _lib = L
    return _lib


def spec(preset, seed=1234, weight_std=0.02, rms_eps=1e-5, **overrides):
    d = dict(PRESETS[preset])
    d.update(overrides)
    s = Spec()
    for k, v in d.items():
        setattr(s, k, v)
    s.rms_eps = rms_eps
    s.weight_std = weight_std
    s.seed = seed
    return s


def write_model(path, preset, seed=1234, **overrides):
    s = spec(preset, seed=seed, **overrides)
    err = ctypes.create_string_buffer(256)
    if lib().pks_write_model(path.encode(), ctypes.byref(s), err, 256) != 1:
        raise RuntimeError("write_model failed: " + err.value.decode())
    return path


CLI = os.path.join(HERE, "lib", "pk_synth_cli")


def write_model_cli(path, preset, seed=1234, weight_std=0.02, rms_eps=1e-5, **overrides):
    """write_model through the pk_synth_cli command: the same file, written by
    a child process, so the caller never loads the writer library."""
    d = dict(PRESETS[preset])
    d.update(overrides)
    d.update(rms_eps=rms_eps, weight_std=weight_std, seed=seed)
    args = [CLI, path] + [f"{k}={v!r}" if isinstance(v, float) else f"{k}={int(v)}" for k, v in d.items()]
    r = subprocess.run(args, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("pk_synth_cli failed: " + r.stderr.strip())
    return path


def weight_bytes_per_token(preset, **overrides):
    """Algorithmic weight bytes read per decoded token: every projection,
    the norms (F32) and one embedding row."""
    d = dict(PRESETS[preset])
    d.update(overrides)
    L = lib()
    dim, hid, nl = d["dim"], d["hidden_dim"], d["n_layers"]
    kvd = dim // d["n_heads"] * d["n_kv_heads"]
    tb = lambda t, n: int(L.pks_type_bytes(t, n))
    total = tb(d["t_embd"], dim) + tb(d["t_output"], dim * d["vocab_size"]) + 4 * dim
    for l in range(nl):
        even = l % 2 == 0
        total += tb(d["t_q"], dim * dim) + tb(d["t_k"], dim * kvd)
        total += tb(d["t_v_even"] if even else d["t_v_odd"], dim * kvd)
        total += tb(d["t_o"], dim * dim) + tb(d["t_gate"], dim * hid) + tb(d["t_up"], dim * hid)
        total += tb(d["t_down_even"] if even else d["t_down_odd"], hid * dim)
        total += 2 * 4 * dim
    return total


def quantize(qtype, x):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    nbytes = int(lib().pks_type_bytes(qtype, x.size))
    out = np.empty(nbytes, dtype=np.uint8)
    assert lib().pks_quantize(qtype, x.ctypes.data, x.size, out.ctypes.data) == 1
    return out


def gaussian(seed, n, std=1.0, start=0):
    out = np.empty(n, dtype=np.float32)
    lib().pks_gaussian(seed, start, n, std, out.ctypes.data)
    return out


def uniform_ints(seed, n, lo, hi):
    out = np.empty(n, dtype=np.int32)
    lib().pks_uniform_ints(seed, n, lo, hi, out.ctypes.data)
    return out


def random_matrix(qtype, rows, cols, seed, std=0.02):
    """Packed weight bytes for a rows x cols matrix of N(0, std) weights."""
    return quantize(qtype, gaussian(seed, rows * cols, std))
