"""ctypes bindings for the CPU oracle (oracle/lib/liboracle.so) and for the
reference built from its own sources (oracle/_ref/libref.so).

Test infrastructure only: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker. The product never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "lib", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref.so")

F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 8, 12, 13, 14
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K",
              Q5_K: "Q5_K", Q6_K: "Q6_K"}

_P = ctypes.c_void_p
_fp = ctypes.POINTER(ctypes.c_float)


def build():
    """Compile the oracle (and the reference, where its sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def row_bytes(qtype, cols):
    if qtype == F32:
        return cols * 4
    if qtype == F16:
        return cols * 2
    bw, bb = BLOCK[qtype]
    assert cols % bw == 0
    return cols // bw * bb


def _ptr(a):
    return a.ctypes.data_as(_P)


class Oracle:
    """The C restatement of the reference's decode path."""

    def __init__(self, path=ORACLE_SO):
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        self.lib = lib
        lib.orc_fp16_to_fp32.restype = ctypes.c_float
        lib.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        lib.orc_dequantize_blocks.restype = ctypes.c_int
        lib.orc_dequantize_blocks.argtypes = [ctypes.c_uint32, _P, ctypes.c_size_t, _P]
        lib.orc_dequantize_row.restype = ctypes.c_int
        lib.orc_dequantize_row.argtypes = [ctypes.c_uint32, _P, ctypes.c_uint64, _P]
        for fn in (lib.orc_matvec, lib.orc_matvec_reference):
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.c_uint32, _P, ctypes.c_uint64, ctypes.c_uint64, _P, _P]
        lib.orc_q4k_scale_min.restype = ctypes.c_int
        lib.orc_q4k_scale_min.argtypes = [_P, ctypes.c_uint, _P, _P]
        lib.orc_open.restype = _P
        lib.orc_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
        lib.orc_close.argtypes = [_P]
        lib.orc_forward.restype = _fp
        lib.orc_forward.argtypes = [_P, ctypes.c_int, ctypes.c_int]
        lib.orc_config.argtypes = [_P, _P, _P]
        lib.orc_kv_write.restype = ctypes.c_int
        lib.orc_kv_write.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, _P]
        lib.orc_set_kv_half.restype = ctypes.c_int
        lib.orc_set_kv_half.argtypes = [_P, ctypes.c_int]
        lib.orc_greedy.restype = ctypes.c_int
        lib.orc_greedy.argtypes = [_P, ctypes.c_int]
        lib.orc_rope_table.argtypes = [_P, ctypes.c_int, _P]

    def fp16_to_fp32_all(self):
        """All 65536 half patterns decoded as an F16 row (the values are
        stored by C, so signalling-NaN payloads survive; a Python float
        round trip would quiet them)."""
        h = np.arange(65536, dtype=np.uint16)
        out = np.empty(65536, dtype=np.float32)
        assert self.lib.orc_dequantize_row(F16, _ptr(h), 65536, _ptr(out)) == 1
        return out

    def dequantize_blocks(self, qtype, raw):
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        bw, bb = BLOCK[qtype]
        nb = raw.size // bb
        out = np.empty(nb * bw, dtype=np.float32)
        assert self.lib.orc_dequantize_blocks(qtype, _ptr(raw), nb, _ptr(out)) == 1
        return out

    def matvec(self, qtype, data, rows, cols, x, reference=False):
        data = np.ascontiguousarray(data, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(rows, dtype=np.float32)
        fn = self.lib.orc_matvec_reference if reference else self.lib.orc_matvec
        assert fn(qtype, _ptr(data), rows, cols, _ptr(x), _ptr(y)) == 1
        return y

    def scale_min(self, scales12, i):
        s = np.ascontiguousarray(scales12, dtype=np.uint8)
        sc = ctypes.c_uint8()
        mn = ctypes.c_uint8()
        ok = self.lib.orc_q4k_scale_min(_ptr(s), i, ctypes.byref(sc), ctypes.byref(mn))
        return ok, sc.value, mn.value

    def open(self, path, max_context=0):
        return OracleModel(self, path, max_context)


class OracleModel:
    def __init__(self, orc, path, max_context):
        self.orc = orc
        err = ctypes.create_string_buffer(256)
        self.h = orc.lib.orc_open(path.encode(), max_context, err, 256)
        if not self.h:
            raise RuntimeError("oracle open failed: " + err.value.decode())
        ints = np.zeros(8, dtype=np.int32)
        fl = np.zeros(3, dtype=np.float32)
        orc.lib.orc_config(self.h, _ptr(ints), _ptr(fl))
        (self.dim, self.hidden_dim, self.n_layers, self.n_heads, self.n_kv_heads,
         self.vocab_size, self.seq_len, self.rope_dim) = [int(v) for v in ints]
        self.rope_freq_base, self.rms_norm_eps, self.rope_scale = [float(v) for v in fl]
        self.kv_dim = self.dim // self.n_heads * self.n_kv_heads

    def forward(self, token, pos):
        p = self.orc.lib.orc_forward(self.h, token, pos)
        if not p:
            return None
        return np.ctypeslib.as_array(p, shape=(self.vocab_size,)).copy()

    def set_kv_half(self, on=True):
        """Round appended K/V entries to IEEE half (not a reference mode)."""
        return self.orc.lib.orc_set_kv_half(self.h, 1 if on else 0)

    def kv_write(self, layer, pos, k, v):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        return self.orc.lib.orc_kv_write(self.h, layer, pos, _ptr(k), _ptr(v))

    def greedy(self, logits):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        return self.orc.lib.orc_greedy(_ptr(logits), logits.size)

    def close(self):
        if self.h:
            self.orc.lib.orc_close(self.h)
            self.h = None

    def __del__(self):
        self.close()


class _GGUFWeight(ctypes.Structure):
    """GGUFWeight, include/gguf_model.h:36-45 of the reference."""
    _fields_ = [("name", ctypes.c_char_p), ("data", _P), ("type", ctypes.c_uint32),
                ("cols", ctypes.c_uint64), ("rows", ctypes.c_uint64),
                ("row_bytes", ctypes.c_uint64), ("byte_size", ctypes.c_uint64)]


class _LLMOptions(ctypes.Structure):
    """LLMOptions, include/engine.h:32-49 of the reference."""
    _fields_ = [("model_path", ctypes.c_char_p), ("tokenizer_path", ctypes.c_char_p),
                ("max_context", ctypes.c_int)]


class _Config(ctypes.Structure):
    """Config, include/transformer.h:58-80 of the reference."""
    _fields_ = [(n, ctypes.c_int) for n in ("dim", "hidden_dim", "n_layers", "n_heads",
                                             "n_kv_heads", "vocab_size", "seq_len", "rope_dim")] + \
               [(n, ctypes.c_float) for n in ("rope_freq_base", "rms_norm_eps", "rope_scale")]


def ref_available():
    return os.path.exists(REF_SO)


class Reference:
    """The reference's own engine and kernels, compiled from its sources."""

    def __init__(self, path=REF_SO):
        lib = ctypes.CDLL(path)
        self.lib = lib
        lib.gguf_fp16_to_fp32.restype = ctypes.c_float
        lib.gguf_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        lib.gguf_dequantize_block.restype = ctypes.c_int
        lib.gguf_dequantize_block.argtypes = [ctypes.c_uint32, _P, _P]
        for fn in (lib.gguf_matvec, lib.gguf_matvec_reference):
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.POINTER(_GGUFWeight), _P, _P]
        lib.engine_open.restype = _P
        lib.engine_open.argtypes = [ctypes.POINTER(_LLMOptions), ctypes.c_char_p, ctypes.c_size_t]
        lib.engine_close.argtypes = [_P]
        lib.engine_forward.restype = _fp
        lib.engine_forward.argtypes = [_P, ctypes.c_int, ctypes.c_int]
        lib.engine_config.restype = ctypes.POINTER(_Config)
        lib.engine_config.argtypes = [_P]
        lib.engine_kv_cache_bytes.restype = ctypes.c_size_t
        lib.engine_kv_cache_bytes.argtypes = [_P]
        lib.engine_description.restype = ctypes.c_char_p
        lib.engine_description.argtypes = [_P]
        lib.engine_file_context.restype = ctypes.c_int
        lib.engine_file_context.argtypes = [_P]
        lib.gguf_weight_dequantize_row.restype = ctypes.c_int
        lib.gguf_weight_dequantize_row.argtypes = [ctypes.POINTER(_GGUFWeight), ctypes.c_uint64, _P]
        lib.sampler_greedy.restype = ctypes.c_int
        lib.sampler_greedy.argtypes = [_P, ctypes.c_size_t]

    def fp16_to_fp32_all(self):
        """All 65536 half patterns through gguf_weight_dequantize_row on an
        F16 row (src/gguf_model.c:335-341 stores gguf_fp16_to_fp32 results
        directly, preserving NaN payloads)."""
        h = np.arange(65536, dtype=np.uint16)
        out = np.empty(65536, dtype=np.float32)
        w = _GGUFWeight(b"h", h.ctypes.data, F16, 65536, 1, 131072, 131072)
        assert self.lib.gguf_weight_dequantize_row(ctypes.byref(w), 0, _ptr(out)) == 1
        return out

    def dequantize_blocks(self, qtype, raw):
        raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
        bw, bb = BLOCK[qtype]
        nb = raw.size // bb
        out = np.empty(nb * bw, dtype=np.float32)
        for i in range(nb):
            blk = raw[i * bb:(i + 1) * bb]
            assert self.lib.gguf_dequantize_block(
                qtype, _ptr(blk), out[i * bw:].ctypes.data_as(_P)) == 1
        return out

    def matvec(self, qtype, data, rows, cols, x, reference=False):
        data = np.ascontiguousarray(data, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(rows, dtype=np.float32)
        rb = row_bytes(qtype, cols)
        w = _GGUFWeight(b"w", data.ctypes.data, qtype, cols, rows, rb, rb * rows)
        fn = self.lib.gguf_matvec_reference if reference else self.lib.gguf_matvec
        assert fn(ctypes.byref(w), _ptr(x), _ptr(y)) == 1
        return y

    def open(self, path, max_context=0):
        return ReferenceModel(self, path, max_context)


class ReferenceModel:
    def __init__(self, ref, path, max_context):
        self.ref = ref
        self._path = path.encode()
        opts = _LLMOptions(self._path, None, max_context)
        err = ctypes.create_string_buffer(512)
        self.h = ref.lib.engine_open(ctypes.byref(opts), err, 512)
        if not self.h:
            raise RuntimeError("reference engine_open failed: " + err.value.decode())
        c = ref.lib.engine_config(self.h).contents
        self.vocab_size = c.vocab_size
        self.seq_len = c.seq_len
        self.config = {n: getattr(c, n) for n, _ in _Config._fields_}

    def forward(self, token, pos):
        p = self.ref.lib.engine_forward(self.h, token, pos)
        if not p:
            return None
        return np.ctypeslib.as_array(p, shape=(self.vocab_size,)).copy()

    def forward_ptr(self, token, pos):
        return self.ref.lib.engine_forward(self.h, token, pos)

    def greedy_ptr(self, p):
        return self.ref.lib.sampler_greedy(ctypes.cast(p, _P), self.vocab_size)

    def description(self):
        return self.ref.lib.engine_description(self.h).decode()

    def kv_cache_bytes(self):
        return self.ref.lib.engine_kv_cache_bytes(self.h)

    def close(self):
        if self.h:
            self.ref.lib.engine_close(self.h)
            self.h = None

    def __del__(self):
        self.close()
