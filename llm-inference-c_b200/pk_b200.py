"""ctypes binding of libpocketllm_b200.so (engine.h, engine_ext.h, gguf_cuda.h).

This is how Python callers (the tests, bench.py) reach the C ABI, in the
same style as the reference's ctypes package (python/pocketllm/__init__.py).
The library is required: there is no CPU fallback, and loading fails loudly
when the built .so is missing.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libpocketllm_b200.so")

F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 8, 12, 13, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144),
         Q5_K: (256, 176), Q6_K: (256, 210)}

_P = ctypes.c_void_p

# Every symbol the public headers declare (include/engine.h, engine_ext.h,
# gguf_cuda.h, tokenizer.h).
EXPORTS = [
    "engine_open", "engine_close", "engine_forward", "engine_config", "engine_file_context",
    "engine_format", "engine_tokenizer", "engine_kv_cache_bytes", "engine_description",
    "engine_is_stop_token", "engine_open_device", "engine_forward_greedy", "engine_last_error",
    "engine_weight_bytes", "engine_generate_greedy", "engine_trace", "engine_launches_per_step",
    "engine_tp_plan", "engine_open_tp", "engine_tp_handle", "engine_tp_connect",
    "engine_batch_open", "engine_forward_batch", "engine_kv_write", "engine_prefill",
    "gguf_cuda_matvec", "gguf_cuda_dequantize_rows", "gguf_cuda_fp16_table", "gguf_cuda_matvec_noalloc",
    "gguf_cuda_matvec_error", "gguf_cuda_matvec_noalloc_error",
    "gguf_cuda_matmul", "gguf_cuda_matmul_plan", "gguf_cuda_matmul_error",
    "tokenizer_free",
]


def row_bytes(qtype, cols):
    bw, bb = BLOCK[qtype]
    assert cols % bw == 0
    return cols // bw * bb


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("dim", "hidden_dim", "n_layers", "n_heads",
                                             "n_kv_heads", "vocab_size", "seq_len", "rope_dim")] + \
               [(n, ctypes.c_float) for n in ("rope_freq_base", "rms_norm_eps", "rope_scale")]


class LLMOptions(ctypes.Structure):
    _fields_ = [("model_path", ctypes.c_char_p), ("tokenizer_path", ctypes.c_char_p),
                ("max_context", ctypes.c_int)]


class TokenizerIndex(ctypes.Structure):
    _fields_ = [("text", ctypes.c_char_p), ("id", ctypes.c_int)]


class Tokenizer(ctypes.Structure):
    _fields_ = [("vocab", ctypes.POINTER(ctypes.c_char_p)), ("scores", ctypes.POINTER(ctypes.c_float)),
                ("sorted_vocab", ctypes.POINTER(TokenizerIndex)), ("vocab_size", ctypes.c_size_t),
                ("max_token_length", ctypes.c_size_t), ("byte_pieces", ctypes.c_ubyte * 512),
                ("bos_id", ctypes.c_int), ("eos_id", ctypes.c_int), ("byte_ids", ctypes.c_int * 256),
                ("special_ids", ctypes.POINTER(ctypes.c_int)), ("n_special", ctypes.c_size_t),
                ("scores_reconstructed", ctypes.c_int)]


class EngineTpPlan(ctypes.Structure):  # include/engine_ext.h
    _fields_ = [(n, ctypes.c_int) for n in ("q_head0", "q_heads", "kv_head0", "kv_heads", "hid0", "hid",
                                             "voc0", "voc", "own0", "own")]


class GGUFWeight(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", _P), ("type", ctypes.c_uint32),
                ("cols", ctypes.c_uint64), ("rows", ctypes.c_uint64),
                ("row_bytes", ctypes.c_uint64), ("byte_size", ctypes.c_uint64)]


_lib = None


def lib(path=LIB_PATH):
    """Load the engine library (RuntimeError if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: run `make -C {HERE}` (the CUDA path has no fallback)")
    L = ctypes.CDLL(path)
    L.engine_open.restype = _P
    L.engine_open.argtypes = [ctypes.POINTER(LLMOptions), ctypes.c_char_p, ctypes.c_size_t]
    L.engine_open_device.restype = _P
    L.engine_open_device.argtypes = [ctypes.POINTER(LLMOptions), ctypes.c_int, ctypes.c_char_p,
                                     ctypes.c_size_t]
    L.engine_close.argtypes = [_P]
    L.engine_forward.restype = ctypes.POINTER(ctypes.c_float)
    L.engine_forward.argtypes = [_P, ctypes.c_int, ctypes.c_int]
    L.engine_forward_greedy.restype = ctypes.c_int
    L.engine_forward_greedy.argtypes = [_P, ctypes.c_int, ctypes.c_int]
    L.engine_config.restype = ctypes.POINTER(Config)
    L.engine_config.argtypes = [_P]
    L.engine_file_context.restype = ctypes.c_int
    L.engine_file_context.argtypes = [_P]
    L.engine_format.restype = ctypes.c_int
    L.engine_format.argtypes = [_P]
    L.engine_tokenizer.restype = ctypes.POINTER(Tokenizer)
    L.engine_tokenizer.argtypes = [_P]
    L.engine_kv_cache_bytes.restype = ctypes.c_size_t
    L.engine_kv_cache_bytes.argtypes = [_P]
    L.engine_description.restype = ctypes.c_char_p
    L.engine_description.argtypes = [_P]
    L.engine_is_stop_token.restype = ctypes.c_int
    L.engine_is_stop_token.argtypes = [_P, ctypes.c_int]
    L.engine_last_error.restype = ctypes.c_char_p
    L.engine_last_error.argtypes = [_P]
    L.engine_weight_bytes.restype = ctypes.c_size_t
    L.engine_weight_bytes.argtypes = [_P]
    L.engine_generate_greedy.restype = ctypes.c_int
    L.engine_generate_greedy.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P,
                                         ctypes.POINTER(ctypes.c_float)]
    L.engine_trace.restype = ctypes.c_int
    L.engine_trace.argtypes = [_P, _P, ctypes.c_int]
    L.engine_launches_per_step.restype = ctypes.c_int
    L.engine_launches_per_step.argtypes = [_P]
    L.engine_tp_plan.restype = ctypes.c_int
    L.engine_tp_plan.argtypes = [ctypes.c_int] * 9 + [ctypes.POINTER(EngineTpPlan), ctypes.c_char_p, ctypes.c_size_t]
    L.engine_open_tp.restype = _P
    L.engine_open_tp.argtypes = [ctypes.POINTER(LLMOptions), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_char_p, ctypes.c_size_t]
    L.engine_tp_handle.restype = ctypes.c_int
    L.engine_tp_handle.argtypes = [_P, _P]
    L.engine_tp_connect.restype = ctypes.c_int
    L.engine_tp_connect.argtypes = [_P, _P, ctypes.c_char_p, ctypes.c_size_t]
    L.engine_batch_open.restype = ctypes.c_int
    L.engine_batch_open.argtypes = [_P, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
    L.engine_forward_batch.restype = ctypes.c_int
    L.engine_forward_batch.argtypes = [_P, _P, _P, _P, ctypes.c_int, _P, _P]
    L.engine_prefill.restype = ctypes.c_int
    L.engine_prefill.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_char_p, ctypes.c_size_t]
    L.engine_kv_write.restype = ctypes.c_int
    L.engine_kv_write.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P,
                                  ctypes.c_char_p, ctypes.c_size_t]
    L.gguf_cuda_matvec.restype = ctypes.c_int
    L.gguf_cuda_matvec.argtypes = [ctypes.POINTER(GGUFWeight), _P, _P, _P]
    L.gguf_cuda_dequantize_rows.restype = ctypes.c_int
    L.gguf_cuda_dequantize_rows.argtypes = [ctypes.POINTER(GGUFWeight), ctypes.c_uint64,
                                            ctypes.c_uint64, _P, _P]
    L.gguf_cuda_fp16_table.restype = ctypes.c_int
    L.gguf_cuda_fp16_table.argtypes = [_P, _P]
    L.gguf_cuda_matvec_noalloc.restype = ctypes.c_int
    L.gguf_cuda_matvec_noalloc.argtypes = [ctypes.POINTER(GGUFWeight), _P, _P, _P, ctypes.c_char_p,
                                           ctypes.c_size_t]
    L.gguf_cuda_matvec_error.restype = ctypes.c_int
    L.gguf_cuda_matvec_error.argtypes = []
    L.gguf_cuda_matvec_noalloc_error.restype = ctypes.c_int
    L.gguf_cuda_matvec_noalloc_error.argtypes = []
    L.gguf_cuda_matmul.restype = ctypes.c_int
    L.gguf_cuda_matmul.argtypes = [ctypes.POINTER(GGUFWeight), _P, ctypes.c_int, _P, _P]
    L.gguf_cuda_matmul_plan.restype = None
    L.gguf_cuda_matmul_plan.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                        ctypes.POINTER(ctypes.c_int)]
    L.gguf_cuda_matmul_error.restype = ctypes.c_int
    L.gguf_cuda_matmul_error.argtypes = []
    _lib = L
    return L


class Engine:
    """One engine_open() handle."""

    def __init__(self, path, max_context=0, device=None, tokenizer_path=None, rank=0, world=1):
        L = lib()
        self._path = path.encode()
        self._tok = tokenizer_path.encode() if tokenizer_path else None
        opts = LLMOptions(self._path, self._tok, max_context)
        err = ctypes.create_string_buffer(512)
        if world > 1:
            self.h = L.engine_open_tp(ctypes.byref(opts), 0 if device is None else device, rank, world, err, 512)
        elif device is None:
            self.h = L.engine_open(ctypes.byref(opts), err, 512)
        else:
            self.h = L.engine_open_device(ctypes.byref(opts), device, err, 512)
        if not self.h:
            raise RuntimeError("engine_open failed: " + err.value.decode())
        self.world = world
        c = L.engine_config(self.h).contents
        self.config = {n: getattr(c, n) for n, _ in Config._fields_}
        self.vocab_size = c.vocab_size
        self.seq_len = c.seq_len

    def tp_handle(self):
        """This rank's 64-byte exchange handle (tensor-parallel handles)."""
        out = ctypes.create_string_buffer(64)
        if lib().engine_tp_handle(self.h, out) != 1:
            raise RuntimeError("engine_tp_handle failed: " + self.last_error())
        return out.raw

    def tp_connect(self, handles):
        """Connect with the ranks' handles (bytes of world * 64, rank order)."""
        err = ctypes.create_string_buffer(512)
        buf = ctypes.create_string_buffer(bytes(handles), len(handles))
        if lib().engine_tp_connect(self.h, buf, err, 512) != 1:
            raise RuntimeError("engine_tp_connect failed: " + err.value.decode())

    def forward(self, token, pos):
        """Logits as a fresh numpy array, or None when engine_forward returns NULL."""
        p = lib().engine_forward(self.h, token, pos)
        if not p:
            return None
        return np.ctypeslib.as_array(p, shape=(self.vocab_size,)).copy()

    def forward_raw(self, token, pos):
        return lib().engine_forward(self.h, token, pos)

    def forward_greedy(self, token, pos):
        return lib().engine_forward_greedy(self.h, token, pos)

    def batch_open(self, max_seqs):
        """engine_batch_open: batched state for max_seqs sequences."""
        err = ctypes.create_string_buffer(512)
        if lib().engine_batch_open(self.h, max_seqs, err, 512) != 1:
            raise RuntimeError("engine_batch_open failed: " + err.value.decode())

    def forward_batch(self, tokens, pos, seq_ids, logits=False):
        """engine_forward_batch: (greedy tokens, n x vocab logits or None);
        None when the call returns 0."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(pos, dtype=np.int32)
        q = np.ascontiguousarray(seq_ids, dtype=np.int32)
        n = t.size
        nxt = np.zeros(max(n, 1), dtype=np.int32)
        lg = np.zeros((n, self.vocab_size), dtype=np.float32) if logits else None
        ok = lib().engine_forward_batch(self.h, t.ctypes.data, p.ctypes.data, q.ctypes.data, n, nxt.ctypes.data,
                                        lg.ctypes.data if logits else None)
        if ok != 1:
            return None
        return nxt[:n], lg

    def prefill(self, tokens, pos0=0, logits=False):
        """engine_prefill: (greedy token of the last position, its logits or
        None); RuntimeError when the call returns -2."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        lg = np.zeros(self.vocab_size, dtype=np.float32) if logits else None
        err = ctypes.create_string_buffer(256)
        r = lib().engine_prefill(self.h, t.ctypes.data, t.size, pos0, lg.ctypes.data if logits else None, err, 256)
        if r == -2:
            raise RuntimeError("engine_prefill failed: " + err.value.decode())
        return r, lg

    def kv_write(self, layer, pos0, k, v, seq=-1):
        """engine_kv_write: rows pos0 .. of layer `layer` (k, v: npos x kv_dim
        floats, every KV head); seq -1 is engine_forward's cache."""
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        npos = k.shape[0] if k.ndim > 1 else 1
        err = ctypes.create_string_buffer(256)
        if lib().engine_kv_write(self.h, seq, layer, pos0, npos, k.ctypes.data, v.ctypes.data, err, 256) != 1:
            raise RuntimeError("engine_kv_write failed: " + err.value.decode())

    def generate_greedy(self, token, pos, n):
        """n device-side greedy steps: (tokens, device milliseconds)."""
        out = np.zeros(max(n, 1), dtype=np.int32)
        ms = ctypes.c_float(0.0)
        if lib().engine_generate_greedy(self.h, token, pos, n, out.ctypes.data, ctypes.byref(ms)) != 1:
            raise RuntimeError("engine_generate_greedy failed: " + self.last_error())
        return out[:n], ms.value

    def trace(self, all_ctas=False):
        """Per-phase device times (us) of the last step, or None when tracing
        is off. CTA 0's rows (stage x, work, 0); with all_ctas, an array
        [cta][phase][2] of (after staging, after work) in us from CTA 0's
        start instead. A tensor-parallel step has seven phases per layer
        (QKV, attention, Wo, its all-reduce, gate/up, down, its all-reduce),
        one GPU five."""
        nph = (7 if self.world > 1 else 5) * self.config["n_layers"] + 1
        out = np.zeros(3 * nph + 1 + 2 * 1024 * nph, dtype=np.uint64)
        n = lib().engine_trace(self.h, out.ctypes.data, out.size)
        if n <= 1:
            return None
        head = out[:3 * nph + 1].astype(np.float64)
        if all_ctas:
            rest = out[3 * nph + 1:n].astype(np.float64)
            return ((rest - head[0]) / 1000.0).reshape(-1, nph, 2)
        d = np.diff(head) / 1000.0
        return d[: (len(d) // 3) * 3].reshape(-1, 3)

    def description(self):
        return lib().engine_description(self.h).decode()

    def kv_cache_bytes(self):
        return lib().engine_kv_cache_bytes(self.h)

    def weight_bytes(self):
        return lib().engine_weight_bytes(self.h)

    def launches_per_step(self):
        return lib().engine_launches_per_step(self.h)

    def file_context(self):
        return lib().engine_file_context(self.h)

    def format(self):
        return lib().engine_format(self.h)

    def tokenizer(self):
        return lib().engine_tokenizer(self.h).contents

    def is_stop(self, token):
        return lib().engine_is_stop_token(self.h, token)

    def last_error(self):
        return lib().engine_last_error(self.h).decode()

    def close(self):
        if self.h:
            lib().engine_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_plan(dim, hidden_dim, n_heads, n_kv_heads, vocab_size, wo_block, down_block, rank, world):
    """engine_tp_plan as a dict; ValueError with the library's message when the split is impossible."""
    out = EngineTpPlan()
    err = ctypes.create_string_buffer(256)
    if lib().engine_tp_plan(dim, hidden_dim, n_heads, n_kv_heads, vocab_size, wo_block, down_block, rank, world,
                            ctypes.byref(out), err, 256) != 1:
        raise ValueError(err.value.decode())
    return {n: getattr(out, n) for n, _ in EngineTpPlan._fields_}


def tp_exchange(handle, world):
    """All-gather the ranks' 64-byte exchange handles in rank order over the
    default torch.distributed group (any backend)."""
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, bytes(handle))
    if any(o is None or len(o) != 64 for o in out):
        raise RuntimeError("tensor-parallel handle exchange failed")
    return b"".join(out)


def make_weight(dev_ptr, qtype, rows, cols):
    rb = row_bytes(qtype, cols)
    return GGUFWeight(b"w", dev_ptr, qtype, cols, rows, rb, rb * rows)


def matvec(weight, x_ptr, y_ptr, stream=0):
    return lib().gguf_cuda_matvec(ctypes.byref(weight), x_ptr, y_ptr, stream)


def matvec_noalloc(weight, x_ptr, y_ptr, stream=0):
    """gguf_cuda_matvec_noalloc: returns (status, message)."""
    err = ctypes.create_string_buffer(256)
    rc = lib().gguf_cuda_matvec_noalloc(ctypes.byref(weight), x_ptr, y_ptr, stream, err, 256)
    return rc, err.value.decode()


def matvec_error():
    """gguf_cuda_matvec_error: 1 if a matvec gave up on a wait since the last read, else 0 (-1: unreadable)."""
    return lib().gguf_cuda_matvec_error()


def matvec_noalloc_error():
    """gguf_cuda_matvec_noalloc_error: the same for the no-allocation entry point."""
    return lib().gguf_cuda_matvec_noalloc_error()


def matmul(weight, x_ptr, n, y_ptr, stream=0):
    """gguf_cuda_matmul: y (n x rows) = x (n x cols) times W transposed."""
    return lib().gguf_cuda_matmul(ctypes.byref(weight), x_ptr, n, y_ptr, stream)


def matmul_plan(rows, nsb, sms):
    """gguf_cuda_matmul_plan: (CTAs, most CTAs sharing one 128-row tile)."""
    g, mp = ctypes.c_int(), ctypes.c_int()
    lib().gguf_cuda_matmul_plan(rows, nsb, sms, ctypes.byref(g), ctypes.byref(mp))
    return g.value, mp.value


def matmul_error():
    return lib().gguf_cuda_matmul_error()


def dequantize_rows(weight, row0, nrows, out_ptr, stream=0):
    return lib().gguf_cuda_dequantize_rows(ctypes.byref(weight), row0, nrows, out_ptr, stream)


def fp16_table(out_ptr, stream=0):
    return lib().gguf_cuda_fp16_table(out_ptr, stream)
