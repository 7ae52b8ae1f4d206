"""ctypes binding of the reference's session API (include/pocket.h), as its
own Python package binds it (python/pocketllm/__init__.py:75-128): the
facade tests load either the reference's whole libpocketllm or its session
layer linked to this repository's engine, and call both the same way."""
import ctypes
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libpocketllm_ref.so")
FACADE_LIB = os.path.join(ROOT, "oracle", "_ref", "libpocketllm_facade.so")

# every pocket_* entry point the reference's Python package resolves at import
POCKET_SYMBOLS = (
    "pocket_version", "pocket_model_open", "pocket_model_close", "pocket_model_description",
    "pocket_model_context", "pocket_model_vocab_size", "pocket_model_is_chat", "pocket_model_seed",
    "pocket_model_set_chat_format", "pocket_model_chat_format", "pocket_model_set_system",
    "pocket_model_reset", "pocket_model_generate", "pocket_model_chat", "pocket_model_stats",
    "pocket_model_error", "pocket_rag_open", "pocket_rag_close", "pocket_rag_refresh", "pocket_rag_reload",
    "pocket_rag_set_auto_refresh", "pocket_rag_change", "pocket_rag_ask", "pocket_rag_last_answer",
    "pocket_rag_last_source", "pocket_rag_last_offer", "pocket_rag_last_found", "pocket_rag_reset",
    "pocket_rag_ask_model", "pocket_rag_last_prompt", "pocket_rag_search", "pocket_rag_hit_text",
    "pocket_rag_hit_source", "pocket_rag_hit_score", "pocket_rag_row_count", "pocket_rag_term_count",
    "pocket_rag_file_count", "pocket_rag_file_name", "pocket_rag_file_readable", "pocket_rag_file_rows",
    "pocket_rag_file_tables", "pocket_rag_warning_count", "pocket_rag_warning", "pocket_rag_error",
)


class GenOptions(ctypes.Structure):  # PocketGenOptions, include/pocket.h:46-51
    _fields_ = [("sampler", ctypes.c_char_p), ("temperature", ctypes.c_float),
                ("top_k", ctypes.c_int), ("max_tokens", ctypes.c_int)]


class Stats(ctypes.Structure):  # PocketStats, include/pocket.h:53-61
    _fields_ = [("prompt_tokens", ctypes.c_int), ("generated_tokens", ctypes.c_int),
                ("stopped_by_eos", ctypes.c_int), ("prompt_seconds", ctypes.c_double),
                ("generate_seconds", ctypes.c_double), ("position", ctypes.c_int),
                ("context", ctypes.c_int)]


TokenFn = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_void_p)


def load(path):
    lib = ctypes.CDLL(path)
    P, S, I = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int
    sig = {
        "pocket_version": (S, []),
        "pocket_model_open": (P, [S, S, I, S, ctypes.c_size_t]),
        "pocket_model_close": (None, [P]),
        "pocket_model_description": (S, [P]),
        "pocket_model_context": (I, [P]),
        "pocket_model_vocab_size": (I, [P]),
        "pocket_model_is_chat": (I, [P]),
        "pocket_model_seed": (None, [P, ctypes.c_ulong]),
        "pocket_model_set_chat_format": (I, [P, S]),
        "pocket_model_reset": (None, [P]),
        "pocket_model_generate": (S, [P, S, ctypes.POINTER(GenOptions), TokenFn, P]),
        "pocket_model_chat": (S, [P, S, ctypes.POINTER(GenOptions), TokenFn, P]),
        "pocket_model_stats": (None, [P, ctypes.POINTER(Stats)]),
        "pocket_model_error": (S, [P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


class Session:
    """One pocket_model_open() handle."""

    def __init__(self, lib, model_path, max_context=0):
        self.lib = lib
        err = ctypes.create_string_buffer(1024)
        self.h = lib.pocket_model_open(model_path.encode(), None, max_context, err, 1024)
        self.error = err.value.decode("utf-8", "replace")
        self.pieces = []

        def on_token(piece, user):
            self.pieces.append(piece)

        self._cb = TokenFn(on_token)

    def generate(self, prompt, max_tokens):
        opts = GenOptions(b"greedy", 0.0, 0, max_tokens)
        self.pieces = []
        return self.lib.pocket_model_generate(self.h, prompt.encode(), ctypes.byref(opts), self._cb, None)

    def chat(self, message, max_tokens):
        opts = GenOptions(b"greedy", 0.0, 0, max_tokens)
        self.pieces = []
        return self.lib.pocket_model_chat(self.h, message.encode(), ctypes.byref(opts), self._cb, None)

    def stats(self):
        st = Stats()
        self.lib.pocket_model_stats(self.h, ctypes.byref(st))
        return st

    def close(self):
        if self.h:
            self.lib.pocket_model_close(self.h)
            self.h = None
