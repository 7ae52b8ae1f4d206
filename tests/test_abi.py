"""The C-ABI library: it loads, exports every function the public headers
declare, and rejects bad inputs on the host exactly like the reference's
engine_open (error values and messages, no crash, no device work).
CPU-only: nothing here launches a kernel.
"""
import ctypes
import os
import re

import pytest

import gguf_min
import pk_b200
from conftest import ROOT, reference_root


def declared_functions():
    names = set()
    for h in ("engine.h", "engine_ext.h", "gguf_cuda.h", "tokenizer.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b([a-z_0-9]+)\s*\(", src):
            name = m.group(1)
            if name not in ("if", "sizeof", "defined"):
                names.add(name)
    return names


def test_library_loads_and_exports_every_declared_symbol():
    L = pk_b200.lib()
    declared = declared_functions()
    assert declared == set(pk_b200.EXPORTS), declared ^ set(pk_b200.EXPORTS)
    for name in declared:
        assert hasattr(L, name), name


LAYOUT_PROBE = r"""
#include <stddef.h>
#include <stdio.h>
#include "engine.h"
#include HEADER_WITH_GGUFWEIGHT
#define P(T, f) printf("%s.%s %zu\n", #T, #f, offsetof(T, f))
int main(void) {
    printf("Config %zu\nLLMOptions %zu\nTokenizer %zu\nGGUFWeight %zu\n", sizeof(Config),
           sizeof(LLMOptions), sizeof(Tokenizer), sizeof(GGUFWeight));
    P(Config, rope_dim); P(Config, rope_scale); P(LLMOptions, max_context);
    P(Tokenizer, byte_pieces); P(Tokenizer, byte_ids); P(Tokenizer, special_ids);
    P(Tokenizer, scores_reconstructed); P(GGUFWeight, type); P(GGUFWeight, byte_size);
    return 0;
}
"""


def _layout(include_dir, weight_header, tmp_path, tag):
    import subprocess
    src = tmp_path / f"probe_{tag}.c"
    src.write_text(LAYOUT_PROBE.replace("HEADER_WITH_GGUFWEIGHT", f'"{weight_header}"'))
    exe = tmp_path / f"probe_{tag}"
    subprocess.run(["gcc", "-std=c11", "-I", include_dir, str(src), "-o", str(exe)], check=True)
    return subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout


def test_struct_layouts_match_reference(tmp_path):
    """Config, LLMOptions, Tokenizer and GGUFWeight have the reference's
    layout (include/transformer.h:58-80, engine.h:32-49, tokenizer.h:13-48,
    gguf_model.h:36-45), checked by compiling both header sets."""
    mine = _layout(os.path.join(ROOT, "include"), "gguf_cuda.h", tmp_path, "mine")
    assert "GGUFWeight 56" in mine and "Config 44" in mine
    root = reference_root()
    ref_inc = os.path.join(root, "include") if root else ""
    if not os.path.isdir(ref_inc):
        pytest.skip("reference headers not present")
    assert mine == _layout(ref_inc, "gguf_model.h", tmp_path, "ref")
    assert ctypes.sizeof(pk_b200.Config) == 44
    assert ctypes.sizeof(pk_b200.GGUFWeight) == 56
    assert ctypes.sizeof(pk_b200.Tokenizer) == int(mine.split("Tokenizer ")[1].split()[0])


def _open(path, max_context=0):
    L = pk_b200.lib()
    err = ctypes.create_string_buffer(256)
    opts = pk_b200.LLMOptions(path.encode() if path else None, None, max_context)
    h = L.engine_open(ctypes.byref(opts), err, 256)
    return h, err.value.decode()


def test_null_and_missing_inputs():
    L = pk_b200.lib()
    err = ctypes.create_string_buffer(64)
    assert not L.engine_open(None, err, 64)
    assert err.value == b"No model path given."
    h, msg = _open("/nonexistent/model.gguf")
    assert not h and msg == "Cannot open model file."
    h, msg = _open("/tmp/x.gguf", max_context=-1)
    assert not h and msg == "Context size must be positive."
    L.engine_close(None)
    assert L.engine_forward(None, 0, 0) is None or not L.engine_forward(None, 0, 0)
    assert L.engine_config(None) is None or not L.engine_config(None)
    assert L.engine_kv_cache_bytes(None) == 0
    assert L.engine_description(None) == b""
    assert L.engine_is_stop_token(None, 5) == 1
    assert L.engine_forward_greedy(None, 0, 0) == -2


CASES = {
    "bad_magic": (dict(magic=b"GGUX"), "Not a GGUF file"),
    "version1": (dict(version=1), "GGUF version 1 is not supported (use a v2/v3 file)."),
    "version4": (dict(version=4), "Unsupported GGUF version."),
}


@pytest.mark.parametrize("case", list(CASES))
def test_header_rejections(tmp_path, case):
    kw, msg = CASES[case]
    p = gguf_min.write(str(tmp_path / "m.gguf"), gguf_min.llama_meta(), gguf_min.llama_tensors(), **kw)
    h, got = _open(p)
    assert not h and got.startswith(msg)


META_CASES = {
    "not_llama": ({"general.architecture": (gguf_min.STR, "gpt2")}, "Only llama architecture is supported."),
    "missing_heads": ({"llama.attention.head_count": None}, "Required LLaMA metadata is missing."),
    "u32_as_i32": ({"llama.block_count": (gguf_min.I32, 1)}, "Invalid or unsupported GGUF metadata."),
    "zero_dim": ({"llama.embedding_length": (gguf_min.U32, 0)}, "Invalid or unsupported GGUF metadata."),
    "yarn": ({"llama.rope.scaling.type": (gguf_min.STR, "yarn")},
             "RoPE scaling type 'yarn' is not supported (only 'none' and 'linear')."),
    "kv_not_divisor": ({"llama.attention.head_count_kv": (gguf_min.U32, 3)}, "Invalid LLaMA model configuration."),
    "odd_rope": ({"llama.rope.dimension_count": (gguf_min.U32, 15)}, "Unsupported RoPE dimension."),
    "bad_eps": ({"llama.attention.layer_norm_rms_epsilon": (gguf_min.F32T, -1.0)},
                "Invalid or unsupported GGUF metadata."),
}


@pytest.mark.parametrize("case", list(META_CASES))
def test_metadata_rejections(tmp_path, case):
    change, msg = META_CASES[case]
    meta = gguf_min.llama_meta()
    for k, v in change.items():
        if v is None:
            meta.pop(k)
        else:
            meta[k] = v
    p = gguf_min.write(str(tmp_path / "m.gguf"), meta, gguf_min.llama_tensors())
    h, got = _open(p)
    assert not h and got == msg


def test_tensor_rejections(tmp_path):
    meta = gguf_min.llama_meta()
    p = gguf_min.write(str(tmp_path / "a.gguf"), meta, gguf_min.llama_tensors(skip=("blk.0.ffn_up.weight",)))
    assert _open(p) == (None, "Missing tensor: blk.0.ffn_up.weight")
    p = gguf_min.write(str(tmp_path / "b.gguf"), meta,
                       gguf_min.llama_tensors(reshape={"blk.0.attn_k.weight": (64, 64)}))
    assert _open(p) == (None, "Tensor blk.0.attn_k.weight has an unexpected shape.")
    t = gguf_min.llama_tensors()
    t.append(("rope_freqs.weight", [8], 0, b"\0" * 32))
    p = gguf_min.write(str(tmp_path / "c.gguf"), meta, t)
    h, msg = _open(p)
    assert not h and msg.startswith("Model uses RoPE frequency factors")
    t = gguf_min.llama_tensors()
    name, dims, _, raw = t[1]
    t[1] = (name, dims, 3, raw)  # Q4_1: a type the engine does not decode
    p = gguf_min.write(str(tmp_path / "d.gguf"), meta, t)
    assert _open(p)[1] == "Tensor blk.0.attn_norm.weight uses unsupported type Q4_1 (3)."
    # truncated data section
    p = gguf_min.write(str(tmp_path / "e.gguf"), meta, gguf_min.llama_tensors())
    data = open(p, "rb").read()
    open(p, "wb").write(data[:-4096])
    assert _open(p)[1] == "Tensor output.weight lies outside the file."


def test_bad_tokenizer_metadata(tmp_path):
    meta = gguf_min.llama_meta()
    meta["tokenizer.ggml.model"] = (gguf_min.STR, "gpt2")
    p = gguf_min.write(str(tmp_path / "t.gguf"), meta, gguf_min.llama_tensors())
    assert _open(p)[1] == "Only SentencePiece ('llama') GGUF tokenizers are supported."
    meta = gguf_min.llama_meta()
    meta["tokenizer.ggml.eos_token_id"] = (gguf_min.U32, 10**6)
    p = gguf_min.write(str(tmp_path / "u.gguf"), meta, gguf_min.llama_tensors())
    assert _open(p)[1] == "BOS/EOS token ID is outside the vocabulary."


def test_valid_file_without_a_device_fails_cleanly(tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    p = gguf_min.write(str(tmp_path / "ok.gguf"), gguf_min.llama_meta(), gguf_min.llama_tensors())
    h, msg = _open(p)
    assert not h and msg.startswith("CUDA")
