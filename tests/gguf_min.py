"""A minimal GGUF v3 writer for crafting valid and malformed test files.

Metadata values are (gguf_type, value) pairs; tensors are
(name, dims, ggml_type, raw bytes).
"""
import struct

U32, I32, F32T, STR, ARR = 4, 5, 6, 8, 9


def _s(b):
    b = b.encode() if isinstance(b, str) else b
    return struct.pack("<Q", len(b)) + b


def _value(t, v):
    if t == U32:
        return struct.pack("<I", v)
    if t == I32:
        return struct.pack("<i", v)
    if t == F32T:
        return struct.pack("<f", v)
    if t == STR:
        return _s(v)
    if t == ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    raise ValueError(t)


def write(path, meta, tensors, version=3, align=32, magic=b"GGUF"):
    out = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(meta)))
    for k, (t, v) in meta.items():
        out += _s(k) + struct.pack("<I", t) + _value(t, v)
    off = 0
    offsets = []
    for name, dims, gt, raw in tensors:
        offsets.append(off)
        out += _s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", gt, off)
        off += (len(raw) + align - 1) // align * align
    out += b"\0" * ((align - len(out) % align) % align)
    for (name, dims, gt, raw), o in zip(tensors, offsets):
        out += raw + b"\0" * ((align - len(raw) % align) % align)
    with open(path, "wb") as f:
        f.write(out)
    return path


def llama_meta(dim=64, hidden=128, layers=1, heads=4, kv=2, vocab=300, ctx=64, **extra):
    toks = ["<unk>", "<s>", "</s>"] + ["<0x%02X>" % b for b in range(256)]
    toks += ["▁w%d" % i for i in range(vocab - len(toks))]
    types = [2, 3, 3] + [6] * 256 + [1] * (vocab - 259)
    meta = {
        "general.architecture": (STR, "llama"),
        "llama.context_length": (U32, ctx),
        "llama.embedding_length": (U32, dim),
        "llama.block_count": (U32, layers),
        "llama.feed_forward_length": (U32, hidden),
        "llama.attention.head_count": (U32, heads),
        "llama.attention.head_count_kv": (U32, kv),
        "tokenizer.ggml.model": (STR, "llama"),
        "tokenizer.ggml.tokens": (ARR, (STR, toks)),
        "tokenizer.ggml.scores": (ARR, (F32T, [-float(i) for i in range(vocab)])),
        "tokenizer.ggml.token_type": (ARR, (I32, types)),
        "tokenizer.ggml.bos_token_id": (U32, 1),
        "tokenizer.ggml.eos_token_id": (U32, 2),
    }
    meta.update(extra)
    return meta


def llama_tensors(dim=64, hidden=128, layers=1, heads=4, kv=2, vocab=300, skip=(), reshape=None):
    """F32 tensors (zeros) for a llama model; `skip` names to omit,
    `reshape` {name: dims} to corrupt shapes."""
    kvd = dim // heads * kv
    specs = [("token_embd.weight", (dim, vocab))]
    for l in range(layers):
        p = f"blk.{l}."
        specs += [(p + "attn_norm.weight", (dim,)), (p + "attn_q.weight", (dim, dim)),
                  (p + "attn_k.weight", (dim, kvd)), (p + "attn_v.weight", (dim, kvd)),
                  (p + "attn_output.weight", (dim, dim)), (p + "ffn_norm.weight", (dim,)),
                  (p + "ffn_gate.weight", (dim, hidden)), (p + "ffn_up.weight", (dim, hidden)),
                  (p + "ffn_down.weight", (hidden, dim))]
    specs += [("output_norm.weight", (dim,)), ("output.weight", (dim, vocab))]
    out = []
    for name, dims in specs:
        if name in skip:
            continue
        if reshape and name in reshape:
            dims = reshape[name]
        n = 1
        for d in dims:
            n *= d
        out.append((name, list(dims), 0, b"\0" * (4 * n)))
    return out
