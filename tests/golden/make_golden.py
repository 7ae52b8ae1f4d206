"""Regenerate the golden fixtures in tests/golden/.

Run in a container that has the reference sources and gguf-py:
    make -C oracle && python tests/golden/make_golden.py

Fixtures:
  blocks_<TYPE>.npz   random blocks (seed 2026, fp16 scale exponents kept
                      finite as the reference's own
                      examples/03_quantization/compare_quant_random.py does)
                      and their FP32 decode by gguf-py 0.19
                      (gguf.quants.dequantize), the third-party decoder the
                      reference is pinned against.
  q4k_scale_min.npz   the packed-scale example of the reference's
                      examples/03_quantization/gguf_q4k_demo.c decoded by the
                      reference's gguf_q4k_get_scale_min.
  matvec_<TYPE>.npz   packed weights + xorshift32 inputs (seeds 12345 / 67890
                      as examples/05_matrix_math/gguf_matvec_demo.c) and the
                      outputs of the reference's gguf_matvec (fast kernels)
                      and gguf_matvec_reference.
  forward_tiny.npz    logits of the reference engine (engine_open /
                      engine_forward) for the first positions of the seeded
                      synthetic "tiny-q4km" model, and 32 greedy tokens, plus
                      the sha256 of the model file so the test can check that
                      the generator reproduced the same bytes.
"""
import ctypes
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "llm-inference-c_b200"))
import oracle  # noqa: E402
import pk_synth  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
TYPES = {"Q4_0": (2, 18, [0]), "Q8_0": (8, 34, [0]), "Q4_K": (12, 144, [0, 2]),
         "Q5_K": (13, 176, [0, 2]), "Q6_K": (14, 210, [208])}


def xorshift_inputs(n, seed):
    """[-1, 1) values of gguf_matvec_demo.c's fill_input (xorshift32)."""
    s = seed
    out = np.empty(n, dtype=np.float32)
    for i in range(n):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        out[i] = np.float32(s / 4294967296.0 * 2.0 - 1.0)
    return out


def main():
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize

    ref = oracle.Reference()
    rng = np.random.default_rng(2026)
    for name, (tid, size, fp16_offsets) in TYPES.items():
        raw = rng.integers(0, 256, size=(256, size), dtype=np.uint8)
        for off in fp16_offsets:
            raw[:, off + 1] &= 0x7B
        deq = dequantize(raw, GGMLQuantizationType(tid)).reshape(-1).astype(np.float32)
        np.savez_compressed(os.path.join(OUT, f"blocks_{name}.npz"), raw=raw, ggufpy=deq)

    packed = np.array([0xC1, 0x82, 0x43, 0x04, 0x85, 0x46, 0xA7, 0xE8, 0xB9, 0x6A, 0xDB, 0xFC],
                      dtype=np.uint8)
    ref.lib.gguf_q4k_get_scale_min.restype = ctypes.c_int
    ref.lib.gguf_q4k_get_scale_min.argtypes = [ctypes.c_void_p, ctypes.c_uint, ctypes.c_void_p,
                                               ctypes.c_void_p]
    sm = []
    for i in range(8):
        sc, mn = ctypes.c_uint8(), ctypes.c_uint8()
        assert ref.lib.gguf_q4k_get_scale_min(packed.ctypes.data, i, ctypes.byref(sc),
                                              ctypes.byref(mn)) == 1
        sm.append((sc.value, mn.value))
    np.savez_compressed(os.path.join(OUT, "q4k_scale_min.npz"), packed=packed,
                        scale_min=np.array(sm, dtype=np.int32))

    shapes = {"Q4_0": (48, 512), "Q8_0": (48, 512), "Q4_K": (48, 512), "Q5_K": (48, 512),
              "Q6_K": (48, 512)}
    for name, (rows, cols) in shapes.items():
        tid = TYPES[name][0]
        w = pk_synth.random_matrix(tid, rows, cols, seed=1000 + tid)
        x = xorshift_inputs(cols, 12345 if tid % 2 else 67890)
        y_fast = ref.matvec(tid, w, rows, cols, x)
        y_ref = ref.matvec(tid, w, rows, cols, x, reference=True)
        np.savez_compressed(os.path.join(OUT, f"matvec_{name}.npz"), w=w, x=x, rows=rows, cols=cols,
                            y_fast=y_fast, y_reference=y_ref)

    path = "/tmp/golden_tiny_q4km.gguf"
    pk_synth.write_model(path, "tiny-q4km", seed=7)
    digest = hashlib.sha256(open(path, "rb").read()).hexdigest()
    m = ref.open(path, 64)
    tokens = pk_synth.uniform_ints(99, 8, 3, m.vocab_size)
    logits = np.stack([m.forward(int(t), p) for p, t in enumerate(tokens)])
    greedy = []
    tok = int(tokens[-1])
    last = logits[-1]
    for step in range(32):
        tok = int(np.argmax(last))
        greedy.append(tok)
        last = m.forward(tok, len(tokens) + step)
    np.savez_compressed(os.path.join(OUT, "forward_tiny.npz"), prompt=tokens, logits=logits,
                        greedy=np.array(greedy, dtype=np.int32), sha256=np.array(digest),
                        seed=7, max_context=64)
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
