"""Regenerate tests/golden/pocket_session.json: what the reference's own
session layer (include/pocket.h over its own engine, the whole
libpocketllm that its Makefile's `lib` target builds) returns for seeded
synthetic models. The facade test runs the same calls through the
reference's session layer linked to this repository's engine and compares.

Run in a container that has the reference sources:
    make -C llm-inference-c_b200 && make -C oracle && python tests/golden/make_pocket_golden.py

Per case: the model preset and seed (pk_synth writes the file, with the
bare word-start piece in its vocabulary so that the reference's
SentencePiece encoder accepts any prompt; the sha256 is recorded so the
test can check the bytes), then
  generate : pocket_model_generate(prompt, greedy, max_tokens) -> text,
             the pieces passed to the token callback, and pocket_model_stats
  chat     : pocket_model_chat turns for `messages` (the model's default
             chat format): reply text, generated tokens, cache position
Texts are stored as hex of the returned bytes (pieces of a synthetic
vocabulary need not be UTF-8).
"""
import hashlib
import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "llm-inference-c_b200"))
sys.path.insert(0, os.path.dirname(HERE))

import pk_synth  # noqa: E402
import pocket_ctypes as pc  # noqa: E402

CASES = [
    {"preset": "tiny-q4km", "seed": 7, "context": 256, "prompt": "The capital of France is",
     "max_tokens": 48, "messages": ["Hello there.", "And again?"], "chat_tokens": 24},
    {"preset": "tiny-q5k", "seed": 7, "context": 256, "prompt": "Once upon a time",
     "max_tokens": 40, "messages": ["Tell me a story."], "chat_tokens": 32},
]


def run_case(lib, path, c):
    s = pc.Session(lib, path, c["context"])
    assert s.h, s.error
    out = {}
    text = s.generate(c["prompt"], c["max_tokens"])
    st = s.stats()
    out["generate"] = {"text": text.hex(), "pieces": [p.hex() for p in s.pieces],
                       "prompt_tokens": st.prompt_tokens, "generated_tokens": st.generated_tokens,
                       "stopped_by_eos": st.stopped_by_eos, "position": st.position}
    turns = []
    s.lib.pocket_model_reset(s.h)
    for msg in c["messages"]:
        reply = s.chat(msg, c["chat_tokens"])
        st = s.stats()
        turns.append({"text": reply.hex(), "generated_tokens": st.generated_tokens, "position": st.position})
    out["chat"] = turns
    s.close()
    return out


def main():
    lib = pc.load(pc.REF_LIB)
    cases = []
    with tempfile.TemporaryDirectory() as d:
        for c in CASES:
            path = os.path.join(d, f"{c['preset']}.gguf")
            pk_synth.write_model(path, c["preset"], seed=c["seed"], space_piece=1)
            sha = hashlib.sha256(open(path, "rb").read()).hexdigest()
            cases.append(dict(c, sha256=sha, **run_case(lib, path, c)))
    out = {"source": "reference libpocketllm (oracle/_ref/libpocketllm_ref.so)", "cases": cases}
    with open(os.path.join(HERE, "pocket_session.json"), "w") as f:
        json.dump(out, f, indent=1)
    for c in cases:
        print(c["preset"], "generate:", c["generate"]["generated_tokens"], "tokens; chat turns:",
              [t["generated_tokens"] for t in c["chat"]])


if __name__ == "__main__":
    main()
