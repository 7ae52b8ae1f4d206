"""The reference's own session layer (include/pocket.h: pocket.c, its
sampler, tokenizer text code and RAG) linked to this repository's engine
instead of the reference's, run on the device: every call must return what
the reference's whole library returned for the same model and arguments
(tests/golden/pocket_session.json: greedy generation text, the pieces passed
to the token callback, the statistics, and two chat turns).

The session layer reaches the engine only through engine.h (engine_open,
engine_forward, engine_tokenizer, engine_config, engine_format,
engine_is_stop_token, engine_description, engine_close), so this is the
drop-in check of that boundary with the reference's unmodified caller.
"""
import hashlib
import json
import os

import pytest

import pk_synth
import pocket_ctypes as pc
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def facade():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    if not os.path.exists(pc.FACADE_LIB):
        pytest.skip("oracle/_ref/libpocketllm_facade.so not built (needs the reference sources)")
    return pc.load(pc.FACADE_LIB)


def cases():
    return json.load(open(os.path.join(GOLDEN, "pocket_session.json")))["cases"]


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["preset"])
def test_session_matches_reference_library(facade, tmp_path, case):
    path = str(tmp_path / f"{case['preset']}.gguf")
    pk_synth.write_model(path, case["preset"], seed=case["seed"], space_piece=1)
    assert hashlib.sha256(open(path, "rb").read()).hexdigest() == case["sha256"]
    s = pc.Session(facade, path, case["context"])
    assert s.h, s.error
    assert facade.pocket_model_context(s.h) == case["context"]
    assert facade.pocket_model_is_chat(s.h) == 1  # a GGUF model
    text = s.generate(case["prompt"], case["max_tokens"])
    assert text is not None, facade.pocket_model_error(s.h)
    g = case["generate"]
    st = s.stats()
    assert (st.prompt_tokens, st.generated_tokens, st.stopped_by_eos, st.position) == \
        (g["prompt_tokens"], g["generated_tokens"], g["stopped_by_eos"], g["position"])
    assert [p.hex() for p in s.pieces] == g["pieces"]
    assert text.hex() == g["text"]
    facade.pocket_model_reset(s.h)
    for msg, want in zip(case["messages"], case["chat"]):
        reply = s.chat(msg, case["chat_tokens"])
        assert reply is not None, facade.pocket_model_error(s.h)
        st = s.stats()
        assert (reply.hex(), st.generated_tokens, st.position) == \
            (want["text"], want["generated_tokens"], want["position"])
    s.close()


def test_session_open_errors_come_from_the_engine(facade, tmp_path):
    s = pc.Session(facade, str(tmp_path / "missing.gguf"))
    assert not s.h
    assert s.error.startswith("cannot load") and "Cannot open model file." in s.error
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF" + b"\0" * 60)
    s = pc.Session(facade, str(bad))
    assert not s.h and s.error.startswith("cannot load")
