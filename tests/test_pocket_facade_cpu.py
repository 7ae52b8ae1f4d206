"""The reference's session layer (include/pocket.h) built against this
repository's engine, without a GPU:
  * the library exports every pocket_* entry point the reference's Python
    package resolves at import, and needs nothing from the engine beyond
    engine.h (it links with --no-undefined against the engine library);
  * the reference's own Python package, unchanged, imports against it
    (POCKETLLM_LIB) and reports an engine failure as its PocketError;
  * the reference's whole library reproduces the session fixture that the
    device test compares against.
"""
import hashlib
import json
import os
import subprocess
import sys

import pytest

import pk_synth
import pocket_ctypes as pc
from conftest import GOLDEN, reference_root

_ROOT = reference_root()
REF_PY = os.path.join(_ROOT, "python") if _ROOT else ""


def need(path):
    if not os.path.exists(path):
        pytest.skip(f"{os.path.relpath(path, pc.ROOT)} not built (needs the reference sources)")


def test_facade_exports_every_wrapper_symbol():
    need(pc.FACADE_LIB)
    import ctypes
    lib = ctypes.CDLL(pc.FACADE_LIB)
    missing = [n for n in pc.POCKET_SYMBOLS if not hasattr(lib, n)]
    assert not missing, missing
    assert len(pc.POCKET_SYMBOLS) == 44
    lib.pocket_version.restype = ctypes.c_char_p
    assert lib.pocket_version()


def test_facade_open_without_device_reports_the_engine_error(tmp_path):
    need(pc.FACADE_LIB)
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    path = pk_synth.write_model(str(tmp_path / "m.gguf"), "tiny-q4km", seed=7, space_piece=1)
    s = pc.Session(pc.load(pc.FACADE_LIB), path, 64)
    assert not s.h
    assert s.error.startswith("cannot load") and "CUDA" in s.error, s.error


def test_reference_python_package_imports_against_the_facade(tmp_path):
    need(pc.FACADE_LIB)
    if not os.path.isdir(os.path.join(REF_PY, "pocketllm")):
        pytest.skip("the reference's Python package is not present")
    path = pk_synth.write_model(str(tmp_path / "m.gguf"), "tiny-q4km", seed=7, space_piece=1)
    code = (
        "import sys\n"
        f"sys.path.insert(0, {REF_PY!r})\n"
        "import pocketllm\n"
        "print('version', pocketllm.version())\n"
        "try:\n"
        f"    pocketllm.Model({path!r}, context=64)\n"
        "    print('opened')\n"
        "except pocketllm.PocketError as e:\n"
        "    print('error', str(e).splitlines()[0])\n")
    env = dict(os.environ, POCKETLLM_LIB=pc.FACADE_LIB, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert lines[0].startswith("version ")
    assert lines[1].startswith("error cannot load") and "CUDA" in lines[1], lines


def test_reference_library_reproduces_the_session_fixture(tmp_path):
    need(pc.REF_LIB)
    lib = pc.load(pc.REF_LIB)
    for case in json.load(open(os.path.join(GOLDEN, "pocket_session.json")))["cases"]:
        path = str(tmp_path / f"{case['preset']}.gguf")
        pk_synth.write_model(path, case["preset"], seed=case["seed"], space_piece=1)
        assert hashlib.sha256(open(path, "rb").read()).hexdigest() == case["sha256"]
        s = pc.Session(lib, path, case["context"])
        assert s.h, s.error
        text = s.generate(case["prompt"], case["max_tokens"])
        assert text.hex() == case["generate"]["text"]
        assert [p.hex() for p in s.pieces] == case["generate"]["pieces"]
        lib.pocket_model_reset(s.h)
        for msg, want in zip(case["messages"], case["chat"]):
            assert s.chat(msg, case["chat_tokens"]).hex() == want["text"]
        s.close()
