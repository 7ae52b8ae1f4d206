import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "llm-inference-c_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def reference_root():
    """The reference checkout the oracle recipe built from (REF_ROOT in the
    environment, else the root oracle/Makefile recorded), or None."""
    env = os.environ.get("REF_ROOT")
    if env:
        return env
    rec = os.path.join(ROOT, "oracle", "_ref", "ref_root.txt")
    if os.path.exists(rec):
        root = open(rec).read().strip()
        return root if os.path.isdir(root) else None
    return None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size model cases")


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.ref_available():
        pytest.skip("reference library oracle/_ref/libref.so not built")
    return oracle.Reference()


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


_models = {}


@pytest.fixture(scope="session")
def synth_model(model_dir):
    """Path of a seeded synthetic GGUF model, written once per session."""
    import pk_synth

    def make(preset, seed=7, **kw):
        key = (preset, seed, tuple(sorted(kw.items())))
        if key not in _models:
            path = os.path.join(str(model_dir), f"{preset}-{seed}-{len(_models)}.gguf")
            pk_synth.write_model(path, preset, seed=seed, **kw)
            _models[key] = path
        return _models[key]

    return make
