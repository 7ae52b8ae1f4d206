"""bench.py's host-side pieces that need no GPU: the prompt ids the
reference arm draws without the writer library equal pk_synth's, and the
synthetic-model command writes the same bytes as the library call."""
import hashlib
import os
import sys

import numpy as np

import pk_synth
from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_prompt_ids_restatement_matches_the_writer_library():
    for seed, n, lo, hi in ((4242, 64, 3, 32000), (4243, 1000, 3, 128256), (5, 17, 0, 7)):
        assert np.array_equal(bench.uniform_ints(seed, n, lo, hi), pk_synth.uniform_ints(seed, n, lo, hi))


def test_synth_command_writes_the_library_file(tmp_path):
    a, b = str(tmp_path / "a.gguf"), str(tmp_path / "b.gguf")
    pk_synth.write_model(a, "tiny-legacy", seed=11)
    pk_synth.write_model_cli(b, "tiny-legacy", seed=11)
    h = lambda p: hashlib.sha256(open(p, "rb").read()).hexdigest()  # noqa: E731
    assert os.path.getsize(a) == os.path.getsize(b) and h(a) == h(b)
