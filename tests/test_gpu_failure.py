"""Failure detection on the device without a fault or a hang.

Every wait inside the decode-step kernel is bounded. The test hook
POCKET_CUDA_TEST_STALL=<phase>:<us> makes one phase poll for a tag that no
producer writes, so that wait runs out after <us> microseconds; the step must
then come back as an error value (engine_forward returns NULL, the message
names the timed-out wait, the handle stays failed), as the reference's
"errors are values" contract asks (documentation/ARCHITECTURE.md:89-92), and
the CUDA context must stay usable for a new handle. The matvec seam's error
queries read 0 after calls that completed.
"""
import os

import numpy as np
import pytest

import pk_b200
import pk_synth

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def test_timed_out_wait_is_an_error_value_and_the_device_stays_usable(torch, orc, synth_model):
    path = synth_model("tiny-q4km")
    os.environ["POCKET_CUDA_TEST_STALL"] = "7:2000"  # layer 1's Wo phase, 2 ms
    try:
        e = pk_b200.Engine(path, 64, device=0)
    finally:
        del os.environ["POCKET_CUDA_TEST_STALL"]
    assert e.forward(1, 0) is None
    msg = e.last_error()
    assert "timed out" in msg, msg
    assert e.forward(1, 1) is None  # the handle stays failed
    with pytest.raises(RuntimeError):
        e.generate_greedy(1, 2, 3)
    e.close()
    # a new handle on the same device decodes correctly
    e = pk_b200.Engine(path, 64, device=0)
    o = orc.open(path, 64)
    tok = 1
    for pos in range(6):
        a, b = e.forward(tok, pos), o.forward(tok, pos)
        assert a is not None, e.last_error()
        assert float(np.abs(a - b).max()) < LOGIT_TOL
        tok = o.greedy(b)
    o.close()
    e.close()


def test_matvec_error_query_reads_zero_after_completed_calls(torch):
    rows, cols = 300, 2048
    w = torch.from_numpy(pk_synth.random_matrix(pk_b200.Q4_K, rows, cols, seed=21)).cuda()
    wt = pk_b200.make_weight(w.data_ptr(), pk_b200.Q4_K, rows, cols)
    x = torch.from_numpy(pk_synth.gaussian(22, cols)).cuda()
    y = torch.empty(rows, device="cuda")
    for _ in range(3):
        assert pk_b200.matvec(wt, x.data_ptr(), y.data_ptr()) == 1
    assert pk_b200.matvec_error() == 0
    assert pk_b200.matvec_error() == 0  # read and cleared: still 0
    assert np.isfinite(y.cpu().numpy()).all()
