"""gguf_cuda_matvec_noalloc (include/gguf_cuda.h) against gguf_cuda_matvec.

The no-allocation entry point computes the same tiles from the same integer
form of x, so its output must equal gguf_cuda_matvec's bit for bit. Each
case makes two calls in a row with different x, so the second call has to
overwrite what the first left in the shared scratch. Collected last, and
self-contained, so it passes alone and after every other test.
"""
import numpy as np
import pytest

import pk_b200
import pk_synth

pytestmark = pytest.mark.gpu

MAX_COLS = 40960  # GGUF_CUDA_NOALLOC_MAX_COLS

CASES = [
    (pk_b200.Q4_0, 300, 2048), (pk_b200.Q8_0, 300, 2048), (pk_b200.Q4_K, 300, 2048),
    (pk_b200.Q5_K, 300, 2048), (pk_b200.Q6_K, 300, 2048), (pk_b200.Q4_K, 2048, 5632),
    (pk_b200.Q6_K, 257, 4096), (pk_b200.Q4_0, 65, 96), (pk_b200.F32, 129, 576),
    (pk_b200.F16, 129, 576), (pk_b200.Q4_K, 64, MAX_COLS),
]


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("qtype,rows,cols", CASES)
def test_noalloc_matches_matvec_on_two_calls_in_a_row(torch, qtype, rows, cols):
    w = dev(torch, pk_synth.random_matrix(qtype, rows, cols, seed=7 * rows + cols + qtype))
    wt = pk_b200.make_weight(w.data_ptr(), qtype, rows, cols)
    xs = [dev(torch, pk_synth.gaussian(seed, cols).astype(np.float32)) for seed in (11, 12)]
    y_ref = [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in xs]
    y_na = [torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda") for _ in xs]
    for x, y in zip(xs, y_ref):
        assert pk_b200.matvec(wt, x.data_ptr(), y.data_ptr()) == 1
    for x, y in zip(xs, y_na):  # two calls in a row through the one scratch
        rc, msg = pk_b200.matvec_noalloc(wt, x.data_ptr(), y.data_ptr())
        assert rc == 1, msg
        assert msg == ""
    torch.cuda.synchronize()
    assert pk_b200.matvec_noalloc_error() == 0  # no wait gave up in either call
    for a, b in zip(y_ref, y_na):
        a, b = a.cpu().numpy(), b.cpu().numpy()
        assert np.isfinite(a).all()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # the two inputs really gave different outputs
    assert not np.array_equal(y_na[0].cpu().numpy(), y_na[1].cpu().numpy())


def test_noalloc_rejects_more_columns_than_the_scratch_holds(torch):
    cols = MAX_COLS + 256
    w = dev(torch, pk_synth.random_matrix(pk_b200.Q4_K, 1, cols, seed=3))
    wt = pk_b200.make_weight(w.data_ptr(), pk_b200.Q4_K, 1, cols)
    x = torch.zeros(cols, dtype=torch.float32, device="cuda")
    y = torch.zeros(1, dtype=torch.float32, device="cuda")
    rc, msg = pk_b200.matvec_noalloc(wt, x.data_ptr(), y.data_ptr())
    assert rc == 0
    assert "GGUF_CUDA_NOALLOC_MAX_COLS" in msg and str(cols) in msg
    torch.cuda.synchronize()


def test_noalloc_rejects_bad_arguments(torch):
    rows, cols = 8, 256
    w = dev(torch, pk_synth.random_matrix(pk_b200.Q4_K, rows, cols, seed=5))
    wt = pk_b200.make_weight(w.data_ptr(), pk_b200.Q4_K, rows, cols)
    x = torch.zeros(cols, dtype=torch.float32, device="cuda")
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    rc, msg = pk_b200.matvec_noalloc(wt, x.data_ptr(), x.data_ptr())  # out aliases x
    assert rc == 0 and "invalid arguments" in msg
    rb = wt.row_bytes
    bad = pk_b200.GGUFWeight(b"w", w.data_ptr(), 3, cols, rows, rb, rb * rows)  # type 3 (Q4_1): unsupported
    rc, msg = pk_b200.matvec_noalloc(bad, x.data_ptr(), y.data_ptr())
    assert rc == 0 and "invalid arguments" in msg
