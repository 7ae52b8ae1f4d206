"""The batched dequant-matmul on the tensor cores (gguf_cuda_matmul, Q4_K and
Q5_K weights) against the oracle, through the C ABI. torch only provides
device buffers.

Every output column b is the matvec of the weights with x_b, so each column
is held to the matvec bar: within 1e-4 relative L2 of the oracle's
restatement of the reference's fast kernel, and per-row normalised error
|y - y64| / sum|W||x| below 1e-5. At the full 7B shapes the columns are
compared with the device matvec (gguf_cuda_matvec), itself pinned to the
oracle.
"""
import numpy as np
import pytest

import pk_b200
import pk_synth

pytestmark = pytest.mark.gpu

REL_L2 = 1e-4
NORM_ERR = 1e-5


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


def activations(n, cols, seed):
    x = np.stack([pk_synth.gaussian(seed + 31 * b, cols) for b in range(n)]).astype(np.float32)
    # magnitudes far apart, so that the per-vector scaling is exercised
    x[0] *= 1000.0
    if n > 1:
        x[1] *= 1e-6
    if n > 3:
        x[3] = 0.0
    if n > 4:
        x[4, ::7] = 0.0
    return x


def gpu_matmul(torch, wb, rows, cols, x, qtype=pk_b200.Q4_K):
    n = x.shape[0]
    w = dev(torch, wb)
    xd = dev(torch, x)
    y = torch.full((n, rows), float("nan"), dtype=torch.float32, device="cuda")
    wt = pk_b200.make_weight(w.data_ptr(), qtype, rows, cols)
    assert pk_b200.matmul(wt, xd.data_ptr(), n, y.data_ptr()) == 1
    torch.cuda.synchronize()
    assert pk_b200.matmul_error() == 0
    return y.cpu().numpy()


def normalised_error(orc, wb, rows, cols, x, y, qtype=pk_b200.Q4_K):
    rb = pk_b200.row_bytes(qtype, cols)
    worst = 0.0
    for r in np.linspace(0, rows - 1, 8).astype(int):
        w = np.empty(cols, dtype=np.float32)
        row = np.ascontiguousarray(wb[r * rb:(r + 1) * rb])
        assert orc.lib.orc_dequantize_row(qtype, row.ctypes.data, cols, w.ctypes.data) == 1
        exact = w.astype(np.float64) @ x.astype(np.float64)
        scale = np.abs(w.astype(np.float64)) @ np.abs(x.astype(np.float64))
        if scale > 0:
            worst = max(worst, abs(float(y[r]) - exact) / scale)
    return worst


# (rows, cols, n): one tile; ragged tiles; a tile over many CTAs; more
# tiles than SMs; odd n (N rounded up to 16); the full 64 vectors.
SHAPES = [(128, 256, 1), (1, 256, 2), (300, 768, 5), (130, 4096, 64), (1000, 2048, 16), (2048, 2048, 33),
          (4096, 4096, 8), (20000, 1024, 3), (640, 5632, 64)]


@pytest.mark.parametrize("qtype", [pk_b200.Q4_K, pk_b200.Q5_K])
@pytest.mark.parametrize("shape", SHAPES)
def test_matmul_columns_match_oracle(torch, orc, shape, qtype):
    rows, cols, n = shape
    wb = pk_synth.random_matrix(qtype, rows, cols, seed=rows + cols + n + qtype)
    x = activations(n, cols, seed=rows + n)
    y = gpu_matmul(torch, wb, rows, cols, x, qtype)
    assert np.isfinite(y).all()
    for b in range(n):
        want = orc.matvec(qtype, wb, rows, cols, x[b])
        if not np.any(x[b]):
            assert np.array_equal(y[b], np.zeros(rows, np.float32)), b
            continue
        assert rel_l2(y[b], want) < REL_L2, (b, rel_l2(y[b], want))
        if b in (0, n - 1):
            assert normalised_error(orc, wb, rows, cols, x[b], y[b], qtype) < NORM_ERR


def test_matmul_repeat_is_deterministic(torch):
    rows, cols, n = 2048, 4096, 24
    wb = pk_synth.random_matrix(pk_b200.Q4_K, rows, cols, seed=5)
    x = activations(n, cols, seed=9)
    a = gpu_matmul(torch, wb, rows, cols, x)
    b = gpu_matmul(torch, wb, rows, cols, x)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)])
def test_matmul_7b_shapes_match_matvec(torch, rows, cols):
    n = 64
    wb = pk_synth.random_matrix(pk_b200.Q4_K, rows, cols, seed=rows ^ cols)
    x = activations(n, cols, seed=cols)
    y = gpu_matmul(torch, wb, rows, cols, x)
    w = dev(torch, wb)
    wt = pk_b200.make_weight(w.data_ptr(), pk_b200.Q4_K, rows, cols)
    yv = torch.empty(rows, dtype=torch.float32, device="cuda")
    for b in (0, 1, 2, 5, 17, 63):
        xd = dev(torch, x[b])
        assert pk_b200.matvec(wt, xd.data_ptr(), yv.data_ptr()) == 1
        torch.cuda.synchronize()
        want = yv.cpu().numpy()
        assert rel_l2(y[b], want) < REL_L2, (b, rel_l2(y[b], want))


def test_matmul_refuses_bad_arguments(torch):
    rows, cols = 256, 512
    wb = pk_synth.random_matrix(pk_b200.Q4_K, rows, cols, seed=1)
    w = dev(torch, wb)
    x = torch.zeros(65 * cols, dtype=torch.float32, device="cuda")
    y = torch.zeros(65 * rows, dtype=torch.float32, device="cuda")
    wt = pk_b200.make_weight(w.data_ptr(), pk_b200.Q4_K, rows, cols)
    assert pk_b200.matmul(wt, x.data_ptr(), 0, y.data_ptr()) == 0
    assert pk_b200.matmul(wt, x.data_ptr(), 65, y.data_ptr()) == 0
    assert pk_b200.matmul(wt, 0, 4, y.data_ptr()) == 0
    other = pk_b200.make_weight(w.data_ptr(), pk_b200.Q6_K, rows, cols)
    assert pk_b200.matmul(other, x.data_ptr(), 4, y.data_ptr()) == 0
    odd = pk_b200.make_weight(w.data_ptr() + 8, pk_b200.Q4_K, rows - 1, cols)
    assert pk_b200.matmul(odd, x.data_ptr(), 4, y.data_ptr()) == 0  # rows not 16-byte aligned
