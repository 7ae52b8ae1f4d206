"""Device decoders and the fused dequant-matvec against the oracle, through
the C ABI (include/gguf_cuda.h). torch only provides device buffers.

Bars: decoders and the fp16 table bit-exact; matvec within 1e-4 relative L2
of the reference's fast kernels (the oracle restates them bit for bit), and
per-row normalised error |y - y64| / sum|W||x| below 1e-5 as the reference's
own examples/05_matrix_math/compare_matvec.py requires of its fast kernel.
"""
import os

import numpy as np
import pytest

import oracle
import pk_b200
import pk_synth
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TYPES = {"Q4_0": pk_b200.Q4_0, "Q8_0": pk_b200.Q8_0, "Q4_K": pk_b200.Q4_K, "Q5_K": pk_b200.Q5_K,
         "Q6_K": pk_b200.Q6_K}
REL_L2 = 1e-4
NORM_ERR = 1e-5


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def gpu_matvec(torch, qtype, w_bytes, rows, cols, x):
    w = dev(torch, w_bytes)
    xd = dev(torch, x.astype(np.float32))
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    wt = pk_b200.make_weight(w.data_ptr(), qtype, rows, cols)
    assert pk_b200.matvec(wt, xd.data_ptr(), y.data_ptr()) == 1
    torch.cuda.synchronize()
    return y.cpu().numpy()


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


def test_fp16_table_bit_exact(torch, orc):
    out = torch.empty(65536, dtype=torch.float32, device="cuda")
    assert pk_b200.fp16_table(out.data_ptr()) == 1
    torch.cuda.synchronize()
    assert np.array_equal(bits(out.cpu().numpy()), bits(orc.fp16_to_fp32_all()))


@pytest.mark.parametrize("name", list(TYPES))
def test_decoders_match_ggufpy_golden(torch, name):
    g = np.load(os.path.join(GOLDEN, f"blocks_{name}.npz"))
    raw = g["raw"].reshape(-1)
    bw, bb = pk_b200.BLOCK[TYPES[name]]
    nb = raw.size // bb
    w = dev(torch, raw)
    out = torch.empty(nb * bw, dtype=torch.float32, device="cuda")
    wt = pk_b200.make_weight(w.data_ptr(), TYPES[name], nb, bw)  # one block per row
    assert pk_b200.dequantize_rows(wt, 0, nb, out.data_ptr()) == 1
    torch.cuda.synchronize()
    assert np.array_equal(bits(out.cpu().numpy()), bits(g["ggufpy"]))


@pytest.mark.parametrize("qtype", list(TYPES.values()) + [pk_b200.F32, pk_b200.F16])
def test_dequantize_rows_match_oracle(torch, orc, qtype):
    rows, cols = 37, 1024
    rng = np.random.default_rng(qtype)
    if qtype in (pk_b200.F32, pk_b200.F16):
        wb = pk_synth.random_matrix(qtype, rows, cols, seed=3)
    else:
        bw, bb = pk_b200.BLOCK[qtype]
        wb = rng.integers(0, 256, size=rows * cols // bw * bb, dtype=np.uint8)  # any bits, inf/NaN scales included
    rb = pk_b200.row_bytes(qtype, cols)
    w = dev(torch, wb)
    out = torch.empty(10 * cols, dtype=torch.float32, device="cuda")
    wt = pk_b200.make_weight(w.data_ptr(), qtype, rows, cols)
    assert pk_b200.dequantize_rows(wt, 20, 10, out.data_ptr()) == 1
    torch.cuda.synchronize()
    want = np.concatenate([np.empty(0, np.float32)] + [
        _orc_row(orc, qtype, wb[r * rb:(r + 1) * rb], cols) for r in range(20, 30)])
    got = out.cpu().numpy()
    # Bit-exact, except that a NaN produced by arithmetic on a NaN/inf scale
    # has a different payload on the GPU (canonical NaN) than on x86.
    same = (bits(got) == bits(want)) | (np.isnan(got) & np.isnan(want))
    assert same.all()
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert pk_b200.dequantize_rows(wt, 30, 8, out.data_ptr()) == 0  # past the last row


def _orc_row(orc, qtype, row, cols):
    out = np.empty(cols, dtype=np.float32)
    r = np.ascontiguousarray(row)
    assert orc.lib.orc_dequantize_row(qtype, r.ctypes.data, cols, out.ctypes.data) == 1
    return out


@pytest.mark.parametrize("name", list(TYPES))
def test_matvec_matches_reference_golden(torch, name):
    g = np.load(os.path.join(GOLDEN, f"matvec_{name}.npz"))
    rows, cols = int(g["rows"]), int(g["cols"])
    y = gpu_matvec(torch, TYPES[name], g["w"], rows, cols, g["x"])
    assert rel_l2(y, g["y_fast"]) < REL_L2
    assert rel_l2(y, g["y_reference"]) < REL_L2


def normalised_error(orc, qtype, wb, rows, cols, x, y):
    rb = pk_b200.row_bytes(qtype, cols)
    worst = 0.0
    for r in np.linspace(0, rows - 1, 16).astype(int):
        w = _orc_row(orc, qtype, wb[r * rb:(r + 1) * rb], cols).astype(np.float64)
        exact = w @ x.astype(np.float64)
        scale = np.abs(w) @ np.abs(x.astype(np.float64))
        worst = max(worst, abs(float(y[r]) - exact) / max(scale, 1e-30))
    return worst


SHAPES_SMALL = [(1, 256), (2, 512), (37, 768), (256, 2048), (300, 4096), (64, 5632)]


@pytest.mark.parametrize("qtype", list(TYPES.values()) + [pk_b200.F32, pk_b200.F16])
@pytest.mark.parametrize("shape", SHAPES_SMALL)
def test_matvec_matches_oracle_small(torch, orc, qtype, shape):
    rows, cols = shape
    wb = pk_synth.random_matrix(qtype, rows, cols, seed=rows + cols + qtype)
    x = pk_synth.gaussian(cols + 17, cols)
    y = gpu_matvec(torch, qtype, wb, rows, cols, x)
    want = orc.matvec(qtype, wb, rows, cols, x)
    assert rel_l2(y, want) < REL_L2
    assert normalised_error(orc, qtype, wb, rows, cols, x, y) < NORM_ERR


def test_matvec_odd_block_count(torch, orc):
    """Q4_0 / Q8_0 rows with an odd number of 32-weight blocks."""
    for qtype in (pk_b200.Q4_0, pk_b200.Q8_0):
        rows, cols = 19, 32 * 7
        wb = pk_synth.random_matrix(qtype, rows, cols, seed=9)
        x = pk_synth.gaussian(4, cols)
        assert rel_l2(gpu_matvec(torch, qtype, wb, rows, cols, x), orc.matvec(qtype, wb, rows, cols, x)) < REL_L2


# Rows longer than a ring stage stream in column chunks of whole blocks.
LONG_ROWS = [(pk_b200.Q6_K, 48, 16384), (pk_b200.Q4_K, 33, 40960), (pk_b200.Q8_0, 40, 8192),
             (pk_b200.Q4_0, 17, 16384 + 32), (pk_b200.F32, 9, 4096 + 64), (pk_b200.F16, 9, 8192 + 128)]


@pytest.mark.parametrize("qtype,rows,cols", LONG_ROWS)
def test_matvec_long_rows_in_column_chunks(torch, orc, qtype, rows, cols):
    wb = pk_synth.random_matrix(qtype, rows, cols, seed=rows * 3 + qtype)
    x = pk_synth.gaussian(cols + 5, cols)
    y = gpu_matvec(torch, qtype, wb, rows, cols, x)
    want = orc.matvec(qtype, wb, rows, cols, x)
    assert rel_l2(y, want) < REL_L2
    assert normalised_error(orc, qtype, wb, rows, cols, x, y) < NORM_ERR


# The isolated sweep shapes (out x in) of the benchmark configuration.
SWEEP = [(2048, 2048), (256, 2048), (5632, 2048), (2048, 5632), (32000, 2048), (4096, 4096),
         (14336, 4096), (128256, 4096)]


@pytest.mark.slow
@pytest.mark.parametrize("qtype", list(TYPES.values()))
@pytest.mark.parametrize("shape", SWEEP)
def test_matvec_sweep_shapes(torch, orc, qtype, shape):
    rows, cols = shape
    wb = pk_synth.random_matrix(qtype, rows, cols, seed=rows * 7 + qtype)
    x = pk_synth.gaussian(rows + 1, cols)
    y = gpu_matvec(torch, qtype, wb, rows, cols, x)
    want = orc.matvec(qtype, wb, rows, cols, x)
    assert rel_l2(y, want) < REL_L2
    assert np.all(np.isfinite(y))


def test_matvec_rejects_bad_arguments(torch):
    w = torch.zeros(144 * 4, dtype=torch.uint8, device="cuda")
    x = torch.zeros(256, dtype=torch.float32, device="cuda")
    y = torch.zeros(4, dtype=torch.float32, device="cuda")
    ok = pk_b200.make_weight(w.data_ptr(), pk_b200.Q4_K, 4, 256)
    assert pk_b200.matvec(ok, x.data_ptr(), y.data_ptr()) == 1
    bad = pk_b200.make_weight(w.data_ptr(), pk_b200.Q4_K, 4, 256)
    bad.type = 3
    assert pk_b200.matvec(bad, x.data_ptr(), y.data_ptr()) == 0
    bad = pk_b200.make_weight(w.data_ptr(), pk_b200.Q4_K, 4, 256)
    bad.row_bytes = 100
    assert pk_b200.matvec(bad, x.data_ptr(), y.data_ptr()) == 0
    assert pk_b200.matvec(ok, None, y.data_ptr()) == 0
    assert pk_b200.matvec(ok, x.data_ptr(), None) == 0
    assert pk_b200.matvec(ok, x.data_ptr(), x.data_ptr()) == 0  # out aliases x
    torch.cuda.synchronize()
