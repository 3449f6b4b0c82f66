"""Kernel-level parity of the CUDA path against the CPU oracle (needs a B200).

* quantizer bytes are identical to the oracle's (src/quant.rs:39-104);
* embedding-row dequantisation is bit-exact (src/kernels.rs:95-121);
* the verify-path GEMV matches kernels::matmul (src/kernels.rs:53-92,123-203) within a float
  reassociation tolerance, for every format the 0.5B/3B configs use and M = 1 .. 33 rows.
"""

import os

import numpy as np
import pytest

import layerstream_b200 as ls
from oracle import oracle as O
import fixtures as F

pytestmark = pytest.mark.gpu

FORMATS = [(8, 64), (8, 32), (8, 16), (4, 32), (4, 16), (4, 64), (4, 128)]


def rand_rows(rows, cols, bits, group, seed, std=0.02):
    """Random stored rows made by the oracle quantizer (the reference's packed format)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * std).astype(np.float32)
    w[:, ::37] *= 8  # a few outliers per row, as real weights have
    rb = O.row_bytes(bits, group, cols)
    raw = np.zeros(rows * rb, np.uint8)
    for r in range(rows):
        raw[r * rb:(r + 1) * rb] = O.quantize_row(bits, group, w[r], True)[0]
    return raw


@pytest.mark.parametrize("bits,group", FORMATS)
def test_dequantised_rows_are_bit_exact(bits, group):
    rows, cols = 100, 896
    raw = rand_rows(rows, cols, bits, group, 1)
    rb = O.row_bytes(bits, group, cols)
    ids = [0, 1, 31, 32, 63, 99, 50, 7]
    got = ls.dequant_rows(bits, group, raw, rows, cols, ids)
    for i, r in enumerate(ids):
        want = O.dequant_row(bits, group, raw[r * rb:(r + 1) * rb], cols)
        assert np.array_equal(got[i].view(np.uint32), want.view(np.uint32)), (bits, group, r)


def tc_tol(want):
    """Tolerance of the tensor-core GEMV: weights (q * scale) and activations enter the MMA as f16
    (relative rounding <= 2^-11 each), accumulation is f32; the error of a K-term dot product is
    then a few 1e-4 of the output's scale."""
    return 2e-3 * np.sqrt(np.mean(want.astype(np.float64) ** 2)) + 2e-3 * np.abs(want)


@pytest.mark.parametrize("bits,group", FORMATS)
@pytest.mark.parametrize("M", [1, 2, 5, 9, 16, 33])
def test_gemv_matches_the_oracle_matmul(bits, group, M):
    rows, cols = 200, 896  # rows not a multiple of the 32-row tile
    raw = rand_rows(rows, cols, bits, group, 2 + M)
    x = np.random.default_rng(M).standard_normal((M, cols)).astype(np.float32)
    y, _ = ls.qgemv(bits, group, raw, rows, cols, x)
    want = O.matmul(bits, group, raw, rows, cols, x)
    err = np.abs(y - want)
    assert np.all(err <= tc_tol(want)), float(err.max())


@pytest.mark.parametrize("rows,cols", [(1152, 896), (896, 896), (9728, 896), (896, 4864), (100, 128), (64, 64)])
@pytest.mark.parametrize("bits,group", [(8, 64), (4, 32)])
def test_gemv_on_the_layer_shapes_of_the_05b_model(rows, cols, bits, group):
    raw = rand_rows(rows, cols, bits, group, rows + cols)
    for M in (1, 5, 9):
        x = np.random.default_rng(M).standard_normal((M, cols)).astype(np.float32)
        y, _ = ls.qgemv(bits, group, raw, rows, cols, x)
        want = O.matmul(bits, group, raw, rows, cols, x)
        assert np.all(np.abs(y - want) <= tc_tol(want))


FMA_CHECK = r"""
import sys, numpy as np
sys.path[:0] = [sys.argv[1], sys.argv[1] + '/tests']
import layerstream_b200 as ls
from oracle import oracle as O
from test_gpu_kernels import rand_rows
worst = 0.0
for bits, group in [(8, 64), (8, 16), (4, 32), (4, 16), (4, 128)]:
    for M in (1, 5, 9, 33):
        raw = rand_rows(160, 896, bits, group, M)
        x = np.random.default_rng(M).standard_normal((M, 896)).astype(np.float32)
        y, _ = ls.qgemv(bits, group, raw, 160, 896, x)
        want = O.matmul(bits, group, raw, 160, 896, x)
        assert np.all(np.abs(y - want) <= 1e-4 * (1 + np.abs(want))), (bits, group, M)
print("fma path ok")
"""


def test_cuda_core_gemv_path_matches_the_oracle_tightly():
    # the CUDA-core kernel (f32 FMA, selected with LS_GEMV=fma) stays a bit-faithful cross-check
    import subprocess, sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, LS_GEMV="fma")
    r = subprocess.run([sys.executable, "-c", FMA_CHECK, root], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "fma path ok" in r.stdout, r.stdout + r.stderr


def test_gpu_quantizer_writes_the_same_bytes_as_the_oracle():
    with F.TempDir("gq") as d:
        F.write_tiny_model(d, 21)
        for body, embed, clip in [((8, 32), (8, 32), True), ((4, 32), (8, 64), True), ((4, 16), (4, 16), False), ((8, 64), (4, 16), True)]:
            a, b = os.path.join(d, "cpu.lsq"), os.path.join(d, "gpu.lsq")
            for p in (a, b):
                if os.path.exists(p):
                    os.remove(p)
            O.quantize_model(d, a, body, embed, clip=clip)
            r = ls.quantize_model(d, b, body, embed, clip=clip)
            assert open(a, "rb").read() == open(b, "rb").read(), (body, embed, clip)
            assert 0 < r < 1
        # the output must not exist already (nothing is overwritten), bad formats are refused
        with pytest.raises(ls.LayerstreamError):
            ls.quantize_model(d, b, (8, 32))
        for bad in [(8, 48), (6, 32), (8, 512)]:
            with pytest.raises(ls.LayerstreamError):
                ls.quantize_model(d, os.path.join(d, "bad.lsq"), bad)
            assert not os.path.exists(os.path.join(d, "bad.lsq"))


def test_gpu_quantizer_on_grid_weights_is_exact():
    # weights on the quantization grid come back exactly (tests/common/mod.rs:44-62)
    with F.TempDir("gq2") as d:
        F.write_tiny_grid_model(d, 5, (8, 32), (4, 16))
        a, b = os.path.join(d, "cpu.lsq"), os.path.join(d, "gpu.lsq")
        O.quantize_model(d, a, (8, 32), (4, 16), clip=True)
        ls.quantize_model(d, b, (8, 32), (4, 16), clip=True)
        assert open(a, "rb").read() == open(b, "rb").read()


@pytest.mark.parametrize("bits,group", [(8, 64), (8, 32), (8, 16), (8, 128), (4, 32), (4, 16)])
@pytest.mark.parametrize("M", [1, 9, 40])
def test_dequantized_weights_enter_the_tensor_cores_exactly(bits, group, M):
    # With activations exactly representable in f16 the only rounding left in the tensor-core paths
    # is the f32 accumulation: int4 weights (q - 8) * s are exact f16 values and int8 weights
    # q * s enter as exact hi + lo f16 parts, so both GEMMs agree with kernels::matmul
    # (src/kernels.rs:53-92) to ~1e-6 relative. (An int8 weight rounded to f16 would be off by up
    # to 2^-11 of itself: about 1e-3 here.)
    rows, cols = 300, 896
    raw = rand_rows(rows, cols, bits, group, 7 + M)
    x = np.random.default_rng(M).standard_normal((M, cols)).astype(np.float16).astype(np.float32)
    want = O.matmul(bits, group, raw, rows, cols, x)
    scale = np.sqrt(np.mean(want.astype(np.float64) ** 2))
    y, _ = ls.qgemv(bits, group, raw, rows, cols, x)
    assert np.max(np.abs(y - want)) <= 2e-5 * scale, float(np.max(np.abs(y - want)) / scale)
    if not (bits == 8 and group > 64):  # the batched GEMM takes int8 groups of up to 64
        yb, _ = ls.bgemm(bits, group, raw, rows, cols, x)
        assert np.max(np.abs(yb - want)) <= 2e-5 * scale, float(np.max(np.abs(yb - want)) / scale)
