"""The batched verify-pass GEMM (tensor cores, every token of a group per weight tile) against the
oracle's matmul (src/kernels.rs:53-92,123-203) (needs a B200).

Weights (q * scale) and activations enter the MMA as f16 and accumulate in f32, the same bound as
the tensor-core GEMV; covered: every format of the configs, token counts from 1 to past one
256-token group (two groups), matrices small enough to split K over CTAs, and row counts that end
in a partial 128-row tile.
"""

import numpy as np
import pytest

import layerstream_b200 as ls
from oracle import oracle as O
from test_gpu_kernels import FORMATS, rand_rows, tc_tol

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits,group", FORMATS)
@pytest.mark.parametrize("M", [1, 7, 40, 160, 300])
def test_batched_gemm_matches_the_oracle_matmul(bits, group, M):
    rows, cols = 200, 896  # a partial 128-row tile; small enough to split K
    raw = rand_rows(rows, cols, bits, group, 5 + M)
    x = np.random.default_rng(M).standard_normal((M, cols)).astype(np.float32)
    y, _ = ls.bgemm(bits, group, raw, rows, cols, x)
    want = O.matmul(bits, group, raw, rows, cols, x)
    err = np.abs(y - want)
    assert np.all(err <= tc_tol(want)), float(err.max())


@pytest.mark.parametrize("rows,cols,M", [(1152, 896, 45), (896, 4864, 45), (2560, 2048, 40), (4096, 896, 320)])
def test_batched_gemm_on_verify_shapes(rows, cols, M):
    for bits, group in [(8, 64), (4, 32)]:
        raw = rand_rows(rows, cols, bits, group, rows + M)
        x = np.random.default_rng(rows).standard_normal((M, cols)).astype(np.float32)
        y, _ = ls.bgemm(bits, group, raw, rows, cols, x)
        want = O.matmul(bits, group, raw, rows, cols, x)
        assert np.all(np.abs(y - want) <= tc_tol(want)), (bits, group)


def test_batched_gemm_rejects_bad_shapes():
    raw = np.zeros(64 * O.row_bytes(8, 64, 64), np.uint8)
    with pytest.raises(ls.LayerstreamError):
        ls.bgemm(8, 64, raw, 64, 64, np.zeros((0, 64), np.float32))
