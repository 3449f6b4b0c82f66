"""The tensor-parallel reduction kernels (layerstream_b200/csrc/ls_p2p.cu) on one GPU (needs a B200).

In a tensor-parallel batch every rank sums the row-parallel projections' partials of all ranks,
read from the peers' memory, into its residual stream (the residual adds after O and down,
src/model.rs:283-297, split over GPUs). Here the peers are emulated in one GPU's memory: with their
flags set before the launch the kernel never waits, and its sums must equal the rank-ordered f32
sums bit for bit, and the fused form (the sum, then the RMSNorm and f16 packing of the next batched
GEMM's operand) must give the same x and the normalised operand; with the flags left unset the
bounded wait must run out, report the error and leave the GPU usable. No two launches wait on one
another.
"""
import numpy as np
import pytest

import layerstream_b200 as ls

pytestmark = pytest.mark.gpu


def _want(x, ys, calls):
    acc = ys[0].copy()
    for y in ys[1:]:  # ranks in order, as every rank sums them
        acc = (acc + y).astype(np.float32)
    out = x.copy()
    for _ in range(calls):
        out = (out + acc).astype(np.float32)
    return out


@pytest.mark.parametrize("world,rank,n,calls", [(2, 0, 8 * 5 * 2048, 1), (2, 1, 1, 2), (4, 3, 4097, 3), (8, 5, 9 * 896 + 3, 2),
                                                 (8, 0, 320 * 4096, 1)])
def test_sums_equal_the_rank_ordered_f32_sums(world, rank, n, calls):
    rng = np.random.default_rng(world * 100 + n)
    x = rng.standard_normal(n).astype(np.float32)
    ys = rng.standard_normal((world, n)).astype(np.float32) * 0.1
    got, ms = ls.tp_reduce(x, ys, rank, preset=True, calls=calls)
    np.testing.assert_array_equal(got, _want(x, ys, calls))
    assert ms > 0


@pytest.mark.parametrize("world,rank,M,K", [(2, 0, 40, 2048), (2, 1, 5, 896), (4, 2, 130, 2048), (8, 7, 17, 1536)])
def test_the_fused_form_adds_then_normalises_the_rows(world, rank, M, K):
    rng = np.random.default_rng(M * K + world)
    x = rng.standard_normal(M * K).astype(np.float32)
    ys = (rng.standard_normal((world, M * K)) * 0.3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    got, ms, op = ls.tp_reduce(x, ys, rank, preset=True, K=K, norm=w, eps=1e-6)
    want = _want(x, ys, 1)
    np.testing.assert_array_equal(got, want)
    rows = want.reshape(M, K).astype(np.float64)
    inv = 1.0 / np.sqrt((rows * rows).mean(axis=1) + 1e-6)
    ref = (rows * inv[:, None] * w[None, :]).astype(np.float32)
    np.testing.assert_allclose(op.astype(np.float32), ref, rtol=2e-3, atol=1e-4)
    # without weights: the plain f16 copy of the summed rows
    _, _, op2 = ls.tp_reduce(x, ys, rank, preset=True, K=K)
    np.testing.assert_array_equal(op2, want.reshape(M, K).astype(np.float16))


def test_a_peer_that_never_answers_ends_the_wait_with_an_error():
    x = np.ones(4096, np.float32)
    ys = np.ones((2, 4096), np.float32)
    with pytest.raises(ls.LayerstreamError) as e:
        ls.tp_reduce(x, ys, 0, preset=False, wait_ms=200)
    assert e.value.code == -4 and "did not answer" in str(e.value)
    # the context stays usable
    got, _ = ls.tp_reduce(x, ys, 1, preset=True)
    np.testing.assert_array_equal(got, np.full(4096, 3, np.float32))
