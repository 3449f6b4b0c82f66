"""The bf16 weight path (needs a B200): unquantized models, as the reference runs them through
matmul_bf16 / dot_bf16 (src/kernels.rs:27-43,178-180) when a model directory holds BF16
safetensors (src/weights.rs:271-324).

A bf16 weight converts exactly to f16 for magnitudes from 2^-17 up to 65504 (f16 keeps 11
significant bits against bf16's 8), so the tensor-core GEMV takes bf16 rows with a conversion in
place of the dequantization. Checked against the CPU path: the GEMV at the tight bound (activations
exactly representable in f16), the embedding gather bit-exact, model logits within the north-star
tolerance 2e-2, greedy tokens wherever the top-2 margin allows, and speculation (lookup drafter and
an int4 draft of the same model) never changing the output (tests/spec.rs:103-132).
"""
import os

import numpy as np
import pytest

import fixtures as F
import layerstream_b200 as ls
from layerstream_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2


def bf16_rows(rows, cols, seed, std=0.05):
    w = (np.random.default_rng(seed).standard_normal((rows, cols)) * std).astype(np.float32)
    return np.ascontiguousarray(synth.f32_to_bf16_rne(w).view(np.uint8).reshape(-1))


@pytest.mark.parametrize("M", [1, 9, 40])
def test_bf16_gemv_matches_kernels_matmul(M):
    rows, cols = 200, 896
    raw = bf16_rows(rows, cols, M)
    x = np.random.default_rng(M).standard_normal((M, cols)).astype(np.float16).astype(np.float32)
    y, _ = ls.qgemv(16, 0, raw, rows, cols, x)
    want = O.matmul(16, 0, raw, rows, cols, x)
    scale = np.sqrt(np.mean(want.astype(np.float64) ** 2))
    assert np.max(np.abs(y - want)) <= 2e-5 * scale, float(np.max(np.abs(y - want)) / scale)


def test_bf16_embedding_rows_are_exact():
    rows, cols = 100, 896
    raw = bf16_rows(rows, cols, 3)
    ids = [0, 1, 31, 32, 99, 50]
    got = ls.dequant_rows(16, 0, raw, rows, cols, ids)
    rb = cols * 2
    for i, r in enumerate(ids):
        want = O.dequant_row(16, 0, raw[r * rb:(r + 1) * rb], cols)
        assert np.array_equal(got[i].view(np.uint32), want.view(np.uint32))


@pytest.fixture(scope="module")
def tiny():
    d = F.TempDir("gpu-bf16").path
    F.write_tiny_model(d, 13)
    q = os.path.join(d, "draft-q4g32.lsq")
    O.quantize_model(d, q, (4, 32), (4, 32), clip=True)
    yield d, q


def test_bf16_model_logits_match_the_cpu_path(tiny):
    d, _ = tiny
    g, c = ls.Model(d, max_ctx=128), O.Model(d, quantized=False, threads=4, max_ctx=128)
    assert g.info.bits == 16 and g.info.embed_bits == 16
    lg, lc = g.forward(F.PROMPT), c.forward(F.PROMPT)
    assert np.max(np.abs(lg - lc)) < TOL
    for t in F.FOLLOW:
        lg, lc = g.forward([t]), c.forward([t])
        assert np.max(np.abs(lg - lc)) < TOL
    block = [5, 6, 7, 8, 9]
    assert np.max(np.abs(g.forward_multi(block, 5) - c.forward_multi(block, 5))) < TOL
    g.close()


def test_bf16_greedy_tokens_match_the_cpu_path_where_margins_allow(tiny):
    d, _ = tiny
    g, c = ls.Model(d, max_ctx=128), O.Model(d, quantized=False, threads=4, max_ctx=128)
    lg, lc = g.forward(F.PROMPT), c.forward(F.PROMPT)
    checked = 0
    for _ in range(30):
        t = int(O.argmax(lc))
        srt = np.sort(lc)
        if srt[-1] - srt[-2] > TOL:
            assert int(np.argmax(lg)) == t
            checked += 1
        lg, lc = g.forward([t]), c.forward([t])
    assert checked >= 20
    g.close()


def test_bf16_speculation_never_changes_the_output(tiny):
    d, q = tiny

    def plain(m, n):
        logits = m.forward(F.PROMPT)
        out = []
        for i in range(n):
            out.append(int(np.argmax(logits)))
            if i + 1 < n:
                logits = m.forward([out[-1]])
        return out

    want = plain(ls.Model(d, max_ctx=128), 25)
    for draft in (None, q):
        for k in (1, 4):
            got, st = ls.speculative_greedy(ls.Model(d, max_ctx=128), ls.Model(draft, max_ctx=128) if draft else None,
                                            F.PROMPT, 25, k)
            assert got == want, (draft, k)


def test_a_bf16_model_is_opened_resident_only(tiny):
    d, _ = tiny
    with pytest.raises(ls.LayerstreamError):
        ls.Model(d, mode="stream", slots=2)
