"""Pins the CPU oracle against the reference's synthetic-model integration tests.

Ports of tests/spec.rs:63-193, tests/quant.rs:75-230 and tests/pipeline.rs:200-229, run on the
tiny LCG model of tests/common/mod.rs. No GPU needed.
"""

import os

import numpy as np
import pytest

from oracle import oracle as O
import fixtures as F


def quantize(d, name, body, embed=None, clip=True):
    out = os.path.join(d, name)
    if os.path.exists(out):
        os.remove(out)
    O.quantize_model(d, out, body, embed or body, clip=clip, threads=3)
    return out


def plain_greedy(m, prompt, max_new, eos=()):
    logits = m.forward(prompt)
    out = []
    for i in range(max_new):
        t = O.argmax(logits)
        out.append(t)
        if t in eos or i + 1 == max_new:
            break
        logits = m.forward([t])
    return out


def test_checking_several_positions_at_once_gives_bit_identical_logits():
    # tests/spec.rs:63-84
    with F.TempDir("multi") as d:
        F.write_tiny_model(d, 11)
        block = [8, 9, 400, 33, 120]
        for n in [1, 2, len(block)]:
            a = O.Model(d, threads=3)
            a.forward(F.PROMPT)
            together = a.forward_multi(block, n)
            b = O.Model(d, threads=3)
            b.forward(F.PROMPT)
            one = np.stack([b.forward([t]) for t in block])
            assert np.array_equal(together.view(np.uint32), one[len(block) - n:].view(np.uint32))
            assert a.pos == b.pos


def test_truncating_the_cache_forgets_the_tail_exactly():
    # tests/spec.rs:86-101
    with F.TempDir("trunc") as d:
        F.write_tiny_model(d, 12)
        a = O.Model(d)
        a.forward(F.PROMPT)
        a.forward([7, 8, 9])
        a.truncate(len(F.PROMPT))
        x = a.forward([20])
        b = O.Model(d)
        b.forward(F.PROMPT)
        y = b.forward([20])
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))


def test_speculation_never_changes_the_output_whatever_the_draft_guesses():
    # tests/spec.rs:103-132 (the stream/resident axis is the same bytes here)
    with F.TempDir("same") as d, F.TempDir("other") as other:
        F.write_tiny_model(d, 13)
        F.write_tiny_model(other, 99)
        q8 = quantize(d, "d8.lsq", (8, 32))
        q4 = quantize(d, "d4.lsq", (4, 32))
        for name, dp in [("int8", q8), ("int4", q4), ("unrelated", other)]:
            for prompt in [F.PROMPT, F.OTHER_PROMPT]:
                for max_new in [1, 2, 9, 30]:
                    want = plain_greedy(O.Model(d), prompt, max_new)
                    for k in [1, 2, 3, 5, 8]:
                        got, st = O.speculative_greedy(O.Model(d), O.Model(dp), prompt, max_new, k)
                        assert got == want, (name, len(prompt), max_new, k)
                        assert st["accepted"] <= st["drafted"]
                        assert st["target_passes"] <= max(len(got) - 1, 0)


def test_it_stops_at_an_end_of_sequence_token_exactly_where_plain_greedy_does():
    # tests/spec.rs:134-151
    with F.TempDir("eos") as d:
        F.write_tiny_model(d, 14)
        full = plain_greedy(O.Model(d), F.PROMPT, 24)
        for cut in [0, 1, 5, 11]:
            eos = [full[cut]]
            want = plain_greedy(O.Model(d), F.PROMPT, 24, eos)
            assert len(want) <= cut + 1 and want[-1] == eos[0]
            for k in [1, 4, 8]:
                got, _ = O.speculative_greedy(O.Model(d), O.Model(d), F.PROMPT, 24, k, eos)
                assert got == want, (cut, k)


def test_a_perfect_draft_needs_far_fewer_passes_over_the_weights():
    # tests/spec.rs:153-173 (pass count; the byte count is checked on the GPU streaming path)
    with F.TempDir("perfect") as d:
        F.write_tiny_model(d, 15)
        max_new, k = 21, 3
        want = plain_greedy(O.Model(d), F.PROMPT, max_new)
        got, st = O.speculative_greedy(O.Model(d), O.Model(d), F.PROMPT, max_new, k)
        assert got == want
        assert st["accepted"] == st["drafted"]
        assert st["target_passes"] == -(-(max_new - 1) // (k + 1))


def test_bad_requests_are_errors_not_panics():
    # tests/spec.rs:175-193 and tests/pipeline.rs:218-229
    with F.TempDir("bad") as d:
        F.write_tiny_model(d, 16)
        t, dr = O.Model(d), O.Model(d)
        for k, prompt, max_new in [(0, F.PROMPT, 5), (33, F.PROMPT, 5), (2, [], 5), (2, F.PROMPT, 0), (2, F.PROMPT, 500)]:
            with pytest.raises(O.OracleError):
                O.speculative_greedy(t, dr, prompt, max_new, k)
        t.forward(F.PROMPT)
        with pytest.raises(O.OracleError):
            O.speculative_greedy(t, dr, F.PROMPT, 5, 2)
        t2 = O.Model(d)
        with pytest.raises(O.OracleError):
            t2.forward_multi([1, 2], 3)
        with pytest.raises(O.OracleError):
            t2.forward_multi([1, 2], 0)
        m = O.Model(d, max_ctx=64)
        with pytest.raises(O.OracleError):
            m.forward([])
        with pytest.raises(O.OracleError):
            m.forward([F.VOCAB])
        with pytest.raises(O.OracleError):
            m.forward([1] * 65)
        m.forward([1] * 60)
        with pytest.raises(O.OracleError):
            m.forward([1] * 5)
        m.reset()
        m.forward([1] * 64)


GRID_CASES = [((8, 32), (8, 32)), ((8, 16), (8, 64)), ((4, 32), (4, 32)), ((4, 16), (4, 64)), ((4, 32), (8, 16)), ((8, 64), (4, 16))]


def run_fixed(m):
    out = [m.forward(F.PROMPT)]
    for t in F.FOLLOW:
        out.append(m.forward([t]))
    return np.stack(out)


@pytest.mark.parametrize("case", range(len(GRID_CASES)))
def test_a_quantized_model_computes_the_same_thing_as_bf16_when_the_weights_fit_the_grid(case):
    # tests/quant.rs:75-103
    body, embed = GRID_CASES[case]
    with F.TempDir(f"grid{case}") as d:
        F.write_tiny_grid_model(d, 100 + case, body, embed)
        ref = run_fixed(O.Model(d, max_ctx=64))
        assert np.max(np.abs(ref)) > 0.01
        for clip in [False, True]:
            q = quantize(d, "m.lsq", body, embed, clip)
            got = run_fixed(O.Model(q, max_ctx=64))
            tol = 1e-3 * (1 + np.max(np.abs(ref)))
            assert np.max(np.abs(ref - got)) < tol, (body, embed, clip)


def test_rounding_real_weights_stays_close_and_eight_bits_is_closer_than_four():
    # tests/quant.rs:105-122
    with F.TempDir("random") as d:
        F.write_tiny_model(d, 7)
        ref = run_fixed(O.Model(d, max_ctx=64))
        scale = np.max(np.abs(ref))

        def err(body):
            got = run_fixed(O.Model(quantize(d, "r.lsq", body), max_ctx=64))
            assert np.all(np.isfinite(got))
            return np.max(np.abs(ref - got)) / scale

        e8, e4 = err((8, 32)), err((4, 32))
        assert e8 < 0.05 and e4 > e8 and e4 < 1.0


def test_quantized_files_are_smaller_and_the_sizes_add_up():
    # tests/quant.rs:174-192
    with F.TempDir("size") as d:
        F.write_tiny_model(d, 4)
        bf16_len = os.path.getsize(os.path.join(d, "model.safetensors"))
        last = 1 << 62
        for body, embed in [((8, 32), (8, 32)), ((4, 32), (8, 32)), ((4, 32), (4, 32))]:
            q = quantize(d, "s.lsq", body, embed, clip=False)
            n = os.path.getsize(q)
            assert n < bf16_len and n < last
            last = n
            info = O.open_files(q, True)
            rb = O.row_bytes(embed[0], embed[1], F.HIDDEN)
            assert n == info["norm_start"] + F.HIDDEN * 2
            assert info["norm_start"] - info["embed_start"] == F.VOCAB * rb


def test_bad_quantization_requests_and_damaged_files_are_errors():
    # tests/quant.rs:194-230
    with F.TempDir("qbad") as d:
        F.write_tiny_model(d, 5)
        out = os.path.join(d, "x.lsq")
        for bad in [(8, 48), (6, 32), (8, 512)]:
            if os.path.exists(out):
                os.remove(out)
            with pytest.raises(O.OracleError):
                O.quantize_model(d, out, bad, bad)
        good = quantize(d, "good.lsq", (8, 32))
        with pytest.raises(O.OracleError, match="exist"):
            O.quantize_model(d, good, (8, 32), (8, 32))
        with pytest.raises(O.OracleError):
            O.open_files(os.path.join(d, "model.safetensors"), True)
        data = open(good, "rb").read()

        def write(name, b):
            p = os.path.join(d, name)
            open(p, "wb").write(b)
            return p

        for name, b in [("trunc.lsq", data[:-3]), ("long.lsq", data + b"\0"), ("magic.lsq", bytes([data[0] ^ 1]) + data[1:]),
                        ("tiny.lsq", data[:5])]:
            with pytest.raises(O.OracleError):
                O.open_files(write(name, b), True)


def test_incremental_decoding_matches_processing_the_whole_prompt():
    # tests/pipeline.rs:200-217
    with F.TempDir("kv") as d:
        F.write_tiny_model(d, 6)
        toks = [(i * 31 + 7) % F.VOCAB for i in range(20)]
        want = O.Model(d, max_ctx=64).forward(toks)
        inc = O.Model(d, max_ctx=64)
        inc.forward(toks[:9])
        for t in toks[9:19]:
            inc.forward([t])
        got = inc.forward(toks[19:])
        assert np.max(np.abs(want - got)) < 1e-4
        assert inc.pos == 20
