"""Model-level parity of the CUDA verify path against the CPU oracle, on the reference's tiny LCG
model (tests/common/mod.rs) quantized by both quantizers (needs a B200).

Bar: logits within 2e-2 absolute of the CPU path; greedy token streams
identical wherever the top-2 margin of the CPU logits exceeds that tolerance. The speculative
invariants of tests/spec.rs are checked on the GPU path itself.
"""

import os

import numpy as np
import pytest

import layerstream_b200 as ls
from oracle import oracle as O
import fixtures as F

pytestmark = pytest.mark.gpu

TOL = 2e-2  # absolute logit tolerance of the north star


@pytest.fixture(scope="module")
def tiny():
    d = F.TempDir("gpu-model").path
    F.write_tiny_model(d, 13)
    paths = {}
    for body, embed in [((8, 32), (8, 32)), ((4, 32), (4, 32)), ((8, 64), (8, 64)), ((4, 16), (8, 32)), ((4, 32), (8, 32))]:
        p = os.path.join(d, f"q{body[0]}g{body[1]}e{embed[0]}g{embed[1]}.lsq")
        O.quantize_model(d, p, body, embed, clip=True)
        paths[(body, embed)] = p
    other = F.TempDir("gpu-other").path
    F.write_tiny_model(other, 99)
    po = os.path.join(other, "o.lsq")
    O.quantize_model(other, po, (4, 32), (4, 32))
    paths["other"] = po
    yield paths


def gpu(p, **kw):
    kw.setdefault("max_ctx", 128)
    return ls.Model(p, **kw)


def cpu(p, max_ctx=128):
    return O.Model(p, quantized=True, threads=4, max_ctx=max_ctx)


@pytest.mark.parametrize("key", [((8, 32), (8, 32)), ((4, 32), (4, 32)), ((8, 64), (8, 64)), ((4, 16), (8, 32))])
def test_prefill_and_decode_logits_match_the_cpu_path(tiny, key):
    p = tiny[key]
    g, c = gpu(p), cpu(p)
    toks = F.PROMPT
    lg, lc = g.forward(toks), c.forward(toks)
    assert np.max(np.abs(lg - lc)) < TOL
    for t in F.FOLLOW + [int(O.argmax(lc))]:
        lg, lc = g.forward([t]), c.forward([t])
        d = float(np.max(np.abs(lg - lc)))
        assert d < TOL, d
    assert g.pos == c.pos


def test_forward_multi_equals_single_token_passes(tiny):
    # tests/spec.rs:63-84 on the GPU path
    p = tiny[((8, 32), (8, 32))]
    block = [8, 9, 400, 33, 120]
    for n in [1, 2, len(block)]:
        a = gpu(p)
        a.forward(F.PROMPT)
        together = a.forward_multi(block, n)
        b = gpu(p)
        b.forward(F.PROMPT)
        one = np.stack([b.forward([t]) for t in block])[len(block) - n:]
        assert np.max(np.abs(together - one)) < 1e-5
        assert a.pos == b.pos
        c = cpu(p)
        c.forward(F.PROMPT)
        assert np.max(np.abs(together - c.forward_multi(block, n))) < TOL


def test_a_long_prompt_spans_several_prefill_chunks(tiny):
    p = tiny[((4, 32), (4, 32))]
    toks = [(i * 31 + 7) % F.VOCAB for i in range(300)]
    g, c = gpu(p, max_ctx=320), cpu(p, max_ctx=320)
    assert np.max(np.abs(g.forward(toks) - c.forward(toks))) < TOL
    assert g.pos == 300


def test_truncating_the_cache_forgets_the_tail(tiny):
    p = tiny[((8, 32), (8, 32))]
    a = gpu(p)
    a.forward(F.PROMPT)
    a.forward([7, 8, 9])
    a.truncate(len(F.PROMPT))
    x = a.forward([20])
    b = gpu(p)
    b.forward(F.PROMPT)
    y = b.forward([20])
    assert np.array_equal(x.view(np.uint32), y.view(np.uint32))


def test_verify_applies_the_acceptance_rule(tiny):
    p = tiny[((8, 32), (8, 32))]
    ref = gpu(p)
    ref.forward(F.PROMPT)
    a = ref.last_argmax
    # the target's own greedy continuation: every guess right
    seq = [a]
    for _ in range(5):
        seq.append(int(np.argmax(ref.forward([seq[-1]]))))
    g = gpu(p)
    g.forward(F.PROMPT)
    m, nxt = g.verify(seq[:5])
    assert (m, nxt) == (4, seq[5]) and g.pos == len(F.PROMPT) + 5
    # a wrong guess at position 2: keep a, d1, d2 ... no: keep [a, d1], the correction is seq[2]
    g2 = gpu(p)
    g2.forward(F.PROMPT)
    bad = seq[:5]
    bad[2] = (bad[2] + 1) % F.VOCAB
    m, nxt = g2.verify(bad)
    assert (m, nxt) == (1, seq[2]) and g2.pos == len(F.PROMPT) + 2
    # the cache now equals a model that saw exactly [a, d1]
    g3 = gpu(p)
    g3.forward(F.PROMPT + seq[:2])
    assert np.max(np.abs(g2.forward([seq[2]]) - g3.forward([seq[2]]))) < 1e-5


def plain_greedy(m, prompt, max_new, eos=()):
    logits = m.forward(prompt)
    out = []
    for i in range(max_new):
        t = int(np.argmax(logits))
        out.append(t)
        if t in eos or i + 1 == max_new:
            break
        logits = m.forward([t])
    return out


def test_speculation_never_changes_the_output(tiny):
    # tests/spec.rs:103-132 on the GPU path (target resident and streamed; three drafts + lookup)
    p = tiny[((8, 32), (8, 32))]
    drafts = [("int4 copy", tiny[((4, 32), (4, 32))]), ("unrelated", tiny["other"]), ("lookup", None)]
    for prompt in [F.PROMPT, F.OTHER_PROMPT]:
        for max_new in [1, 2, 9, 30]:
            want = plain_greedy(gpu(p), prompt, max_new)
            for name, dp in drafts:
                for k in [1, 3, 8]:
                    for mode in ["resident", "stream"]:
                        t = gpu(p, mode=mode, slots=2)
                        d = gpu(dp) if dp else None
                        got, st = ls.speculative_greedy(t, d, prompt, max_new, k)
                        assert got == want, (name, len(prompt), max_new, k, mode)
                        assert st["accepted"] <= st["drafted"]
                        assert st["target_passes"] <= max(len(got) - 1, 0)


def test_greedy_streams_match_the_cpu_path_where_margins_allow(tiny):
    # teacher-forced on the CPU tokens: every position whose top-2 margin exceeds TOL must agree
    p = tiny[((4, 32), (4, 32))]
    c = cpu(p)
    cpu_tokens = plain_greedy(c, F.PROMPT, 40)
    g, c2 = gpu(p), cpu(p)
    lg, lc = g.forward(F.PROMPT), c2.forward(F.PROMPT)
    checked = 0
    for i, t in enumerate(cpu_tokens):
        srt = np.sort(lc)
        if srt[-1] - srt[-2] > TOL:
            assert int(np.argmax(lg)) == int(np.argmax(lc)) == t
            checked += 1
        lg, lc = g.forward([t]), c2.forward([t])
    assert checked >= 30


def test_eos_stops_exactly_where_plain_greedy_does(tiny):
    p = tiny[((8, 32), (8, 32))]
    full = plain_greedy(gpu(p), F.PROMPT, 24)
    for cut in [0, 1, 5, 11]:
        eos = [full[cut]]
        want = plain_greedy(gpu(p), F.PROMPT, 24, eos)
        for k in [1, 4, 8]:
            got, _ = ls.speculative_greedy(gpu(p), gpu(p), F.PROMPT, 24, k, eos)
            assert got == want, (cut, k)


def test_a_perfect_draft_needs_far_fewer_passes_and_bytes(tiny):
    # tests/spec.rs:153-173: streamed target, the same model as draft
    p = tiny[((8, 32), (8, 32))]
    max_new, k = 21, 3
    base = gpu(p, mode="stream", slots=2)
    want = plain_greedy(base, F.PROMPT, max_new)
    base_bytes = base.report()["bytes_read"]
    t = gpu(p, mode="stream", slots=2)
    got, st = ls.speculative_greedy(t, gpu(p), F.PROMPT, max_new, k)
    assert got == want
    assert st["accepted"] == st["drafted"]
    assert st["target_passes"] == -(-(max_new - 1) // (k + 1))
    assert t.report()["bytes_read"] * 3 < base_bytes


@pytest.mark.parametrize("slots", [1, 2, 3])
def test_streaming_gives_bit_identical_logits_and_reads_the_expected_bytes(tiny, slots):
    # tests/quant.rs:142-172 and 232-248
    p = tiny[((4, 32), (8, 32))]
    r, s = gpu(p), gpu(p, mode="stream", slots=slots)
    out_r, out_s = [r.forward(F.PROMPT)], [s.forward(F.PROMPT)]
    for _ in range(3):
        nxt = int(np.argmax(out_r[-1]))
        out_r.append(r.forward([nxt]))
        out_s.append(s.forward([nxt]))
    assert np.array_equal(np.stack(out_r).view(np.uint32), np.stack(out_s).view(np.uint32))
    info = s.info
    per_pass = info.layers * info.layer_bytes + info.vocab * info.embed_row_bytes
    assert s.report()["bytes_read"] == 4 * per_pass + 9 * info.embed_row_bytes
    # HBM holds `slots` slots of one layer or head chunk (raw bytes + repacked planes), never the model
    chunk = min(4096, info.vocab) * info.embed_row_bytes
    slot_max = 2 * max(info.layer_bytes, chunk) + 64 * 1024
    assert s.report()["resident_weight_bytes"] <= slots * slot_max


def test_bad_requests_are_errors_not_crashes(tiny):
    p = tiny[((8, 32), (8, 32))]
    t, d = gpu(p), gpu(p)
    for k, prompt, max_new in [(0, F.PROMPT, 5), (33, F.PROMPT, 5), (2, [], 5), (2, F.PROMPT, 0), (2, F.PROMPT, 500)]:
        with pytest.raises(ls.LayerstreamError):
            ls.speculative_greedy(t, d, prompt, max_new, k)
    t.forward(F.PROMPT)
    with pytest.raises(ls.LayerstreamError):
        ls.speculative_greedy(t, d, F.PROMPT, 5, 2)
    m = gpu(p, max_ctx=64)
    for bad in [[], [F.VOCAB], [1] * 65]:
        with pytest.raises(ls.LayerstreamError):
            m.forward(bad)
    with pytest.raises(ls.LayerstreamError):
        m.forward_multi([1, 2], 3)
    with pytest.raises(ls.LayerstreamError):
        m.forward_multi([1, 2], 0)
    m.forward([1] * 60)
    with pytest.raises(ls.LayerstreamError):
        m.forward([1] * 5)
    with pytest.raises(ls.LayerstreamError):
        m.truncate(61)
    m.reset()
    m.forward([1] * 64)
    with pytest.raises(ls.LayerstreamError):
        ls.Model(os.path.join(os.path.dirname(p), "model.safetensors"))
