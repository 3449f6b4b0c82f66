"""Batched verify (configs 4 and 5: independent sequences sharing one model) against the
single-sequence path and the CPU oracle (needs a B200).

Sequences share only the weights, so each sequence of a batch must decode exactly as it would
alone (src/spec.rs:8-11: speculation never changes the greedy output); against the CPU path the
north-star bar applies (identical tokens wherever the top-2 margin exceeds 2e-2).
"""

import os

import numpy as np
import pytest

import fixtures as F
import layerstream_b200 as ls
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2
PROMPTS = [F.PROMPT, [9, 8, 7, 6, 5, 4], [100, 200, 300, 400, 500, 1], [42, 42, 42, 1, 2, 3]]


@pytest.fixture(scope="module")
def tiny():
    d = F.TempDir("gpu-batch").path
    F.write_tiny_model(d, 13)
    paths = {}
    for body in [(8, 32), (4, 32)]:
        p = os.path.join(d, f"q{body[0]}g{body[1]}.lsq")
        O.quantize_model(d, p, body, body, clip=True)
        paths[body] = p
    yield paths


def plain_greedy(m, prompt, max_new):
    logits = m.forward(prompt)
    out = []
    for i in range(max_new):
        t = int(np.argmax(logits))
        out.append(t)
        if i + 1 == max_new:
            break
        logits = m.forward([t])
    return out


def cpu_greedy_with_margins(p, prompt, max_new):
    c = O.Model(p, quantized=True, threads=4, max_ctx=128)
    logits = c.forward(prompt)
    toks, margins = [], []
    for i in range(max_new):
        srt = np.sort(logits)
        toks.append(int(np.argmax(logits)))
        margins.append(float(srt[-1] - srt[-2]))
        if i + 1 == max_new:
            break
        logits = c.forward([toks[-1]])
    return toks, margins


@pytest.mark.parametrize("body", [(8, 32), (4, 32)])
def test_each_sequence_of_a_batch_decodes_as_it_would_alone(tiny, body):
    p = tiny[body]
    model = ls.Model(p, max_ctx=128)
    max_new = 20
    want = [plain_greedy(ls.Model(p, max_ctx=128), pr, max_new) for pr in PROMPTS]
    for k in [1, 4]:
        b = ls.Batch(model, len(PROMPTS), max_ctx=64, max_block=k + 1)
        got, st = b.spec(np.array(PROMPTS, np.uint32), max_new, k)
        assert got == want, k
        assert st["accepted"] <= st["drafted"]
        b.close()


@pytest.mark.parametrize("body", [(8, 32), (4, 32)])
def test_sixty_four_sequences_decode_as_they_would_alone(tiny, body):
    # 64 sequences x 5 verify rows = 320 rows: two token groups of 160, the batched GEMM's large-group
    # plan (int8: one MMA issuer, four tensor-memory A buffers) in every projection and the head
    # (tokens must equal the CPU path's up to its first near tie, where the streams may diverge)
    p = tiny[body]
    prompts = [[(11 * i + 17 * s + 3) % 600 for i in range(6)] for s in range(64)]
    b = ls.Batch(ls.Model(p, max_ctx=128), 64, max_ctx=64, max_block=5)
    got, _ = b.spec(np.array(prompts, np.uint32), 8, 4)
    checked = 0
    for pr, g in zip(prompts, got):
        toks, margins = cpu_greedy_with_margins(p, pr, 8)
        for i, (t, mg) in enumerate(zip(toks, margins)):
            if mg <= TOL:
                break
            assert g[i] == t, (pr, i)
            checked += 1
    assert checked >= 64
    b.close()


def test_batch_tokens_match_the_cpu_path_where_margins_allow(tiny):
    p = tiny[(4, 32)]
    b = ls.Batch(ls.Model(p, max_ctx=128), len(PROMPTS), max_ctx=64, max_block=5)
    got, _ = b.spec(np.array(PROMPTS, np.uint32), 24, 4)
    for pr, g in zip(PROMPTS, got):
        toks, margins = cpu_greedy_with_margins(p, pr, 24)
        for i, (t, mg) in enumerate(zip(toks, margins)):
            if mg <= TOL:
                break  # past a near tie the streams may legitimately diverge
            assert g[i] == t, (pr, i)


def test_batch_verify_accepts_a_perfect_draft_and_advances_each_sequence(tiny):
    p = tiny[(8, 32)]
    model = ls.Model(p, max_ctx=128)
    M = 5
    conts = [plain_greedy(ls.Model(p, max_ctx=128), pr, M + 1) for pr in PROMPTS]
    b = ls.Batch(model, len(PROMPTS), max_ctx=64, max_block=M)
    for i, pr in enumerate(PROMPTS):
        assert b.prefill(i, pr) == conts[i][0]
    blocks = np.array([c[:M] for c in conts], np.uint32)
    m, nxt = b.verify(blocks)
    assert m == [M - 1] * len(PROMPTS)
    assert nxt == [c[M] for c in conts]
    assert [b.pos(i) for i in range(len(PROMPTS))] == [len(pr) + M for pr in PROMPTS]
    # a wrong guess at position 2 of sequence 1 only: it accepts 1, the others continue from M
    b2 = ls.Batch(model, 2, max_ctx=64, max_block=M)
    for i in range(2):
        b2.prefill(i, PROMPTS[i])
    blk = np.array([conts[0][:M], conts[1][:M]], np.uint32)
    blk[1, 2] = (blk[1, 2] + 1) % F.VOCAB
    m2, nxt2 = b2.verify(blk)
    assert m2 == [M - 1, 1] and nxt2 == [conts[0][M], conts[1][2]]
    b2.truncate(1, len(PROMPTS[1]))
    assert b2.pos(1) == len(PROMPTS[1])


def test_bad_batch_requests_are_errors(tiny):
    p = tiny[(8, 32)]
    model = ls.Model(p, max_ctx=128)
    b = ls.Batch(model, 2, max_ctx=16, max_block=3)
    with pytest.raises(ls.LayerstreamError):
        b.prefill(0, [F.VOCAB])  # id outside the vocabulary
    with pytest.raises(ls.LayerstreamError):
        b.prefill(2, [1])  # no such sequence
    with pytest.raises(ls.LayerstreamError):
        b.prefill(0, list(range(1, 18)))  # context overflow
    with pytest.raises(ls.LayerstreamError):
        b.verify(np.zeros((2, 4), np.uint32))  # block longer than max_block


@pytest.mark.parametrize("slots", [1, 2])
def test_a_batch_over_streamed_weights_decodes_like_the_resident_one(tiny, slots):
    # config 5 (a): the layers and head chunks stream through HBM slots; the batch's tokens and the
    # streamed bytes follow tests/quant.rs:232-248 per pass
    p = tiny[(4, 32)]
    prompts = np.array(PROMPTS, np.uint32)
    want, _ = ls.Batch(ls.Model(p, max_ctx=128), len(PROMPTS), max_ctx=64, max_block=5).spec(prompts, 16, 4)
    sm = ls.Model(p, mode="stream", slots=slots, max_ctx=128)
    b = ls.Batch(sm, len(PROMPTS), max_ctx=64, max_block=5)
    got, st = b.spec(prompts, 16, 4)
    assert got == want
    info = sm.info
    per_pass = info.layers * info.layer_bytes
    head = info.vocab * info.embed_row_bytes
    passes = b.report()["passes"]
    # the prompts' chunks run together (up to 16 sequences per pass): one pass for these short
    # prompts, with the head on every sequence's last row
    prefill_passes = 1
    verify_passes = st["target_passes"]
    rows = len(PROMPTS) * len(PROMPTS[0]) + verify_passes * len(PROMPTS) * 5
    assert passes == prefill_passes + verify_passes
    assert sm.report()["bytes_read"] == passes * (per_pass + head) + rows * info.embed_row_bytes


def test_a_wide_model_verifies_a_large_batch_without_splitting_the_head():
    # hidden 2048 (the 3B width): the staged activations of 40 verify rows outgrow one K slice of
    # the LM-head GEMV, whose argmax epilogue needs whole dot products; the head narrows its token
    # groups instead. Every sequence must still decode as it does alone.
    from layerstream_b200 import synth

    synth.SHAPES["wide-test"] = dict(hidden_size=2048, num_attention_heads=16, num_key_value_heads=2,
                                     intermediate_size=256, num_hidden_layers=1, vocab_size=1000, rope_theta=1e6,
                                     max_position_embeddings=4096)
    d = F.TempDir("gpu-wide").path
    synth.write_random_model(d, "wide-test", 3)
    p = os.path.join(d, "w.lsq")
    ls.quantize_model(d, p, body=(4, 32), embed=(4, 32))
    prompts = [[(7 * i + 13 * s) % 1000 for i in range(12)] for s in range(8)]
    want = [plain_greedy(ls.Model(p, max_ctx=64), pr, 10) for pr in prompts]
    b = ls.Batch(ls.Model(p, max_ctx=64), 8, max_ctx=64, max_block=5)
    got, _ = b.spec(np.array(prompts, np.uint32), 10, 4)
    assert got == want
