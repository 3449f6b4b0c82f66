"""Pins the CPU oracle against the reference's unit tests (known answers and invariants).

Ports of src/quant.rs:272-397, src/kernels.rs:285-347, src/weights.rs:430-464 and
src/model.rs:372-376. These run without a GPU.
"""

import numpy as np
import pytest

from oracle import oracle as O
from fixtures import Lcg

BASE_CFG = (
    '{"model_type":"qwen2","hidden_act":"silu","tie_word_embeddings":true,"hidden_size":896,\n'
    '            "num_attention_heads":14,"num_key_value_heads":2,"intermediate_size":4864,"num_hidden_layers":24,\n'
    '            "vocab_size":151936,"rms_norm_eps":1e-6,"rope_theta":1000000.0,"max_position_embeddings":32768}\n'
)


def lcg_vals(seed, n):
    return Lcg(seed).many(n)


def test_bf16_rounding_is_round_to_nearest_even():
    # src/quant.rs:272-282
    assert O.bf16_round(1.0) == 1.0
    assert O.bf16_round(1.0 + 2.0**-8) == 1.0
    assert O.bf16_round(1.0 + 3.0 * 2.0**-8) == 1.0 + 2.0**-6
    assert O.bf16_round(1.0 + 2.0**-9) == 1.0
    assert np.isnan(O.bf16_round(float("nan")))
    assert O.bf16_round(float("inf")) == float("inf")
    v = float(np.float32(0.12345679))
    assert O.bf16_round(O.bf16_round(v)) == O.bf16_round(v)


def test_quantized_formats_are_validated_and_sized():
    # src/weights.rs:430-446
    assert O.row_bytes(16, 0, 896) == 1792
    assert O.row_bytes(8, 64, 896) == 896 + 14 * 2
    assert O.row_bytes(4, 32, 896) == 448 + 28 * 2
    O.validate_format(8, 64, [896, 4864])
    O.validate_format(4, 32, [896, 4864])
    for bits, group in [(6, 32), (8, 24), (8, 512), (8, 256)]:
        with pytest.raises(O.OracleError):
            O.validate_format(bits, group, [896, 4864])


def test_config_rejects_unsupported_architectures():
    # src/weights.rs:448-464
    c = O.config_parse(BASE_CFG)
    assert (c["head_dim"], c["heads"] // c["heads"] * c["kv_heads"] * c["head_dim"]) == (64, 128)
    assert c["bits"] == 16  # bf16
    for a, b in [('"qwen2"', '"llama"'), ('"silu"', '"gelu"'), ('"tie_word_embeddings":true', '"tie_word_embeddings":false'),
                 ('"num_key_value_heads":2', '"num_key_value_heads":5')]:
        with pytest.raises(O.OracleError):
            O.config_parse(BASE_CFG.replace(a, b))


def test_inject_quant_produces_a_config_that_parses_back():
    # src/quant.rs:375-397
    t = O.inject_quant(BASE_CFG, 4, 32)
    c = O.config_parse(t)
    assert (c["bits"], c["group"], c["embed_bits"], c["embed_group"]) == (4, 32, 4, 32)
    assert O.row_bytes(c["embed_bits"], c["embed_group"], c["hidden"]) == 448 + 56
    t2 = O.inject_quant(BASE_CFG, 4, 32, embed=(8, 64))
    c2 = O.config_parse(t2)
    assert (c2["bits"], c2["group"], c2["embed_bits"], c2["embed_group"]) == (4, 32, 8, 64)
    assert O.row_bytes(8, 64, 896) == 896 + 28
    with pytest.raises(O.OracleError):
        O.config_parse(O.inject_quant(BASE_CFG, 8, 256))
    with pytest.raises(O.OracleError):
        O.config_parse(t2.replace(',"embed_group":64', ""))


def test_greedy_picks_the_first_maximum():
    # src/model.rs:372-376 and src/spec.rs:41-49
    assert O.argmax(np.array([0.1, 3.0, 3.0, -1.0], np.float32)) == 1


def _bf16(vals):
    return (np.ascontiguousarray(vals, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _bf16_f32(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def test_dot_matches_a_double_precision_reference():
    # src/kernels.rs:285-296
    rng = Lcg(7)
    for n in [1, 7, 8, 9, 16, 17, 64, 896, 4864]:
        w = rng.many(n)
        x = rng.many(n)
        wb = _bf16(w)
        want = float(np.sum(_bf16_f32(wb).astype(np.float64) * x.astype(np.float64)))
        got = O.dot(16, 0, wb.view(np.uint8), x)
        assert abs(got - want) < 1e-4 * (1 + abs(want)), n


def test_matmul_single_and_batched_agree_and_match_naive():
    # src/kernels.rs:298-316
    rows, cols = 50, 40
    rng = Lcg(99)
    w = rng.many(rows * cols)
    wb = _bf16(w).view(np.uint8)
    wf = _bf16_f32(_bf16(w)).reshape(rows, cols).astype(np.float64)
    for t in [1, 2, 5]:
        x = rng.many(t * cols).reshape(t, cols)
        y = O.matmul(16, 0, wb, rows, cols, x)
        want = x.astype(np.float64) @ wf.T
        assert np.max(np.abs(y - want)) < 1e-4


def test_rms_norm_has_unit_rms_for_unit_weights():
    x = np.array([3.0, -4.0, 12.0, 0.5], np.float32)
    out = O.rms_norm_bf16(x, _bf16(np.ones(4, np.float32)), 0.0)
    assert abs(np.sqrt(np.mean(out.astype(np.float64) ** 2)) - 1.0) < 1e-5


def test_rope_at_position_zero_is_identity_and_preserves_norm():
    inv = np.array([np.float32(10000.0) ** np.float32(-(i / 4.0)) for i in range(4)], np.float32)
    v = np.arange(1, 9, dtype=np.float32)
    assert np.array_equal(O.rope(v, inv, 0), v)
    r = O.rope(v, inv, 37)
    assert abs(float(np.sum(v * v)) - float(np.sum(r * r))) < 1e-3


def test_softmax_sums_to_one_and_is_stable():
    v = O.softmax(np.array([1000.0, 1001.0, 999.0], np.float32))
    assert abs(float(v.sum()) - 1.0) < 1e-6
    assert v[1] > v[0] > v[2]


def _outlier_row(n, rng):
    return np.array([rng.next() * (np.float32(0.5) if i % 37 == 0 else np.float32(0.05)) for i in range(n)], np.float32)


def test_round_trip_error_is_bounded_by_half_a_step():
    # src/quant.rs:284-307
    rng = Lcg(5)
    for bits, group in [(8, 16), (8, 32), (8, 64), (4, 16), (4, 32), (4, 64)]:
        w = _outlier_row(256, rng)
        packed, _, _ = O.quantize_row(bits, group, w, False)
        back = O.dequant_row(bits, group, packed, 256)
        for g in range(256 // group):
            wg, bg = w[g * group:(g + 1) * group], back[g * group:(g + 1) * group]
            amax = float(np.max(np.abs(wg)))
            step = amax / (127.0 if bits == 8 else 7.0)
            assert np.all(np.abs(wg - bg) <= step * 0.52)
            big = wg[np.argmax(np.abs(wg))]
            assert abs(big - bg[np.argmax(np.abs(wg))]) <= amax * 0.01


def test_clip_search_never_does_worse_and_helps_four_bit():
    # src/quant.rs:309-325
    rng = Lcg(11)
    plain = clipped = 0.0
    for _ in range(40):
        w = _outlier_row(128, rng)
        _, ea, _ = O.quantize_row(4, 32, w, False)
        _, eb, _ = O.quantize_row(4, 32, w, True)
        assert eb <= ea * (1 + 1e-9)
        plain += ea
        clipped += eb
    assert clipped < plain * 0.97


def test_zero_and_tiny_rows_do_not_produce_nan():
    # src/quant.rs:327-343
    for bits, group in [(8, 32), (4, 32)]:
        for w in [np.zeros(64, np.float32), np.full(64, 1e-45, np.float32), np.full(64, -3.0, np.float32)]:
            p, _, _ = O.quantize_row(bits, group, w, True)
            assert np.all(np.isfinite(O.dequant_row(bits, group, p, 64)))
    p, _, _ = O.quantize_row(8, 32, np.zeros(32, np.float32), True)
    assert np.all(O.dequant_row(8, 32, p, 32) == 0.0)


def test_quantized_matmul_equals_a_matmul_over_the_dequantized_weights():
    # src/quant.rs:345-373
    rng = Lcg(21)
    for bits, group in [(8, 32), (8, 64), (4, 32), (4, 64)]:
        rows, cols = 37, 128
        rb = O.row_bytes(bits, group, cols)
        packed = np.zeros(rows * rb, np.uint8)
        deq = np.zeros((rows, cols), np.float64)
        for r in range(rows):
            p, _, _ = O.quantize_row(bits, group, _outlier_row(cols, rng), True)
            packed[r * rb:(r + 1) * rb] = p
            deq[r] = O.dequant_row(bits, group, p, cols)
        for t in [1, 3]:
            x = rng.many(t * cols).reshape(t, cols)
            y = O.matmul(bits, group, packed, rows, cols, x)
            want = x.astype(np.float64) @ deq.T
            assert np.all(np.abs(y - want) < 1e-4 * (1 + np.abs(want)))


def test_quantize_group_known_answer():
    # Hand-computed: amax = 1.0, int8 clip 1.0 -> s = bf16(1/127) = 0.00787353515625;
    # q = round(v / s) clamped.
    w = np.array([1.0, -0.5, 0.25, 0.0] + [0.0] * 12, np.float32)
    p, _, _ = O.quantize_row(8, 16, w, False)
    s = np.frombuffer(p[16:18].tobytes(), "<u2")[0]
    assert float(_bf16_f32(np.array([s], np.uint16))[0]) == 0.00787353515625
    inv = np.float32(1.0) / np.float32(0.00787353515625)
    assert list(p[:4].view(np.int8)) == [127, int(np.round(np.float32(-0.5) * inv)), 32, 0]
    # int4 nibble order: byte j = (w_j + 8) | (w_{j+half} + 8) << 4
    w4 = np.zeros(16, np.float32)
    w4[0], w4[8] = 7 * 0.125, -7 * 0.125
    p4, _, _ = O.quantize_row(4, 16, w4, False)
    assert p4[0] == (7 + 8) | ((-7 + 8) << 4)
