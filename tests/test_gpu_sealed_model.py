"""Sealed model files on the GPU (src/seal.rs: SealedSource with the resident and streaming
providers) against the plain files and the CPU restatement of the sealed format (oracle/seal.py);
needs a B200.

Mirrors the reference's pipeline tests (tests/pipeline.rs:61-168): the sealed file decrypts to
exactly the original weights (here: the GPU sealer writes the same bytes as the CPU restatement,
and the CPU opens them back to the source's plaintext), every mode gives bit-identical logits,
a wrong key is refused at open, a flipped bit in a layer fails the load (resident) or the pass that
streams the layer, a changed header, tag, truncation or magic is refused, and swapped chunks do not
authenticate.
"""

import os

import numpy as np
import pytest

import fixtures as F
import layerstream_b200 as ls
from oracle import oracle as O
from oracle import seal as OS

pytestmark = pytest.mark.gpu

SMALL = (1500, 64)  # layer_chunk bytes, embed_chunk_rows (tests/pipeline.rs:25)
PREFIX = b"abcdefgh"


def key(n):
    return bytes([n] * 32)


@pytest.fixture(scope="module")
def models():
    d = F.TempDir("gpu-sealed").path
    F.write_tiny_model(d, 2)
    out = {"bf16": d}
    for body in [(8, 32), (4, 32)]:
        p = os.path.join(d, f"q{body[0]}g{body[1]}.lsq")
        O.quantize_model(d, p, body, body, clip=True)
        out[body] = p
    out["dir"] = d
    return out


def run(m):
    """tests/pipeline.rs:46-56: the prompt's logits, then three greedy steps' logits."""
    logits = [m.forward(F.PROMPT)]
    for _ in range(3):
        logits.append(m.forward([int(np.argmax(logits[-1]))]))
    return np.stack(logits)


def seal(models, src, name, k, params=SMALL):
    p = os.path.join(models["dir"], name)
    if os.path.exists(p):
        os.remove(p)
    ls.seal_model(src, p, k, PREFIX, *params)
    return p


@pytest.mark.parametrize("src", [(8, 32), (4, 32), "bf16"])
@pytest.mark.parametrize("params", [SMALL, (1 << 20, 512), (64, 7)])
def test_the_gpu_sealer_writes_the_reference_format_byte_for_byte(models, src, params):
    p = seal(models, models[src], "gpu.sealed", key(7), params)
    q = os.path.join(models["dir"], "cpu.sealed")
    if os.path.exists(q):
        os.remove(q)
    OS.seal_model(models[src], q, key(7), PREFIX, *params)
    assert open(p, "rb").read() == open(q, "rb").read()
    # and the CPU opens it back to the source's plaintext (sealed_file_decrypts_to_exactly_the_original_weights)
    s = OS.source(models[src])
    raw = open(s["path"], "rb").read()
    want = b"".join(raw[st:st + s["layer_bytes"]] for st in s["starts"])
    want += raw[s["embed_start"]:s["embed_start"] + s["embed_bytes"]] + raw[s["norm_start"]:s["norm_start"] + s["norm_bytes"]]
    assert OS.open_sealed(p, key(7))["plain"] == want


@pytest.mark.parametrize("body", [(8, 32), (4, 32)])
def test_every_mode_produces_bit_identical_logits(models, body):
    p = seal(models, models[body], f"modes{body[0]}.sealed", key(9))
    reference = run(ls.Model(models[body], max_ctx=64))
    assert np.all(np.isfinite(reference))
    np.testing.assert_array_equal(run(ls.Model(p, max_ctx=64, key=key(9))), reference)
    # streaming runs the separate kernels (the resident pass kernel sums in another order): the
    # sealed stream must equal the plain stream bit for bit
    for slots in [1, 2]:
        plain = run(ls.Model(models[body], max_ctx=64, mode="stream", slots=slots))
        np.testing.assert_allclose(plain, reference, atol=2e-2)
        np.testing.assert_array_equal(run(ls.Model(p, max_ctx=64, mode="stream", slots=slots, key=key(9))), plain)


def test_a_sealed_bf16_model_runs_resident_like_the_plain_one(models):
    p = seal(models, models["bf16"], "bf16.sealed", key(3))
    np.testing.assert_array_equal(run(ls.Model(p, max_ctx=64, key=key(3))), run(ls.Model(models["bf16"], max_ctx=64)))


def test_speculative_decoding_over_a_sealed_stream_matches_the_plain_model(models):
    p = seal(models, models[(4, 32)], "spec.sealed", key(4))
    want, _ = ls.speculative_greedy(ls.Model(models[(4, 32)], max_ctx=96), None, F.PROMPT, 24, 4)
    got, _ = ls.speculative_greedy(ls.Model(p, max_ctx=96, mode="stream", slots=2, key=key(4)), None, F.PROMPT, 24, 4)
    assert got == want


def test_wrong_key_and_tampering_are_rejected(models):
    p = seal(models, models[(8, 32)], "tamper.sealed", key(1))
    with pytest.raises(ls.LayerstreamError) as e:
        ls.Model(p, max_ctx=64, key=key(2))
    assert e.value.code == -2 and "authentication failed" in str(e.value)
    good = open(p, "rb").read()
    total = len(good)

    def flip(pos, name):
        bad = bytearray(good)
        bad[pos] ^= 1
        q = os.path.join(models["dir"], name)
        open(q, "wb").write(bytes(bad))
        return q

    # a flipped bit inside a layer: the file opens for streaming (only the final norm is checked
    # up front) but the pass that streams the layer fails; a resident load fails
    mid = flip(total // 3, "bad-ct.sealed")
    with pytest.raises(ls.LayerstreamError) as e:
        ls.Model(mid, max_ctx=64, key=key(1))
    assert "authentication failed" in str(e.value)
    m = ls.Model(mid, max_ctx=64, mode="stream", slots=2, key=key(1))
    with pytest.raises(ls.LayerstreamError) as e:
        m.forward(F.PROMPT)
    assert e.value.code == -2 and "authentication failed" in str(e.value)
    # a flipped bit in the header: refused; in the tag table: detected at load
    with pytest.raises(ls.LayerstreamError):
        ls.Model(flip(30, "bad-header.sealed"), max_ctx=64, key=key(1))
    tag_pos = 20 + int.from_bytes(good[16:20], "little") + 5
    with pytest.raises(ls.LayerstreamError):
        ls.Model(flip(tag_pos, "bad-tag.sealed"), max_ctx=64, key=key(1))
    # truncated, wrong magic
    short = os.path.join(models["dir"], "short.sealed")
    open(short, "wb").write(good[:-1])
    with pytest.raises(ls.LayerstreamError):
        ls.Model(short, max_ctx=64, key=key(1))
    with pytest.raises(ls.LayerstreamError):
        ls.Model(flip(0, "magic.sealed"), max_ctx=64, key=key(1))
    # a plain file with a key, a sealed file without one
    with pytest.raises(ls.LayerstreamError):
        ls.Model(models[(8, 32)], max_ctx=64, key=key(1))
    with pytest.raises(ls.LayerstreamError):
        ls.Model(p, max_ctx=64)


def test_chunks_cannot_be_swapped(models):
    # layers have identical sizes, so swapping two layers' ciphertext gives a valid-looking file;
    # the per-chunk nonce and associated data make it fail (tests/pipeline.rs:142-166)
    p = seal(models, models[(4, 32)], "swap.sealed", key(5), (1 << 20, 64))
    good = bytearray(open(p, "rb").read())
    s = OS.open_sealed(p, key(5))
    lb = s["header"]["layer_bytes"]
    ct_base = len(good) - len(s["plain"])
    a, b = good[ct_base:ct_base + lb], good[ct_base + lb:ct_base + 2 * lb]
    good[ct_base:ct_base + lb], good[ct_base + lb:ct_base + 2 * lb] = b, a
    q = os.path.join(models["dir"], "swapped.sealed")
    open(q, "wb").write(bytes(good))
    with pytest.raises(ls.LayerstreamError):
        ls.Model(q, max_ctx=64, key=key(5))
