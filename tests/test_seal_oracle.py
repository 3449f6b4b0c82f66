"""The cipher oracle pinned to the reference's golden vectors (no GPU): Python's `cryptography`
ChaCha20-Poly1305 (the package the reference's own tests were checked against, src/seal.rs:4-6)
reproduces every vector of src/seal.rs's test module, so it can stand in as the oracle of the GPU
cipher for inputs the vectors do not cover."""

import struct

from cryptography.hazmat.primitives.ciphers import Cipher, algorithms
from cryptography.hazmat.primitives.ciphers.aead import ChaCha20Poly1305

import seal_vectors as SV


def test_oracle_reproduces_the_rfc_keystream_block():
    v = SV.VECTORS["chacha_block1"]
    nonce16 = struct.pack("<I", v["counter"]) + bytes.fromhex(v["nonce"])
    enc = Cipher(algorithms.ChaCha20(bytes.fromhex(v["key"]), nonce16), mode=None).encryptor()
    assert enc.update(bytes(64)).hex() == v["keystream"]


def test_oracle_reproduces_the_rfc_aead_vector():
    v = SV.VECTORS["aead_2_8_2"]
    out = ChaCha20Poly1305(bytes.fromhex(v["key"])).encrypt(bytes.fromhex(v["nonce"]), v["plaintext"].encode(),
                                                           bytes.fromhex(v["aad"]))
    assert out[:16].hex() == v["ciphertext_first16"]
    assert out[-16:].hex() == v["tag"]


def test_oracle_reproduces_the_tags_for_many_lengths():
    aead = ChaCha20Poly1305(SV.KEY)
    assert len(SV.VECTORS["many_lengths"]) == 23
    for n, tag in SV.VECTORS["many_lengths"]:
        out = aead.encrypt(SV.NONCE, SV.plaintext(n), SV.aad(n))
        assert out[-16:].hex() == tag, n


def test_oracle_sealed_file_opens_to_the_source_bytes_and_refuses_changes(tmp_path):
    # the CPU restatement of the sealed format (oracle/seal.py) round-trips a quantized and a bf16
    # model, and a wrong key or a swapped pair of layer chunks fails (tests/pipeline.rs:61-166)
    import os

    import pytest

    import fixtures as F
    from oracle import oracle as O
    from oracle import seal as OS

    d = str(tmp_path)
    F.write_tiny_model(d, 1)
    lsq = os.path.join(d, "m.lsq")
    O.quantize_model(d, lsq, (4, 32), (4, 32), clip=True)
    for src in [lsq, d]:
        out = os.path.join(d, "m.sealed" if src == lsq else "b.sealed")
        n = OS.seal_model(src, out, bytes([7] * 32), b"abcdefgh", 1500, 64)
        s = OS.source(src)
        raw = open(s["path"], "rb").read()
        want = b"".join(raw[st:st + s["layer_bytes"]] for st in s["starts"])
        want += raw[s["embed_start"]:s["embed_start"] + s["embed_bytes"]] + raw[s["norm_start"]:s["norm_start"] + s["norm_bytes"]]
        got = OS.open_sealed(out, bytes([7] * 32))
        assert got["plain"] == want and got["header"]["layer_chunk"] == 1500
        assert os.path.getsize(out) == 20 + int.from_bytes(open(out, "rb").read()[16:20], "little") + 16 * n + len(want)
        with pytest.raises(Exception):
            OS.open_sealed(out, bytes([8] * 32))
    # swapped layer blocks (equal sizes) do not authenticate
    buf = bytearray(open(os.path.join(d, "m.sealed"), "rb").read())
    s = OS.source(lsq)
    lb = s["layer_bytes"]
    base = len(buf) - (len(s["starts"]) * lb + s["embed_bytes"] + s["norm_bytes"])
    buf[base:base + lb], buf[base + lb:base + 2 * lb] = buf[base + lb:base + 2 * lb], buf[base:base + lb]
    open(os.path.join(d, "s.sealed"), "wb").write(bytes(buf))
    with pytest.raises(Exception):
        OS.open_sealed(os.path.join(d, "s.sealed"), bytes([7] * 32))
