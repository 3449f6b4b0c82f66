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
