"""ChaCha20-Poly1305 on the GPU (the cipher of sealed model files, src/seal.rs:340-400) against the
reference's golden vectors and the pinned oracle (Python's `cryptography`, tests/test_seal_oracle.py);
needs a B200.

Covered as the reference's own cipher tests cover it (src/seal.rs test module): the RFC 8439
vector, 23 message lengths from 0 to 65537 with associated data of len % 13 bytes, a round trip,
and rejection of any single modified byte, tag, key, nonce or associated data with the data left
untouched; beyond them, the sealed file's per-chunk messages (nonce prefix || chunk index, the
chunk index appended to the associated data) at chunk sizes that do and do not divide the data, and
multi-MiB inputs that span many MAC segments.
"""

import struct

import numpy as np
import pytest
from cryptography.hazmat.primitives.ciphers.aead import ChaCha20Poly1305

import layerstream_b200 as ls
import seal_vectors as SV

pytestmark = pytest.mark.gpu


def test_gpu_cipher_matches_the_rfc_aead_vector():
    v = SV.VECTORS["aead_2_8_2"]
    key, nonce, aad = bytes.fromhex(v["key"]), bytes.fromhex(v["nonce"]), bytes.fromhex(v["aad"])
    ct, tags, _ = ls.aead_seal(key, nonce, aad, v["plaintext"].encode())
    assert ct[:16].hex() == v["ciphertext_first16"]
    assert tags[0].hex() == v["tag"]
    assert ls.aead_open(key, nonce, aad, ct, tags) == v["plaintext"].encode()


def test_gpu_cipher_matches_the_golden_tags_for_many_lengths():
    oracle = ChaCha20Poly1305(SV.KEY)
    for n, tag in SV.VECTORS["many_lengths"]:
        pt, aad = SV.plaintext(n), SV.aad(n)
        ct, tags, _ = ls.aead_seal(SV.KEY, SV.NONCE, aad, pt)
        assert tags[0].hex() == tag, n
        assert ct + tags[0] == oracle.encrypt(SV.NONCE, pt, aad), n
        assert ls.aead_open(SV.KEY, SV.NONCE, aad, ct, tags) == pt, n


def test_any_modification_is_rejected_and_nothing_is_decrypted():
    key, nonce, aad = bytes([7] * 32), bytes([9] * 12), b"hdr"
    pt = bytes(i & 0xFF for i in range(700))
    ct, tags, _ = ls.aead_seal(key, nonce, aad, pt)
    for pos in list(range(0, len(ct), 37)) + [len(ct) - 1]:
        bad = bytearray(ct)
        bad[pos] ^= 1
        with pytest.raises(ls.LayerstreamError) as e:
            ls.aead_open(key, nonce, aad, bytes(bad), tags)
        assert e.value.code == -2 and "authentication failed" in str(e.value), pos
    bad_tag = bytearray(tags[0])
    bad_tag[0] ^= 1
    for args in [(key, nonce, aad, ct, [bytes(bad_tag)]), (bytes([8] * 32), nonce, aad, ct, tags),
                 (key, bytes([1] * 12), aad, ct, tags), (key, nonce, b"other", ct, tags)]:
        with pytest.raises(ls.LayerstreamError):
            ls.aead_open(*args)


def test_a_failed_open_leaves_the_data_as_it_was():
    # the library decrypts only chunks whose tag matched: a chunk that fails keeps its ciphertext
    key, prefix, aad = bytes(range(32)), b"abcdefgh" + bytes(4), b"frame+header"
    pt = np.random.default_rng(3).integers(0, 256, 5000, np.uint8).tobytes()
    ct, tags, _ = ls.aead_seal(key, prefix, aad, pt, chunk_bytes=1024)
    bad = bytearray(ct)
    bad[2 * 1024 + 5] ^= 0x80  # chunk 2
    buf = np.frombuffer(bytes(bad), np.uint8).copy()
    t = np.frombuffer(b"".join(tags), np.uint8).copy()
    import ctypes as C
    ms, which = C.c_double(), C.c_int64()
    k, n, a = (np.frombuffer(x, np.uint8).copy() for x in (key, prefix, aad))
    rc = ls.lib().ls_aead_host(0, ls._p(k), ls._p(n), ls._p(a), len(aad), ls._p(buf), len(pt), 1024, 0, ls._p(t), 1,
                               C.byref(ms), C.byref(which))
    assert rc == -2 and which.value == 2
    assert buf[2 * 1024:3 * 1024].tobytes() == bytes(bad[2 * 1024:3 * 1024])  # untouched
    assert buf[:2 * 1024].tobytes() == pt[:2 * 1024]  # the chunks that verified are plaintext


@pytest.mark.parametrize("length,chunk,first", [(1 << 20, 1 << 16, 0), (3 * (1 << 20) + 17, 1 << 20, 5),
                                                (100_000, 7 * 64 + 3, 40_000), (4096, 4096, 9)])
def test_sealed_file_chunks_match_the_oracle(length, chunk, first):
    # chunk i: nonce = prefix || le32(first + i), associated data = aad || le32(first + i)
    key = bytes((3 * i + 1) & 0xFF for i in range(32))
    prefix = b"\x01\x02\x03\x04\x05\x06\x07\x08"
    aad = b"LSS1" + bytes(range(200))
    pt = np.random.default_rng(length).integers(0, 256, length, np.uint8).tobytes()
    ct, tags, _ = ls.aead_seal(key, prefix + bytes(4), aad, pt, chunk_bytes=chunk, first=first)
    oracle = ChaCha20Poly1305(key)
    n = -(-length // chunk)
    assert len(tags) == n
    for i in range(n):
        idx = struct.pack("<I", first + i)
        want = oracle.encrypt(prefix + idx, pt[i * chunk:(i + 1) * chunk], aad + idx)
        assert ct[i * chunk:(i + 1) * chunk] + tags[i] == want, i
    assert ls.aead_open(key, prefix + bytes(4), aad, ct, tags, chunk_bytes=chunk, first=first) == pt
    # chunks cannot be moved: the same bytes under another index fail
    with pytest.raises(ls.LayerstreamError):
        ls.aead_open(key, prefix + bytes(4), aad, ct, tags, chunk_bytes=chunk, first=first + 1)
