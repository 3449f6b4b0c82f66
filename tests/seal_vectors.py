"""The reference's cipher test vectors (tests/golden/seal_vectors.json, read from src/seal.rs's
test module) and the formulas of its many-lengths case (src/seal.rs, matches_python_for_many_lengths):
key byte i = 7i + 3, nonce byte i = 11i + 5, plaintext byte i = 31i + 7 + 3(i >> 8), associated
data of length len % 13 with byte i = 5i + 1 (all mod 256)."""

import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))
VECTORS = json.load(open(os.path.join(HERE, "golden", "seal_vectors.json")))

KEY = bytes((i * 7 + 3) & 0xFF for i in range(32))
NONCE = bytes((i * 11 + 5) & 0xFF for i in range(12))


def plaintext(n: int) -> bytes:
    return bytes((i * 31 + 7 + (i >> 8) * 3) & 0xFF for i in range(n))


def aad(n: int) -> bytes:
    return bytes((i * 5 + 1) & 0xFF for i in range(n % 13))
