"""Writes seal_vectors.json: the golden vectors of the reference's cipher tests, read as text from
its source (src/seal.rs, test module: chacha20_block_matches_rfc8439, aead_matches_rfc8439_section_2_8_2,
matches_python_for_many_lengths). Run where the reference tree is present:

    python tests/golden/make_seal_vectors.py /path/to/reference

The message, key, nonce and associated-data patterns of the many-lengths vectors are restated in
tests/seal_vectors.py (they are formulas, not data); only the expected tags come from the file.
"""

import json
import os
import re
import sys


def main(ref: str):
    src = open(os.path.join(ref, "src", "seal.rs")).read()
    tests = src[src.index("fn chacha20_block_matches_rfc8439"):]
    out = {"source": "src/seal.rs test module"}
    # RFC 8439 2.3.2: keystream block 1 of key 00..1f, nonce 000000090000004a00000000
    m = re.search(r'unhex\(\s*"([0-9a-f]+)\\\s*\n\s*([0-9a-f]+)"\s*\)', tests)
    out["chacha_block1"] = {"key": "".join(f"{i:02x}" for i in range(32)), "nonce": "000000090000004a00000000",
                            "counter": 1, "keystream": m.group(1) + m.group(2)}
    # RFC 8439 2.8.2 AEAD
    a = tests[tests.index("fn aead_matches_rfc8439_section_2_8_2"):]
    nonce = re.search(r'let nonce: \[u8; 12\] = unhex\("([0-9a-f]+)"\)', a).group(1)
    aad = re.search(r'let aad = unhex\("([0-9a-f]+)"\)', a).group(1)
    pt = re.search(r'let pt = b"([^"]+)";', a).group(1)
    ct16 = re.search(r'&unhex\("([0-9a-f]+)"\)\[\.\.\]', a).group(1)
    tag = re.search(r'tag\.to_vec\(\), unhex\("([0-9a-f]+)"\)', a).group(1)
    out["aead_2_8_2"] = {"key": "".join(f"{0x80 + i:02x}" for i in range(32)), "nonce": nonce, "aad": aad,
                         "plaintext": pt, "ciphertext_first16": ct16, "tag": tag}
    # many lengths: (len, tag)
    b = tests[tests.index("fn matches_python_for_many_lengths"):]
    b = b[:b.index("];")]
    out["many_lengths"] = [[int(n), t] for n, t in re.findall(r'\((\d+), "([0-9a-f]{32})"\)', b)]
    here = os.path.dirname(os.path.abspath(__file__))
    with open(os.path.join(here, "seal_vectors.json"), "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print(f"{len(out['many_lengths'])} length vectors")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_seal_vectors.py <reference source tree>")
    main(sys.argv[1])
