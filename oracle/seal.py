"""Test infrastructure, not product code: a CPU restatement of the reference's sealed-file writer and
reader (src/seal.rs: file layout 13-27, SealedLayout::to_json 574-591, seal_model 726-827,
SealedSource::open 860-903 and its chunk opening 958-1030), with the ChaCha20-Poly1305 of Python's
`cryptography` package (pinned to the reference's own cipher vectors in tests/test_seal_oracle.py).
The tests use it to check the library's GPU sealer byte for byte and to open files independently.
"""

from __future__ import annotations

import json
import os
import struct

from cryptography.hazmat.primitives.ciphers.aead import ChaCha20Poly1305

from oracle import oracle as O

FRAME = 20
TAG = 16


def json_string(s: str) -> str:
    """src/seal.rs:646-664 (the reference's escaping: quote, backslash, \\n \\r \\t, other controls as
    \\u00XX, everything else as is)."""
    out = ['"']
    for c in s:
        if c == '"':
            out.append('\\"')
        elif c == "\\":
            out.append("\\\\")
        elif c == "\n":
            out.append("\\n")
        elif c == "\r":
            out.append("\\r")
        elif c == "\t":
            out.append("\\t")
        elif ord(c) < 0x20:
            out.append("\\u%04x" % ord(c))
        else:
            out.append(c)
    out.append('"')
    return "".join(out)


def source(path: str) -> dict:
    """The plaintext a sealed file carries (src/seal.rs:783-812): config text, the layer layout (12
    slot ranges), each layer block's file offset, the embedding table and the final norm."""
    quantized = not os.path.isdir(path)
    f = O.open_files(path, quantized)
    if quantized:
        with open(path, "rb") as fh:
            hl = struct.unpack("<I", fh.read(8)[4:8])[0]
            cfg_text = json.loads(fh.read(hl))["config_json"]
        data_path = path
        layers = json.loads(cfg_text)["num_hidden_layers"]
        data_start = f["embed_start"] - layers * f["total"]
        starts = [data_start + l * f["total"] for l in range(layers)]
    else:
        cfg_text = open(os.path.join(path, "config.json")).read()
        data_path = os.path.join(path, "model.safetensors")
        with open(data_path, "rb") as fh:
            n = struct.unpack("<Q", fh.read(8))[0]
            hdr = json.loads(fh.read(n))
        layers = json.loads(cfg_text)["num_hidden_layers"]
        starts = []
        for l in range(layers):
            pre = f"model.layers.{l}."
            starts.append(8 + n + min(v["data_offsets"][0] for k, v in hdr.items() if k.startswith(pre)))
    cfg = json.loads(cfg_text)
    q = cfg.get("layerstream_quant")
    h = cfg["hidden_size"]
    rb = O.row_bytes(q.get("embed_bits", q["bits"]), q.get("embed_group", q["group"]), h) if q else 2 * h
    return {"config_text": cfg_text, "path": data_path, "layout": list(zip(f["off"], f["len"])), "layer_bytes": f["total"],
            "starts": starts, "embed_start": f["embed_start"], "embed_bytes": cfg["vocab_size"] * rb, "row_bytes": rb,
            "norm_start": f["norm_start"], "norm_bytes": 2 * h}


def seal_model(src: str, out: str, key: bytes, prefix: bytes, layer_chunk: int = 1 << 20, embed_chunk_rows: int = 512):
    """seal_model (src/seal.rs:726-827) on the CPU; returns the number of chunks."""
    s = source(src)
    cfg = json.loads(s["config_text"])
    hidden, vocab = cfg["hidden_size"], cfg["vocab_size"]
    norm_bytes = hidden * 2
    rb = s["row_bytes"]
    ranges = ",".join(f"[{o},{n}]" for o, n in s["layout"])
    header = ('{"format":"layerstream-sealed-1","config_json":' + json_string(s["config_text"]) +
              f',"layer_bytes":{s["layer_bytes"]},"layer_chunk":{layer_chunk},"embed_chunk_rows":{embed_chunk_rows}'
              f',"final_norm_bytes":{norm_bytes},"layer_layout":[{ranges}]}}').encode()
    frame = b"LSS1" + struct.pack("<I", 1) + prefix + struct.pack("<I", len(header)) + header
    aead = ChaCha20Poly1305(key)
    tags, body = [], []

    def seal(data: bytes, first: int, clen: int):
        for i in range(0, max(len(data), 1), clen):
            idx = struct.pack("<I", first + i // clen)
            ct = aead.encrypt(prefix + idx, data[i:i + clen], frame + idx)
            body.append(ct[:-TAG])
            tags.append(ct[-TAG:])

    with open(s["path"], "rb") as fh:
        def read(off, n):
            fh.seek(off)
            return fh.read(n)
        lc = -(-s["layer_bytes"] // layer_chunk)
        for l, st in enumerate(s["starts"]):
            seal(read(st, s["layer_bytes"]), l * lc, layer_chunk)
        first = len(s["starts"]) * lc
        for r in range(0, vocab, embed_chunk_rows):
            rows = min(embed_chunk_rows, vocab - r)
            seal(read(s["embed_start"] + r * rb, rows * rb), first + r // embed_chunk_rows, rows * rb)
        seal(read(s["norm_start"], norm_bytes), len(tags), norm_bytes)
    with open(out, "xb") as fo:
        fo.write(frame + b"".join(tags) + b"".join(body))
    return len(tags)


def open_sealed(path: str, key: bytes) -> dict:
    """SealedSource::open + reading every chunk: the header and the whole plaintext (raises on a
    failed tag)."""
    data = open(path, "rb").read()
    if data[:4] != b"LSS1":
        raise ValueError("not a sealed layerstream model (bad magic bytes)")
    prefix = data[8:16]
    hl = struct.unpack("<I", data[16:20])[0]
    frame = data[:FRAME + hl]
    hdr = json.loads(data[FRAME:FRAME + hl])
    cfg = json.loads(hdr["config_json"])
    lb, lc_bytes, ecr = hdr["layer_bytes"], hdr["layer_chunk"], hdr["embed_chunk_rows"]
    layers, vocab = cfg["num_hidden_layers"], cfg["vocab_size"]
    lc = -(-lb // lc_bytes)
    n_chunks = layers * lc + -(-vocab // ecr) + 1
    tags = data[FRAME + hl:FRAME + hl + TAG * n_chunks]
    ct = data[FRAME + hl + TAG * n_chunks:]
    total = len(ct)
    embed_bytes = total - layers * lb - hdr["final_norm_bytes"]
    rb = embed_bytes // vocab
    aead = ChaCha20Poly1305(key)
    out, pos, idx = [], 0, 0

    def take(n):
        nonlocal pos, idx
        c = struct.pack("<I", idx)
        out.append(aead.decrypt(prefix + c, ct[pos:pos + n] + tags[TAG * idx:TAG * idx + TAG], frame + c))
        pos += n
        idx += 1

    for _ in range(layers):
        for i in range(0, lb, lc_bytes):
            take(min(lc_bytes, lb - i))
    for r in range(0, vocab, ecr):
        take(min(ecr, vocab - r) * rb)
    take(hdr["final_norm_bytes"])
    return {"header": hdr, "plain": b"".join(out)}
