"""Tiny synthetic Qwen2-shaped models written to disk, as the reference's own test fixture does.

Port of the reference's ``tests/common/mod.rs``: the same LCG (constants 6364136223846793005 /
1442695040888963407, values ``((s >> 33) / 2^31) * 2 - 1`` in f32), the same shapes
(hidden 64, 4 heads, 2 KV heads, FFN 128, 3 layers, vocab 600), the same value recipes
(0.15 * U for matrices and biases, 1 + 0.1 * U for norm gains), the same bf16 truncation and the
same tensor order, plus the "grid model" whose weights sit exactly on a quantization grid
(``tests/common/mod.rs:44-62``).
"""

from __future__ import annotations

import json
import os
import shutil
import struct
import tempfile

import numpy as np

HIDDEN, HEADS, KV_HEADS, INTER, LAYERS, VOCAB = 64, 4, 2, 128, 3, 600

_A = 6364136223846793005
_B = 1442695040888963407
_MASK = (1 << 64) - 1
_TWO31 = np.float32(2.0**31)


class Lcg:
    def __init__(self, seed: int):
        self.s = seed & _MASK

    def next(self) -> np.float32:
        self.s = (self.s * _A + _B) & _MASK
        return np.float32(np.float32(self.s >> 33) / _TWO31) * np.float32(2.0) - np.float32(1.0)

    def many(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        s = self.s
        vals = []
        for _ in range(n):
            s = (s * _A + _B) & _MASK
            vals.append(s >> 33)
        self.s = s
        out[:] = np.array(vals, dtype=np.float64).astype(np.float32)
        return (out / _TWO31) * np.float32(2.0) - np.float32(1.0)


def bf16_trunc_bytes(vals: np.ndarray) -> bytes:
    """``(v.to_bits() >> 16) as u16`` little-endian, as tests/common/mod.rs:26-28."""
    u = np.ascontiguousarray(vals, dtype=np.float32).view(np.uint32) >> 16
    return u.astype("<u2").tobytes()


def tensor_list(hidden=HIDDEN, heads=HEADS, kv_heads=KV_HEADS, inter=INTER, layers=LAYERS, vocab=VOCAB):
    kv = kv_heads * (hidden // heads)
    t = [("model.embed_tokens.weight", [vocab, hidden])]
    for l in range(layers):
        p = f"model.layers.{l}"
        for suffix, shape in [
            ("input_layernorm.weight", [hidden]),
            ("mlp.down_proj.weight", [hidden, inter]),
            ("mlp.gate_proj.weight", [inter, hidden]),
            ("mlp.up_proj.weight", [inter, hidden]),
            ("post_attention_layernorm.weight", [hidden]),
            ("self_attn.k_proj.bias", [kv]),
            ("self_attn.k_proj.weight", [kv, hidden]),
            ("self_attn.o_proj.weight", [hidden, hidden]),
            ("self_attn.q_proj.bias", [hidden]),
            ("self_attn.q_proj.weight", [hidden, hidden]),
            ("self_attn.v_proj.bias", [kv]),
            ("self_attn.v_proj.weight", [kv, hidden]),
        ]:
            t.append((f"{p}.{suffix}", shape))
    t.append(("model.norm.weight", [hidden]))
    return t


def write_safetensors(path: str, named_bytes) -> None:
    """Write BF16 tensors in the given order (``[(name, shape, bytes)]``)."""
    entries, off = [], 0
    for name, shape, b in named_bytes:
        dims = ",".join(str(d) for d in shape)
        entries.append(f'"{name}":{{"dtype":"BF16","shape":[{dims}],"data_offsets":[{off},{off + len(b)}]}}')
        off += len(b)
    header = '{"__metadata__":{"format":"pt"},' + ",".join(entries) + "}"
    while len(header) % 8:
        header += " "
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header)))
        f.write(header.encode())
        for _, _, b in named_bytes:
            f.write(b)


def _grid_values(rng: Lcg, rows: int, cols: int, bits: int, group: int) -> np.ndarray:
    """tests/common/mod.rs:47-62: codes * 2^-k with the largest code of every group at qmax."""
    qmax, scale = (127, np.float32(2.0**-10)) if bits == 8 else (7, np.float32(2.0**-6))
    out = np.empty(rows * cols, dtype=np.float32)
    i = 0
    half_span = np.float32(qmax + 0.5)
    for _ in range(rows):
        for g in range(cols // group):
            for j in range(group):
                v = rng.next() * half_span
                # Rust f32::round is half away from zero
                fv = float(v)  # exact in double: floor(|v| + 0.5) is round-half-away
                code = int(np.floor(abs(fv) + 0.5)) * (1 if fv >= 0 else -1)
                code = max(-qmax, min(qmax, code))
                if j == (g * 7) % group:
                    code = -qmax if rng.next() < 0 else qmax
                out[i] = np.float32(code) * scale
                i += 1
    return out


def config_text(hidden=HIDDEN, heads=HEADS, kv_heads=KV_HEADS, inter=INTER, layers=LAYERS, vocab=VOCAB,
                rope_theta="10000.0", max_pos=512) -> str:
    return (
        '{"model_type":"qwen2","hidden_act":"silu","tie_word_embeddings":true,'
        f'"hidden_size":{hidden},\n"num_attention_heads":{heads},"num_key_value_heads":{kv_heads},'
        f'"intermediate_size":{inter},\n"num_hidden_layers":{layers},"vocab_size":{vocab},"rms_norm_eps":1e-6,'
        f'"rope_theta":{rope_theta},\n"max_position_embeddings":{max_pos}}}'
    )


def write_model(d: str, seed: int, grid=None) -> str:
    """tests/common/mod.rs:74-135. ``grid`` = ((body_bits, body_group), (embed_bits, embed_group))."""
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "config.json"), "w") as f:
        f.write(config_text())
    rng = Lcg(seed)
    out = []
    for name, shape in tensor_list():
        n = int(np.prod(shape))
        is_norm = name.endswith("layernorm.weight") or name == "model.norm.weight"
        if is_norm:
            vals = np.float32(1.0) + np.float32(0.1) * rng.many(n)
        elif grid is not None and len(shape) == 2:
            bits, group = grid[1] if name == "model.embed_tokens.weight" else grid[0]
            vals = _grid_values(rng, shape[0], shape[1], bits, group)
        else:
            vals = np.float32(0.15) * rng.many(n)
        out.append((name, shape, bf16_trunc_bytes(vals)))
    write_safetensors(os.path.join(d, "model.safetensors"), out)
    return d


def write_tiny_model(d: str, seed: int) -> str:
    return write_model(d, seed)


def write_tiny_grid_model(d: str, seed: int, body, embed) -> str:
    return write_model(d, seed, grid=(body, embed))


class TempDir:
    def __init__(self, tag: str):
        self.path = tempfile.mkdtemp(prefix=f"ls-b200-{tag}-")

    def __enter__(self):
        return self.path

    def __exit__(self, *a):
        shutil.rmtree(self.path, ignore_errors=True)


PROMPT = [5, 17, 301, 42, 599, 0]
OTHER_PROMPT = [250, 3, 77]
FOLLOW = [7, 33, 120]
