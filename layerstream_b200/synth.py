"""Seeded synthetic inputs for the benchmark configurations.

No checkpoints or datasets are available offline, so the models are random-init Qwen2-architecture
decoders: weights N(0, 0.02), norm gains 1, biases 0, drawn in f32 and rounded to BF16 (nearest,
ties to even) because the reference reads only BF16 safetensors (src/weights.rs:276-285,
src/safetensors.rs:110-119). Prompts are uniform-random token ids with repeated spans.
"""

from __future__ import annotations

import json
import os
import struct

import numpy as np

SHAPES = {
    # Qwen2.5-0.5B architecture
    "0.5b": dict(hidden_size=896, num_attention_heads=14, num_key_value_heads=2, intermediate_size=4864,
                 num_hidden_layers=24, vocab_size=151936, rope_theta=1000000.0, max_position_embeddings=32768),
    # Qwen2.5-3B architecture
    "3b": dict(hidden_size=2048, num_attention_heads=16, num_key_value_heads=2, intermediate_size=11008,
               num_hidden_layers=36, vocab_size=151936, rope_theta=1000000.0, max_position_embeddings=32768),
}
# The 3B widths (head size 128, 16 / 2 heads, FFN 11008, full vocabulary) with 2 layers: parity
# tests at those shapes without 36 layers of CPU work per token.
SHAPES["3b-2l"] = dict(SHAPES["3b"], num_hidden_layers=2)

SUFFIXES = [
    "input_layernorm.weight", "mlp.down_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
    "post_attention_layernorm.weight", "self_attn.k_proj.bias", "self_attn.k_proj.weight", "self_attn.o_proj.weight",
    "self_attn.q_proj.bias", "self_attn.q_proj.weight", "self_attn.v_proj.bias", "self_attn.v_proj.weight",
]


def config_json(shape: str) -> str:
    s = SHAPES[shape]
    cfg = {"model_type": "qwen2", "hidden_act": "silu", "tie_word_embeddings": True, **s, "rms_norm_eps": 1e-6}
    return json.dumps(cfg)


def _tensors(s: dict):
    h, I, L, V = s["hidden_size"], s["intermediate_size"], s["num_hidden_layers"], s["vocab_size"]
    kv = s["num_key_value_heads"] * (h // s["num_attention_heads"])
    shapes = {
        "input_layernorm.weight": [h], "mlp.down_proj.weight": [h, I], "mlp.gate_proj.weight": [I, h],
        "mlp.up_proj.weight": [I, h], "post_attention_layernorm.weight": [h], "self_attn.k_proj.bias": [kv],
        "self_attn.k_proj.weight": [kv, h], "self_attn.o_proj.weight": [h, h], "self_attn.q_proj.bias": [h],
        "self_attn.q_proj.weight": [h, h], "self_attn.v_proj.bias": [kv], "self_attn.v_proj.weight": [kv, h],
    }
    out = [("model.embed_tokens.weight", [V, h])]
    for l in range(L):
        for suf in SUFFIXES:
            out.append((f"model.layers.{l}.{suf}", shapes[suf]))
    out.append(("model.norm.weight", [h]))
    return out


def f32_to_bf16_rne(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (src/quant.rs:26-33 semantics, finite inputs)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))) >> 16).astype(np.uint16)


def write_random_model(d: str, shape: str, seed: int, std: float = 0.02) -> str:
    """config.json + model.safetensors (BF16) of a random-init model, streamed tensor by tensor."""
    os.makedirs(d, exist_ok=True)
    s = SHAPES[shape]
    tensors = _tensors(s)
    entries, off = [], 0
    for name, shp in tensors:
        n = int(np.prod(shp)) * 2
        entries.append(f'"{name}":{{"dtype":"BF16","shape":[{",".join(map(str, shp))}],"data_offsets":[{off},{off + n}]}}')
        off += n
    header = '{"__metadata__":{"format":"pt"},' + ",".join(entries) + "}"
    while len(header) % 8:
        header += " "
    rng = np.random.default_rng(seed)
    tmp = os.path.join(d, "model.safetensors.partial")
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(header)))
        f.write(header.encode())
        for name, shp in tensors:
            n = int(np.prod(shp))
            if name.endswith("norm.weight"):
                f.write(np.full(n, 0x3F80, np.uint16).tobytes())  # 1.0
            elif name.endswith(".bias"):
                f.write(np.zeros(n, np.uint16).tobytes())
            else:
                step = 1 << 24
                for a in range(0, n, step):
                    m = min(step, n - a)
                    v = rng.standard_normal(m, dtype=np.float32) * np.float32(std)
                    f.write(f32_to_bf16_rne(v).tobytes())
    os.replace(tmp, os.path.join(d, "model.safetensors"))
    with open(os.path.join(d, "config.json"), "w") as f:
        f.write(config_json(shape))
    return d


def make_prompt(n: int, vocab: int, span: int, repeats: int, seed: int) -> list[int]:
    """n uniform-random ids in which one random span of `span` ids appears `repeats` times."""
    rng = np.random.default_rng(seed)
    p = rng.integers(0, vocab, size=n, dtype=np.int64)
    if span and repeats:
        s = rng.integers(0, vocab, size=span, dtype=np.int64)
        slots = np.linspace(0, n - span, repeats + 1, dtype=np.int64)[1:] if repeats > 1 else [n - span]
        for st in slots[:repeats]:
            p[st:st + span] = s
    return [int(v) for v in p]


def make_prompt_spans(n: int, vocab: int, span: int, seed: int) -> list[int]:
    """n ids built from random `span`-long blocks, each block repeated once right after itself."""
    rng = np.random.default_rng(seed)
    out: list[int] = []
    while len(out) < n:
        b = rng.integers(0, vocab, size=span, dtype=np.int64).tolist()
        out += b + b
    return [int(v) for v in out[:n]]


def ensure_model(root: str, shape: str, seed: int) -> str:
    """Directory of the BF16 random-init model, generated once per (shape, seed)."""
    d = os.path.join(root, f"{shape}-s{seed}")
    if not os.path.exists(os.path.join(d, "model.safetensors")):
        write_random_model(d, shape, seed)
    return d


def ensure_lsq(root: str, shape: str, seed: int, body, embed=None, clip: bool = True, device: int = 0) -> str:
    """`.lsq` file of the random-init model quantized on the GPU by the product quantizer."""
    import layerstream_b200 as ls

    d = ensure_model(root, shape, seed)
    e = embed or body
    p = os.path.join(root, f"{shape}-s{seed}-q{body[0]}g{body[1]}-e{e[0]}g{e[1]}{'-clip' if clip else ''}.lsq")
    if not os.path.exists(p):
        tmp = p + f".{os.getpid()}.partial"
        if os.path.exists(tmp):
            os.remove(tmp)
        ls.quantize_model(d, tmp, body, e, clip=clip, device=device)
        os.replace(tmp, p)
    return p
