"""ctypes binding of the CPU oracle (test infrastructure, not product code).

The oracle is a C++ restatement of layerstream's verify path (src/kernels.rs, src/model.rs,
src/spec.rs, src/quant.rs, src/weights.rs) with the reference's float operation order. Only the
tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` load it; the product
library never does.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblsoracle.so")

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (g++, no fast-math, no FMA contraction)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "ls_oracle.cpp")
    ):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = C.CDLL(LIB_PATH)
    u64, i32, f32, f64, vp, cp = C.c_uint64, C.c_int, C.c_float, C.c_double, C.c_void_p, C.c_char_p
    P = C.POINTER
    sig = {
        "orc_last_error": (i32, [C.c_char_p, C.c_size_t]),
        "orc_bf16_round": (f32, [f32]),
        "orc_row_bytes": (u64, [i32, u64, u64]),
        "orc_validate_format": (i32, [i32, u64, P(u64), u64]),
        "orc_quantize_row": (i32, [i32, u64, vp, u64, i32, vp, P(f64), P(f64)]),
        "orc_dequant_row": (i32, [i32, u64, vp, u64, vp]),
        "orc_dot": (f32, [i32, u64, vp, vp, u64]),
        "orc_matmul": (i32, [i32, u64, vp, u64, u64, vp, u64, vp, i32]),
        "orc_rms_norm_bf16": (None, [vp, vp, u64, u64, f32, vp]),
        "orc_rms_norm_f32": (None, [vp, vp, u64, f32, vp]),
        "orc_rope": (None, [vp, vp, u64, u64]),
        "orc_softmax": (None, [vp, u64]),
        "orc_silu": (f32, [f32]),
        "orc_argmax": (C.c_uint32, [vp, u64]),
        "orc_inject_quant": (i32, [cp, i32, u64, i32, i32, u64, C.c_char_p, u64, P(u64)]),
        "orc_config_parse": (i32, [cp, P(u64), P(f32)]),
        "orc_quantize_model": (i32, [cp, cp, i32, u64, i32, u64, i32, i32, P(f64)]),
        "orc_open_files": (i32, [cp, i32, P(u64), P(u64), P(u64)]),
        "orc_model_open": (vp, [cp, i32, i32, u64]),
        "orc_model_free": (None, [vp]),
        "orc_model_pos": (u64, [vp]),
        "orc_model_vocab": (u64, [vp]),
        "orc_model_hidden": (u64, [vp]),
        "orc_model_reset": (None, [vp]),
        "orc_model_truncate": (i32, [vp, u64]),
        "orc_forward": (i32, [vp, vp, u64, vp]),
        "orc_forward_multi": (i32, [vp, vp, u64, u64, vp]),
        "orc_forward_hidden": (i32, [vp, vp, u64, u64, vp]),
        "orc_speculative_greedy": (i32, [vp, vp, vp, u64, u64, u64, vp, u64, vp, P(u64), P(u64), P(f64)]),
        "orc_spec_continue": (i32, [vp, vp, vp, u64, C.c_uint32, u64, u64, vp, u64, vp, P(u64), P(u64), P(f64)]),
        "orc_forward_argmax": (i32, [vp, vp, u64, P(C.c_uint32)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


class OracleError(RuntimeError):
    pass


def _check(rc: int):
    if rc != 0:
        buf = C.create_string_buffer(4096)
        lib().orc_last_error(buf, 4096)
        raise OracleError(buf.value.decode())


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def bf16_round(v: float) -> float:
    return lib().orc_bf16_round(C.c_float(v))


def row_bytes(bits: int, group: int, cols: int) -> int:
    return lib().orc_row_bytes(bits, group, cols)


def validate_format(bits: int, group: int, cols) -> None:
    arr = (C.c_uint64 * len(cols))(*cols)
    _check(lib().orc_validate_format(bits, group, arr, len(cols)))


def quantize_row(bits: int, group: int, row: np.ndarray, clip: bool):
    row = np.ascontiguousarray(row, dtype=np.float32)
    out = np.zeros(row_bytes(bits, group, row.size), dtype=np.uint8)
    e, n = C.c_double(), C.c_double()
    _check(lib().orc_quantize_row(bits, group, _ptr(row), row.size, int(clip), _ptr(out), C.byref(e), C.byref(n)))
    return out, e.value, n.value


def dequant_row(bits: int, group: int, raw: np.ndarray, cols: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.zeros(cols, dtype=np.float32)
    _check(lib().orc_dequant_row(bits, group, _ptr(raw), cols, _ptr(out)))
    return out


def dot(bits: int, group: int, row: np.ndarray, x: np.ndarray) -> float:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    return lib().orc_dot(bits, group, _ptr(row), _ptr(x), x.size)


def matmul(bits: int, group: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, threads: int = 4) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
    y = np.zeros((x.shape[0], rows), dtype=np.float32)
    _check(lib().orc_matmul(bits, group, _ptr(w), rows, cols, _ptr(x), x.shape[0], _ptr(y), threads))
    return y


def rms_norm_bf16(x: np.ndarray, w_bf16: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = w_bf16.size
    out = np.zeros_like(x)
    lib().orc_rms_norm_bf16(_ptr(x), _ptr(np.ascontiguousarray(w_bf16, dtype=np.uint16)), n, x.size // n, eps, _ptr(out))
    return out


def rope(head: np.ndarray, inv_freq: np.ndarray, pos: int) -> np.ndarray:
    h = np.ascontiguousarray(head, dtype=np.float32).copy()
    lib().orc_rope(_ptr(h), _ptr(np.ascontiguousarray(inv_freq, dtype=np.float32)), h.size, pos)
    return h


def softmax(v: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.float32).copy()
    lib().orc_softmax(_ptr(v), v.size)
    return v


def silu(x: float) -> float:
    return lib().orc_silu(C.c_float(x))


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, dtype=np.float32)
    return lib().orc_argmax(_ptr(v), v.size)


def inject_quant(cfg_text: str, bits: int, group: int, embed=None) -> str:
    out = C.create_string_buffer(len(cfg_text) + 256)
    n = C.c_uint64()
    eb, eg = embed if embed else (0, 0)
    _check(lib().orc_inject_quant(cfg_text.encode(), bits, group, int(embed is not None), eb, eg, out, len(out), C.byref(n)))
    return out.value.decode()


def config_parse(text: str) -> dict:
    ints = (C.c_uint64 * 12)()
    fl = (C.c_float * 2)()
    _check(lib().orc_config_parse(text.encode(), ints, fl))
    keys = ["hidden", "inter", "layers", "heads", "kv_heads", "head_dim", "vocab", "max_pos", "bits", "group", "embed_bits", "embed_group"]
    d = {k: int(v) for k, v in zip(keys, ints)}
    d["eps"], d["rope_theta"] = fl[0], fl[1]
    return d


def quantize_model(src_dir: str, out_path: str, body, embed=None, clip: bool = True, threads: int = 4) -> float:
    eb, eg = embed if embed else body
    r = C.c_double()
    _check(lib().orc_quantize_model(src_dir.encode(), out_path.encode(), body[0], body[1], eb, eg, int(clip), threads, C.byref(r)))
    return r.value


def open_files(path: str, quantized: bool):
    lay = (C.c_uint64 * 25)()
    es, ns = C.c_uint64(), C.c_uint64()
    _check(lib().orc_open_files(path.encode(), int(quantized), lay, C.byref(es), C.byref(ns)))
    return {"off": list(lay[:12]), "len": list(lay[12:24]), "total": lay[24], "embed_start": es.value, "norm_start": ns.value}


class Model:
    """CPU restatement of ``layerstream::model::Model`` with resident weights."""

    def __init__(self, path: str, quantized: bool | None = None, threads: int = 4, max_ctx: int = 128):
        if quantized is None:
            quantized = not os.path.isdir(path)
        h = lib().orc_model_open(path.encode(), int(quantized), threads, max_ctx)
        if not h:
            _check(-1)
        self._h = h
        self.vocab = lib().orc_model_vocab(h)
        self.hidden = lib().orc_model_hidden(h)
        self.max_ctx = max_ctx

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().orc_model_free(h)
            self._h = None

    @property
    def pos(self) -> int:
        return lib().orc_model_pos(self._h)

    def reset(self):
        lib().orc_model_reset(self._h)

    def truncate(self, pos: int):
        _check(lib().orc_model_truncate(self._h, pos))

    def forward(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros(self.vocab, dtype=np.float32)
        _check(lib().orc_forward(self._h, _ptr(t), t.size, _ptr(out)))
        return out

    def forward_multi(self, tokens, n: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros((max(n, 1), self.vocab), dtype=np.float32)
        _check(lib().orc_forward_multi(self._h, _ptr(t), t.size, n, _ptr(out)))
        return out

    def forward_hidden(self, tokens, n_layers: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros((t.size, self.hidden), dtype=np.float32)
        _check(lib().orc_forward_hidden(self._h, _ptr(t), t.size, n_layers, _ptr(out)))
        return out


def speculative_greedy(target: Model, draft: Model | None, prompt, max_new: int, k: int, eos=()):
    """src/spec.rs:57-152; draft=None selects the prompt-lookup drafter."""
    p = np.ascontiguousarray(prompt, dtype=np.uint32)
    e = np.ascontiguousarray(list(eos) if len(eos) else [0], dtype=np.uint32)
    out = np.zeros(max(max_new, 1), dtype=np.uint32)
    n = C.c_uint64()
    stats = (C.c_uint64 * 4)()
    times = (C.c_double * 4)()
    _check(lib().orc_speculative_greedy(target._h, draft._h if draft is not None else None, _ptr(p), p.size, max_new, k, _ptr(e),
                                        len(eos), _ptr(out), C.byref(n), stats, times))
    st = dict(zip(["target_passes", "drafted", "accepted", "draft_forwards"], list(stats)))
    st.update(zip(["target_secs", "draft_secs", "first_secs", "decode_secs"], list(times)))
    return out[: n.value].tolist(), st


def spec_continue(target: Model, draft: Model | None, hist, first: int, max_new: int, k: int, eos=()):
    """The decode loop from a prefilled state (both models hold ``hist``)."""
    h = np.ascontiguousarray(hist, dtype=np.uint32)
    e = np.ascontiguousarray(list(eos) if len(eos) else [0], dtype=np.uint32)
    out = np.zeros(max(max_new, 1), dtype=np.uint32)
    n = C.c_uint64()
    stats = (C.c_uint64 * 4)()
    times = (C.c_double * 4)()
    _check(lib().orc_spec_continue(target._h, draft._h if draft is not None else None, _ptr(h), h.size, first, max_new, k,
                                   _ptr(e), len(eos), _ptr(out), C.byref(n), stats, times))
    st = dict(zip(["target_passes", "drafted", "accepted", "draft_forwards"], list(stats)))
    st.update(zip(["target_secs", "draft_secs", "first_secs", "decode_secs"], list(times)))
    return out[: n.value].tolist(), st


def forward_argmax(m: Model, tokens) -> int:
    t = np.ascontiguousarray(tokens, dtype=np.uint32)
    r = C.c_uint32()
    _check(lib().orc_forward_argmax(m._h, _ptr(t), t.size, C.byref(r)))
    return r.value
