"""layerstream_b200: the speculative-decode verify path of layerstream on NVIDIA B200 (sm_100a).

Python binding (ctypes) of ``liblayerstream_b200.so``, whose C ABI is ``include/layerstream.h``.
The names mirror the reference's Rust API (``model::Model``, ``spec::speculative_greedy``,
``quant::quantize_model``): errors are raised as ``LayerstreamError`` carrying the library's message.
There is no CPU fallback: without the built library (and a CUDA device) every call fails.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblayerstream_b200.so")

MODE_RESIDENT = 0
MODE_STREAM = 1


class LayerstreamError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class ModelInfo(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("hidden", "inter", "layers", "heads", "kv_heads", "head_dim", "vocab", "max_ctx")] + [
        (n, C.c_int32) for n in ("bits", "group", "embed_bits", "embed_group")
    ] + [("eps", C.c_float), ("rope_theta", C.c_float), ("layer_bytes", C.c_uint64), ("embed_row_bytes", C.c_uint64),
         ("weight_bytes", C.c_uint64), ("persistent_pass", C.c_int32), ("kv_page", C.c_int32),
         ("kv_pages_total", C.c_uint64), ("kv_pages_used", C.c_uint64)]


class Report(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("resident_weight_bytes", "bytes_read", "wait_ns", "passes", "h2d_bytes", "d2h_bytes")]


PROF_CLASSES = ("qkv", "attention", "o", "gate_up", "down", "head", "pass")


class Profile(C.Structure):
    _fields_ = [("launches", C.c_uint64 * 7), ("ms", C.c_double * 7), ("bytes", C.c_double * 7),
                ("busy_ms", C.c_double * 7), ("crit_ms", (C.c_double * 6) * 7)]


BATCH_PROF_CLASSES = ("qkv", "attention", "o", "gate_up", "down", "head", "collective", "pass")


class BatchProfile(C.Structure):
    _fields_ = [("launches", C.c_uint64 * 8), ("ms", C.c_double * 8), ("bytes", C.c_double * 8)]


class SpecStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("target_passes", "drafted", "accepted", "draft_forwards")] + [
        (n, C.c_double) for n in ("target_secs", "draft_secs", "first_secs", "decode_secs")
    ]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


_lib = None

# C signatures of include/layerstream.h
_SIGS = {
    "ls_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "ls_model_open": (C.c_int, [C.c_char_p, C.c_int, C.c_uint64, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "ls_model_free": (C.c_int, [C.c_void_p]),
    "ls_model_open_sealed": (C.c_int, [C.c_char_p, C.c_void_p, C.c_int, C.c_uint64, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "ls_seal_model": (C.c_int, [C.c_char_p, C.c_char_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_int,
                                C.POINTER(C.c_uint64)]),
    "ls_model_info": (C.c_int, [C.c_void_p, C.POINTER(ModelInfo)]),
    "ls_model_report": (C.c_int, [C.c_void_p, C.POINTER(Report)]),
    "ls_model_stream": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "ls_model_profile_enable": (C.c_int, [C.c_void_p, C.c_int]),
    "ls_model_profile": (C.c_int, [C.c_void_p, C.POINTER(Profile)]),
    "ls_pos": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64)]),
    "ls_reset": (C.c_int, [C.c_void_p]),
    "ls_truncate": (C.c_int, [C.c_void_p, C.c_uint64]),
    "ls_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p, C.POINTER(C.c_uint32)]),
    "ls_forward_multi": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p]),
    "ls_verify": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "ls_speculative_greedy": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_void_p,
                                        C.c_uint64, C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(SpecStats)]),
    "ls_spec_continue": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint64,
                                   C.c_void_p, C.c_uint64, C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(SpecStats)]),
    "ls_quantize_model": (C.c_int, [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.POINTER(C.c_double)]),
    "ls_qgemv_host": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_uint64, C.c_void_p,
                                C.c_int, C.POINTER(C.c_double)]),
    "ls_bgemm_host": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_uint64, C.c_void_p,
                                C.c_int, C.POINTER(C.c_double)]),
    "ls_qweights_upload": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_uint64, C.c_uint64, C.POINTER(C.c_void_p)]),
    "ls_qweights_free": (C.c_int, [C.c_void_p]),
    "ls_qgemv_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p]),
    "ls_qgemv_bytes": (C.c_uint64, [C.c_int, C.c_int, C.c_uint64, C.c_uint64, C.c_uint64]),
    "ls_batch_open": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.POINTER(C.c_void_p)]),
    "ls_batch_free": (C.c_int, [C.c_void_p]),
    "ls_tp_unique_id": (C.c_int, [C.c_void_p, C.c_size_t]),
    "ls_batch_open_tp": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_int, C.c_int, C.c_void_p,
                                   C.POINTER(C.c_void_p)]),
    "ls_batch_pos": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_uint64)]),
    "ls_batch_truncate": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64]),
    "ls_batch_prefill": (C.c_int, [C.c_void_p, C.c_uint64, C.c_void_p, C.c_uint64, C.POINTER(C.c_uint32)]),
    "ls_batch_verify": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_void_p]),
    "ls_batch_spec": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_void_p, C.c_uint64,
                                C.c_void_p, C.c_void_p, C.POINTER(SpecStats)]),
    "ls_batch_report": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "ls_batch_profile_enable": (C.c_int, [C.c_void_p, C.c_int]),
    "ls_batch_profile": (C.c_int, [C.c_void_p, C.POINTER(BatchProfile)]),
    "ls_batch_tp_peer": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "ls_attention_host": (C.c_int, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_uint64, C.c_uint64, C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_double)]),
    "ls_batch_inject_error": (C.c_int, [C.c_void_p, C.c_int]),
    "ls_model_inject_stall": (C.c_int, [C.c_void_p, C.c_int]),
    "ls_attention_paged_host": (C.c_int, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_uint64, C.c_uint64, C.c_void_p,
                                          C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_void_p, C.c_int,
                                          C.POINTER(C.c_double)]),
    "ls_qgemv_rows_noalloc": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_uint64,
                                        C.c_void_p, C.c_void_p]),
    "ls_dequant_rows_host": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_uint64, C.c_void_p]),
    "ls_aead_host": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p, C.c_uint64, C.c_uint64,
                               C.c_uint32, C.c_void_p, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
    "ls_tp_reduce_host": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint64, C.c_int, C.c_uint32, C.c_int,
                                    C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_double), C.c_uint32, C.c_void_p, C.c_float,
                                    C.c_void_p]),
}


def lib():
    """Loads the CUDA library (raises if it has not been built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m layerstream_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc: int):
    if rc != 0:
        buf = C.create_string_buffer(4096)
        lib().ls_last_error(buf, 4096)
        raise LayerstreamError(rc, buf.value.decode(errors="replace"))


def _u32(a):
    return np.ascontiguousarray(a, dtype=np.uint32)


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class Model:
    """``model::Model`` (src/model.rs) backed by CUDA: a `.lsq` model resident in HBM or streamed
    through ``slots`` HBM layer slots from pinned host memory."""

    def __init__(self, path: str, device: int = 0, max_ctx: int = 1024, mode: str = "resident", slots: int = 2,
                 key: bytes = None):
        """key: the 32-byte key of a sealed file (bytes, or 64 hex digits; src/seal.rs:422-440)."""
        h = C.c_void_p()
        md = {"resident": MODE_RESIDENT, "stream": MODE_STREAM}[mode]
        if key is None:
            _check(lib().ls_model_open(str(path).encode(), device, max_ctx, md, slots, C.byref(h)))
        else:
            k = _bytes_arr(_key_bytes(key), 32)
            _check(lib().ls_model_open_sealed(str(path).encode(), _p(k), device, max_ctx, md, slots, C.byref(h)))
        self._h = h
        info = self.info
        self.vocab = info.vocab
        self.max_ctx = max_ctx
        self.mode = mode

    def close(self):
        if getattr(self, "_h", None):
            lib().ls_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def info(self) -> ModelInfo:
        """ls_model_info, read now (the K/V page counts change as the cache grows and shrinks)."""
        info = ModelInfo()
        _check(lib().ls_model_info(self._h, C.byref(info)))
        return info

    @property
    def pos(self) -> int:
        p = C.c_uint64()
        _check(lib().ls_pos(self._h, C.byref(p)))
        return p.value

    def reset(self):
        _check(lib().ls_reset(self._h))

    def truncate(self, pos: int):
        _check(lib().ls_truncate(self._h, pos))

    def forward(self, tokens, want_logits: bool = True):
        """Returns the last position's logits (and keeps the greedy token in ``self.last_argmax``)."""
        t = _u32(tokens)
        out = np.empty(self.vocab, np.float32) if want_logits else None
        a = C.c_uint32()
        _check(lib().ls_forward(self._h, _p(t), t.size, _p(out) if out is not None else None, C.byref(a)))
        self.last_argmax = a.value
        return out if want_logits else a.value

    def forward_multi(self, tokens, n: int) -> np.ndarray:
        t = _u32(tokens)
        out = np.empty((max(n, 1), self.vocab), np.float32)
        _check(lib().ls_forward_multi(self._h, _p(t), t.size, n, _p(out)))
        return out

    def verify(self, block):
        """The verify step: returns (m, next) and keeps [a, d_1 .. d_m] in the cache."""
        b = _u32(block)
        m, nxt = C.c_uint32(), C.c_uint32()
        _check(lib().ls_verify(self._h, _p(b), b.size, C.byref(m), C.byref(nxt)))
        return m.value, nxt.value

    @property
    def stream(self) -> int:
        """cudaStream_t (as an int) of this model's kernels."""
        p = C.c_void_p()
        _check(lib().ls_model_stream(self._h, C.byref(p)))
        return p.value or 0

    def profile_enable(self, on=True):
        """Live timing: 1/True = CUDA events (per-kernel classes, or the whole persistent pass);
        2 = also the persistent pass kernel's barrier timeline (per-phase split, a few % slower)."""
        _check(lib().ls_model_profile_enable(self._h, int(on)))

    def profile(self) -> dict:
        p = Profile()
        _check(lib().ls_model_profile(self._h, C.byref(p)))
        return {c: {"launches": p.launches[i], "ms": p.ms[i], "bytes": p.bytes[i], "busy_ms": p.busy_ms[i],
                    "crit_ms": list(p.crit_ms[i])}
                for i, c in enumerate(PROF_CLASSES)}

    def inject_stall(self, barrier: int):
        """Test hook: the next persistent pass waits at grid barrier `barrier` until its bounded
        wait runs out (the call then fails with a device error; the model stays usable)."""
        _check(lib().ls_model_inject_stall(self._h, barrier))

    def report(self) -> dict:
        r = Report()
        _check(lib().ls_model_report(self._h, C.byref(r)))
        return {n: getattr(r, n) for n, _ in r._fields_}


def speculative_greedy(target: Model, draft: Model | None, prompt, max_new: int, k: int, eos=()):
    """``spec::speculative_greedy`` (src/spec.rs:57-152). ``draft=None`` uses the prompt-lookup drafter."""
    p = _u32(prompt)
    e = _u32(list(eos) if len(eos) else [0])
    out = np.zeros(max(max_new, 1), np.uint32)
    n = C.c_uint64()
    st = SpecStats()
    _check(lib().ls_speculative_greedy(target._h, draft._h if draft is not None else None, _p(p), p.size, max_new, k, _p(e),
                                       len(eos), _p(out), C.byref(n), C.byref(st)))
    return out[: n.value].tolist(), st.as_dict()


def spec_continue(target: Model, draft: Model | None, hist, first: int, max_new: int, k: int, eos=()):
    """The decode loop of ``speculative_greedy`` from a prefilled state (both models hold ``hist``)."""
    h = _u32(hist)
    e = _u32(list(eos) if len(eos) else [0])
    out = np.zeros(max(max_new, 1), np.uint32)
    n = C.c_uint64()
    st = SpecStats()
    _check(lib().ls_spec_continue(target._h, draft._h if draft is not None else None, _p(h), h.size, first, max_new, k,
                                  _p(e), len(eos), _p(out), C.byref(n), C.byref(st)))
    return out[: n.value].tolist(), st.as_dict()


class Batch:
    """B independent sequences sharing one resident model's weights (configs 4 and 5): per-sequence
    K/V caches, one verify pass for all sequences' [B][M] blocks."""

    def __init__(self, model: Model, batch: int, max_ctx: int, max_block: int, tp=None):
        """tp = (rank, world, id): this rank's shard of a tensor-parallel split (id from tp_unique_id
        on one rank, the same bytes on every rank; opening is collective)."""
        h = C.c_void_p()
        if tp is None:
            _check(lib().ls_batch_open(model._h, batch, max_ctx, max_block, C.byref(h)))
        else:
            rank, world, uid = tp
            buf = (C.c_uint8 * len(uid)).from_buffer_copy(bytes(uid))
            _check(lib().ls_batch_open_tp(model._h, batch, max_ctx, max_block, rank, world, buf, C.byref(h)))
        self._h, self.model, self.batch, self.max_ctx, self.max_block = h, model, batch, max_ctx, max_block

    def pos(self, seq: int) -> int:
        v = C.c_uint64()
        _check(lib().ls_batch_pos(self._h, seq, C.byref(v)))
        return v.value

    def truncate(self, seq: int, pos: int):
        _check(lib().ls_batch_truncate(self._h, seq, pos))

    def prefill(self, seq: int, ids) -> int:
        a = _u32(ids)
        out = C.c_uint32()
        _check(lib().ls_batch_prefill(self._h, seq, _p(a), a.size, C.byref(out)))
        return out.value

    def verify(self, blocks) -> tuple[list[int], list[int]]:
        b = np.ascontiguousarray(blocks, np.uint32)
        nseq, M = b.shape
        m = np.zeros(nseq, np.uint32)
        nxt = np.zeros(nseq, np.uint32)
        _check(lib().ls_batch_verify(self._h, _p(b), nseq, M, _p(m), _p(nxt)))
        return m.tolist(), nxt.tolist()

    def spec(self, prompts, max_new: int, k: int, eos=()):
        p = np.ascontiguousarray(prompts, np.uint32)
        B, plen = p.shape
        e = _u32(list(eos) if len(eos) else [0])
        out = np.zeros((B, max(max_new, 1)), np.uint32)
        n = np.zeros(B, np.uint64)
        st = SpecStats()
        _check(lib().ls_batch_spec(self._h, _p(p), plen, max_new, k, _p(e), len(eos), _p(out), _p(n), C.byref(st)))
        return [out[i, : int(n[i])].tolist() for i in range(B)], st.as_dict()

    def inject_error(self, code: int = 4):
        """Test hook: the next pass fails with a device error (no fault on the GPU)."""
        _check(lib().ls_batch_inject_error(self._h, code))

    def report(self) -> dict:
        a, b, c = C.c_uint64(), C.c_uint64(), C.c_uint64()
        _check(lib().ls_batch_report(self._h, C.byref(a), C.byref(b), C.byref(c)))
        return {"passes": a.value, "h2d_bytes": b.value, "d2h_bytes": c.value}

    def profile_enable(self, on=True):
        """Live timing: CUDA events around every launch class of each pass (clears the counters)."""
        _check(lib().ls_batch_profile_enable(self._h, int(on)))

    def profile(self) -> dict:
        p = BatchProfile()
        _check(lib().ls_batch_profile(self._h, C.byref(p)))
        return {c: {"launches": p.launches[i], "ms": p.ms[i], "bytes": p.bytes[i]} for i, c in enumerate(BATCH_PROF_CLASSES)}

    def tp_peer(self) -> bool:
        """True when the tensor-parallel sums go through the peers' memory, False on NCCL."""
        on = C.c_int()
        _check(lib().ls_batch_tp_peer(self._h, C.byref(on)))
        return bool(on.value)

    def close(self):
        if getattr(self, "_h", None):
            lib().ls_batch_free(self._h)
            self._h = None

    def __del__(self):
        self.close()


def tp_unique_id() -> bytes:
    """NCCL unique id for a tensor-parallel group (made on one rank, shared with the others)."""
    buf = (C.c_uint8 * 128)()
    _check(lib().ls_tp_unique_id(buf, 128))
    return bytes(buf)


def quantize_model(src_dir: str, out_path: str, body=(8, 64), embed=None, clip: bool = True, device: int = 0) -> float:
    """``quant::quantize_model`` (src/quant.rs:158-251) with the group quantization on the GPU."""
    eb, eg = embed if embed else body
    r = C.c_double()
    _check(lib().ls_quantize_model(str(src_dir).encode(), str(out_path).encode(), body[0], body[1], eb, eg, int(clip), device,
                                   C.byref(r)))
    return r.value


def qgemv(bits: int, group: int, rows_raw: np.ndarray, rows: int, cols: int, x: np.ndarray, iters: int = 1):
    """y = W x through the verify-path GEMV kernel; W in the stored row format. Returns (y, ms)."""
    w = np.ascontiguousarray(rows_raw, np.uint8)
    xx = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    y = np.empty((xx.shape[0], rows), np.float32)
    ms = C.c_double()
    _check(lib().ls_qgemv_host(bits, group, _p(w), rows, cols, _p(xx), xx.shape[0], _p(y), iters, C.byref(ms)))
    return y, ms.value


def dequant_rows(bits: int, group: int, rows_raw: np.ndarray, rows: int, cols: int, ids) -> np.ndarray:
    """Embedding gather + dequantisation of stored rows `ids` on the GPU (bit-exact)."""
    w = np.ascontiguousarray(rows_raw, np.uint8)
    i = _u32(ids)
    out = np.empty((i.size, cols), np.float32)
    _check(lib().ls_dequant_rows_host(bits, group, _p(w), rows, cols, _p(i), i.size, _p(out)))
    return out


class QWeights:
    """A quantized matrix uploaded once (device planes) for timing the GEMV on device buffers."""

    def __init__(self, bits: int, group: int, rows_raw: np.ndarray, rows: int, cols: int, device: int = 0):
        h = C.c_void_p()
        w = np.ascontiguousarray(rows_raw, np.uint8)
        _check(lib().ls_qweights_upload(device, bits, group, _p(w), rows, cols, C.byref(h)))
        self._h, self.rows, self.cols, self.bits, self.group = h, rows, cols, bits, group

    def gemv(self, x_ptr: int, M: int, y_ptr: int, stream: int = 0):
        _check(lib().ls_qgemv_device(self._h, C.c_void_p(x_ptr), M, C.c_void_p(y_ptr), C.c_void_p(stream)))

    def bytes(self, M: int) -> int:
        return lib().ls_qgemv_bytes(self.bits, self.group, self.rows, self.cols, M)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().ls_qweights_free(self._h)
            self._h = None


def bgemm(bits: int, group: int, rows_raw, rows: int, cols: int, x, iters: int = 1):
    """The batched verify-pass GEMM: y = x W^T for M rows of x (stored rows in the .lsq format).
    Returns (y M x rows, ms per launch when iters > 1)."""
    w = np.ascontiguousarray(rows_raw, np.uint8)
    xx = np.ascontiguousarray(x, np.float32)
    M = xx.shape[0]
    y = np.empty((M, rows), np.float32)
    ms = C.c_double()
    _check(lib().ls_bgemm_host(bits, group, _p(w), rows, cols, _p(xx), M, _p(y), iters, C.byref(ms)))
    return y, ms.value


def aead_seal(key: bytes, nonce: bytes, aad: bytes, data: bytes, chunk_bytes: int = 0, first: int = 0, iters: int = 1):
    """ChaCha20-Poly1305 sealing on the GPU (RFC 8439 2.8; chunk_bytes > 0: the sealed file's
    per-chunk messages, chunk i under nonce[:8] + le32(first + i) and aad + le32(first + i)).
    Returns (ciphertext, tags: one 16-byte tag per chunk, ms per call when iters > 1)."""
    buf = np.frombuffer(bytes(data), np.uint8).copy()
    n = 1 if chunk_bytes == 0 or len(data) == 0 else -(-len(data) // chunk_bytes)
    tags = np.zeros(16 * n, np.uint8)
    k, nn, a = _bytes_arr(key, 32), _bytes_arr(nonce, 12), np.frombuffer(bytes(aad) or b"\0", np.uint8)
    ms, bad = C.c_double(), C.c_int64()
    _check(lib().ls_aead_host(1, _p(k), _p(nn), _p(a), len(aad), _p(buf), len(data), chunk_bytes, first, _p(tags), iters,
                              C.byref(ms), C.byref(bad)))
    return buf.tobytes(), [tags[16 * i:16 * i + 16].tobytes() for i in range(n)], ms.value


def aead_open(key: bytes, nonce: bytes, aad: bytes, data: bytes, tags, chunk_bytes: int = 0, first: int = 0):
    """ChaCha20-Poly1305 opening on the GPU: every tag is checked, then the data decrypted. Raises
    LayerstreamError (LS_ERR_IO) on a mismatch; returns the plaintext."""
    buf = np.frombuffer(bytes(data), np.uint8).copy()
    t = np.frombuffer(b"".join(bytes(x) for x in tags), np.uint8).copy()
    k, nn, a = _bytes_arr(key, 32), _bytes_arr(nonce, 12), np.frombuffer(bytes(aad) or b"\0", np.uint8)
    ms, bad = C.c_double(), C.c_int64()
    _check(lib().ls_aead_host(0, _p(k), _p(nn), _p(a), len(aad), _p(buf), len(data), chunk_bytes, first, _p(t), 1,
                              C.byref(ms), C.byref(bad)))
    return buf.tobytes()


def tp_reduce(x, ys, rank: int, preset: bool = True, wait_ms: int = 1000, calls: int = 1, K: int = 0, norm=None,
              eps: float = 1e-6):
    """The tensor-parallel reduction kernel on one GPU, as rank `rank` of len(ys) emulated ranks
    whose partials all sit in this GPU's memory: returns (x + calls * sum(ys), ms per call), and
    with K > 0 the fused form's f16 operand (rows x K, RMSNorm-ed with norm) as a third item.
    preset=False leaves the peers' flags unset: the kernel's wait runs out after wait_ms and
    LayerstreamError (LS_ERR_DEVICE) is raised."""
    x = np.ascontiguousarray(x, np.float32).ravel()
    ys = np.ascontiguousarray(ys, np.float32)
    if ys.ndim != 2 or ys.shape[1] != x.size:
        raise ValueError("ys must be world x n")
    out = np.empty_like(x)
    op = np.zeros(x.size if K else 1, np.uint16)
    nw = None if norm is None else np.ascontiguousarray(norm, np.float32)
    st, ms = C.c_int(), C.c_double()
    _check(lib().ls_tp_reduce_host(_p(x), _p(ys), ys.shape[0], rank, x.size, int(preset), wait_ms, calls, _p(out), C.byref(st),
                                   C.byref(ms), K, None if nw is None else _p(nw), eps, _p(op)))
    if K:
        return out, ms.value, op.view(np.float16).reshape(-1, K)
    return out, ms.value


def _key_bytes(key) -> bytes:
    if isinstance(key, str):
        key = bytes.fromhex(key.strip())
    return bytes(key)


def seal_model(src: str, out: str, key, nonce_prefix: bytes, layer_chunk: int = 1 << 20, embed_chunk_rows: int = 512,
               device: int = 0) -> int:
    """seal_model (src/seal.rs:726-827) with the cipher on the GPU: src is a .lsq file or a bf16
    model directory, out a new file. Returns the number of chunks."""
    k, p = _bytes_arr(_key_bytes(key), 32), _bytes_arr(bytes(nonce_prefix), 8)
    n = C.c_uint64()
    _check(lib().ls_seal_model(str(src).encode(), str(out).encode(), _p(k), _p(p), layer_chunk, embed_chunk_rows, device,
                               C.byref(n)))
    return n.value


def _bytes_arr(b: bytes, n: int) -> np.ndarray:
    if len(b) != n:
        raise ValueError(f"expected {n} bytes, got {len(b)}")
    return np.frombuffer(bytes(b), np.uint8).copy()


def attention(heads: int, kv_heads: int, hd: int, pos0: int, qkv: np.ndarray, k_cache=None, v_cache=None,
              rope_theta: float = 1e6, iters: int = 1):
    """One layer's causal GQA attention of an M-row block (qkv: M x (heads + 2 kv_heads) * hd f32,
    pre-RoPE) over pos0 cached rows (kv_heads x pos0 x hd f16 arrays). Returns (out M x heads*hd, ms)."""
    q = np.ascontiguousarray(qkv, np.float32)
    M = q.shape[0]
    out = np.empty((M, heads * hd), np.float32)
    kc = np.ascontiguousarray(k_cache, np.float16).view(np.uint16) if pos0 else None
    vc = np.ascontiguousarray(v_cache, np.float16).view(np.uint16) if pos0 else None
    ms = C.c_double()
    _check(lib().ls_attention_host(heads, kv_heads, hd, rope_theta, pos0, M, _p(q), _p(kc) if kc is not None else None,
                                   _p(vc) if vc is not None else None, _p(out), iters, C.byref(ms)))
    return out, ms.value


def attention_paged(heads: int, kv_heads: int, hd: int, pos0: int, qkv: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray,
                    page: int, table, rope_theta: float = 1e6, iters: int = 1):
    """The same attention through a paged K/V cache: k_pool, v_pool are kv_heads x num_pages x page x
    hd f16 arrays, table[i] the pool page of positions [i * page, (i + 1) * page). The block's K/V rows
    are written into their pages (the pools are updated in place). Returns (out, ms)."""
    q = np.ascontiguousarray(qkv, np.float32)
    M = q.shape[0]
    if k_pool.dtype != np.float16 or v_pool.dtype != np.float16 or not k_pool.flags.c_contiguous or not v_pool.flags.c_contiguous:
        raise ValueError("k_pool and v_pool must be C-contiguous float16 arrays")
    num_pages = k_pool.shape[1]
    t = np.ascontiguousarray(table, np.int32)
    out = np.empty((M, heads * hd), np.float32)
    ms = C.c_double()
    _check(lib().ls_attention_paged_host(heads, kv_heads, hd, rope_theta, pos0, M, _p(q), _p(k_pool), _p(v_pool), num_pages, page,
                                         _p(t), _p(out), iters, C.byref(ms)))
    return out, ms.value


def qgemv_rows_noalloc(bits: int, group: int, rows_ptr: int, rows: int, cols: int, x_ptr: int, M: int, y_ptr: int,
                       stream: int = 0):
    """y = W x on device buffers the caller owns (W in the stored row format); the library allocates
    nothing (its K-split scratch is a fixed per-GPU array shared by all calls)."""
    _check(lib().ls_qgemv_rows_noalloc(bits, group, C.c_void_p(rows_ptr), rows, cols, C.c_void_p(x_ptr), M,
                                       C.c_void_p(y_ptr), C.c_void_p(stream)))


SYMBOLS = tuple(_SIGS)
