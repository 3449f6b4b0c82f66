#!/usr/bin/env python
"""Benchmark of the speculative-decode verify path: accepted tokens/s on BASELINE.json's configs.

Default workload (N=1): config 2 of BASELINE.json -- a Qwen2.5-0.5B-architecture random-init model
(seeded N(0, 0.02) weights, BF16 then int4 group-32 with the clip search), batch 1 per GPU, a
512-token prompt of random ids built from repeated 32-token spans, greedy decode of 256 tokens with
k = 8 guesses per verify pass (prompt-lookup drafter by default; --drafter model uses a second,
int4 model through the reference's draft-Model API).

A step is the decode loop of one sequence (src/spec.rs:94-149): from the prefilled prompt, draft,
verify (one (k+1)-row pass over all weights with the device-side argmax + acceptance), roll back,
until 256 tokens. `value` = tokens emitted after the first / decode seconds (the reference's
definition, src/main.rs:358-359), whole job over all ranks, device-timed with CUDA events on the
model's stream. `e2e` = the same metric through ls_speculative_greedy with host buffers (prefill,
token uploads and result reads inside the timed region). Each rank decodes its own sequence (weak
scaling, no collective on the data path). Inputs: the weights (278 MB per verify pass) exceed L2,
so every pass streams them from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1|2|3|4|5]
"""

from __future__ import annotations

import argparse
import csv
import datetime
import io
import json
import os
import re
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# the pass kernel's critical CTA per phase (last to reach the closing barrier): where its time went
CRIT_SEGMENTS = ("prep", "first_stage", "first_item", "more_items", "to_barrier", "barrier")
MICRO_SHAPES = {"qkv": (1152, 896), "o": (896, 896), "gate_up": (9728, 896), "down": (896, 4864), "head": (151936, 896)}

CONFIGS = {
    1: dict(shape="0.5b", body=(8, 64), embed=(8, 64), prompt=128, span=16, repeats=3, max_new=32, k=4, drafter="model",
            draft=(4, 32)),
    2: dict(shape="0.5b", body=(4, 32), embed=(4, 32), prompt=512, span=32, repeats=0, max_new=256, k=8, drafter="lookup",
            draft=(4, 32)),
}
CONFIGS[4] = dict(shape="0.5b", body=(8, 64), embed=(8, 64), prompt=2048, span=32, repeats=0, max_new=512, k=4,
                  drafter="lookup", draft=(4, 32), batch=64)
CONFIGS[5] = dict(shape="3b", body=(4, 32), embed=(4, 32), prompt=1024, span=32, repeats=0, max_new=256, k=4,
                  drafter="lookup", draft=(4, 32), batch=8, stream_slots=2)
CONFIGS[3] = dict(shape="0.5b", body=(8, 64), embed=(8, 64), prompt=0, span=0, repeats=0, max_new=0, k=0, drafter="none",
                  draft=(4, 32), micro=True)
METRIC = "spec-decode accepted tokens/s"
UNIT = "tok/s"


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=2)
    ap.add_argument("--drafter", choices=["lookup", "model"], default=None)
    ap.add_argument("--target", choices=["quantized", "bf16"], default="quantized",
                    help="configs 1/2: the target's weights, quantized as the config says or the unquantized bf16 "
                         "model (the reference's matmul_bf16 path)")
    ap.add_argument("--root", default=os.environ.get("LS_BENCH_ROOT", "/tmp/ls_b200_bench"))
    ap.add_argument("--tp", action="store_true",
                    help="config 5 (b): the resident model split tensor-parallel over the launched ranks (NCCL), "
                         "instead of 2-slot streaming per GPU")
    ap.add_argument("--sealed", action="store_true",
                    help="config 5 (streaming): the model sealed (ChaCha20-Poly1305, src/seal.rs) and streamed from the "
                         "sealed file, each layer block opened on the GPU after its host-to-device copy")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-sample-tokens", type=int, default=0, help="decode tokens per CPU sample (0: auto)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true", help="print the per-kernel profile to stderr")
    ap.add_argument("--ncu-case", choices=["pass", "gemv", "attention", "bgemm", "bgemm4"], default=None,
                    help="short fixed workloads for ncu: 'pass' = prefill + 3 verify passes of the bench model, "
                         "'gemv' = 3 launches of the LM-head GEMV (151936 x 896, int4 g32, M = 9), "
                         "'attention' = 3 launches of the tensor-core attention (14/2 heads, hd 64, M = 9, "
                         "KV length 32768), 'bgemm' = the batched GEMM on the 3B gate/up shape (M = 40), "
                         "'bgemm4' = the batched GEMM on config 4's gate/up (9728 x 896, int8 g64, M = 320)")
    return ap.parse_args()


def ncu_case(args, cfg):
    """Small deterministic workloads to capture under ncu."""
    import torch

    import layerstream_b200 as ls
    from layerstream_b200 import synth

    torch.cuda.set_device(0)
    if args.ncu_case == "attention":
        # the config-3 attention shape (14 q / 2 kv heads, hd 64, 9 verify rows) at KV length 32768:
        # 256 chunks of 128 positions per kv head over 148 context splits, then the merge kernel
        heads, kvh, hd, M = 14, 2, 64, 9
        pos0 = 32768 - M
        rng = np.random.default_rng(7)
        qkv = rng.standard_normal((M, (heads + 2 * kvh) * hd)).astype(np.float32)
        kc = rng.standard_normal((kvh, pos0, hd)).astype(np.float16)
        vc = rng.standard_normal((kvh, pos0, hd)).astype(np.float16)
        for _ in range(3):
            ls.attention(heads, kvh, hd, pos0, qkv, kc, vc)
        print(json.dumps({"ncu_case": "attention", "heads": heads, "kv_heads": kvh, "hd": hd, "pos0": pos0, "M": M,
                          "kv_bytes": 2 * kvh * (pos0 + M) * hd * 2}))
        return
    if args.ncu_case == "bgemm":
        # the 3B gate/up projection (22016 x 2048, int4 g32) over the 40 rows of a config-5 verify
        # pass (8 sequences x 5), through the batched GEMM
        rows, cols, M = 22016, 2048, 40
        raw = stored_rows(4, 32, rows, cols, seed=3)
        x = np.random.default_rng(3).standard_normal((M, cols)).astype(np.float32)
        _, ms = ls.bgemm(4, 32, raw, rows, cols, x, iters=3)
        print(json.dumps({"ncu_case": "bgemm", "rows": rows, "cols": cols, "M": M, "ms": ms}))
        return
    if args.ncu_case == "bgemm4":
        # config 4's gate/up projection (9728 x 896, int8 g64) over the 320 rows of a verify pass of
        # 64 sequences x 5
        rows, cols, M = 9728, 896, 320
        raw = stored_rows(8, 64, rows, cols, seed=4)
        x = np.random.default_rng(4).standard_normal((M, cols)).astype(np.float32)
        _, ms = ls.bgemm(8, 64, raw, rows, cols, x, iters=3)
        print(json.dumps({"ncu_case": "bgemm4", "rows": rows, "cols": cols, "M": M, "ms": ms}))
        return
    os.makedirs(args.root, exist_ok=True)
    t_path = synth.ensure_lsq(args.root, cfg["shape"], 0, cfg["body"], cfg["embed"], clip=True)
    if args.ncu_case == "pass":
        plen, k = cfg["prompt"], cfg["k"]
        m = ls.Model(t_path, max_ctx=plen + cfg["max_new"] + k + 16)
        prompt = prompt_for(cfg, m.vocab, 0)
        first = m.forward(prompt, want_logits=False)
        block = [first] + prompt[-k:]
        for _ in range(3):
            m.truncate(plen)
            m.verify(block)
        print(json.dumps({"ncu_case": "pass", "verify_passes": 3, "block": len(block)}))
        return
    # gemv: the LM head matrix of the bench model as a standalone GEMV, M = k + 1 rows
    info_m = ls.Model(t_path, max_ctx=64)
    V, h = info_m.vocab, info_m.info.hidden
    rb = info_m.info.embed_row_bytes
    start = os.path.getsize(t_path) - h * 2 - V * rb
    info_m.close()
    raw = np.fromfile(t_path, dtype=np.uint8, count=V * rb, offset=start)
    w = ls.QWeights(cfg["embed"][0], cfg["embed"][1], raw, V, h)
    M = cfg["k"] + 1
    x = torch.randn(M, h, device="cuda")
    y = torch.empty(M, V, device="cuda")
    for _ in range(3):
        w.gemv(x.data_ptr(), M, y.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    print(json.dumps({"ncu_case": "gemv", "rows": V, "cols": h, "M": M, "bytes_per_launch": w.bytes(M)}))



def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(key: str):
    """DRAM bytes (read + write) per launch of a kernel on a bench workload, as an ncu capture of
    that workload measured them (dram__bytes_read.sum + dram__bytes_write.sum). ncu cannot run
    inside the timed region, so the figures are recorded beside the profile summaries in
    profiles/traffic.json, keyed "<kernel>-<workload>"; None when no capture exists."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    v = json.load(open(p)).get(key)
    return float(v["bytes_per_launch"]) if isinstance(v, dict) and v.get("bytes_per_launch") is not None else None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in csv.reader(io.StringIO(out)):
            if len(row) < 9:
                continue
            try:
                sm.append(float(row[1]))
                mx.append(float(row[2]))
            except ValueError:
                continue
            for n, v in zip(names, row[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def setup_dist(args):
    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    dist = None
    if world > 1:
        import torch.distributed as dist

        backend = "nccl" if args.impl == "ours" else "gloo"
        if backend == "nccl":
            import torch

            torch.cuda.set_device(local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=900),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=900))
    return rank, world, local, dist


def barrier(dist):
    if dist is not None:
        dist.barrier()


def reduce_over_ranks(dist, ms: float, tokens: float, device="cpu"):
    """Whole-job figures of a data-parallel run: the slowest rank's device time and the tokens of
    all ranks (every rank takes the same two collectives, in the same order)."""
    import torch

    t_ms = torch.tensor([float(ms)], device=device)
    t_tok = torch.tensor([float(tokens)], device=device)
    per_rank = [float(ms)]
    if dist is not None:
        g = torch.zeros(dist.get_world_size(), device=device)
        dist.all_gather_into_tensor(g, t_ms.clone())
        per_rank = [float(v) for v in g.tolist()]
        dist.all_reduce(t_ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(t_tok, op=dist.ReduceOp.SUM)
    reduce_over_ranks.per_rank_ms = per_rank
    return float(t_ms.item()), float(t_tok.item())


def prompt_for(cfg, vocab, index):
    """Prompt `index` of a config's seeded prompt set. Every rank of a data-parallel run takes the
    same indices, so each GPU does identical work (weak scaling that measures the hardware, not
    the acceptance rate of different prompts)."""
    from layerstream_b200 import synth

    if cfg["repeats"]:
        return synth.make_prompt(cfg["prompt"], vocab, cfg["span"], cfg["repeats"], seed=1000 + index)
    return synth.make_prompt_spans(cfg["prompt"], vocab, cfg["span"], seed=1000 + index)


# ------------------------------------------------------------------------------------------------
# CPU path (oracle): the reference's algorithm restated in C++, timed on the host cores
# ------------------------------------------------------------------------------------------------


def cpu_files(args, cfg, rank, dist):
    """Model files made with the CPU quantizer (bytes identical to the GPU quantizer's)."""
    from layerstream_b200 import synth
    from oracle import oracle as O

    os.makedirs(args.root, exist_ok=True)
    d = synth.ensure_model(args.root, cfg["shape"], 0)

    def lsq(body, embed):
        p = os.path.join(args.root, f"{cfg['shape']}-s0-q{body[0]}g{body[1]}-e{embed[0]}g{embed[1]}-clip.lsq")
        if not os.path.exists(p):
            tmp = p + f".{os.getpid()}.partial"
            O.quantize_model(d, tmp, body, embed, clip=True, threads=os.cpu_count() or 1)
            os.replace(tmp, p)
        return p

    t = d if cfg.get("bf16_target") else lsq(cfg["body"], cfg["embed"])
    dr = lsq(cfg["draft"], cfg["draft"]) if cfg["drafter"] == "model" else None
    return t, dr


def cpu_sample(args, cfg, target_path, draft_path, steps, warmup, keep=None):
    """Times the oracle's decode loop on a bounded sample: prefill once, then `steps` decodes of
    n_tok tokens from the prefilled state. Returns (tokens/s, per-step list, sample text, cores).
    keep (a dict): receives the prefilled CPU model, its greedy first token and the prompt."""
    from oracle import oracle as O

    threads = os.cpu_count() or 1
    plen, k = cfg["prompt"], cfg["k"]
    n_tok = args.cpu_sample_tokens or (2 * (k + 1) + 1)
    max_ctx = plen + cfg["max_new"] + k + 16
    T = O.Model(target_path, quantized=not os.path.isdir(target_path), threads=threads, max_ctx=max_ctx)
    D = O.Model(draft_path, quantized=True, threads=threads, max_ctx=max_ctx) if draft_path else None
    prompt = prompt_for(cfg, T.vocab, 0)
    first = O.forward_argmax(T, prompt)
    if D is not None:
        O.forward_argmax(D, prompt)
    rates = []
    for i in range(warmup + steps):
        T.truncate(plen)
        if D is not None:
            D.truncate(plen)
        toks, st = O.spec_continue(T, D, prompt, first, n_tok, k)
        if i >= warmup:
            rates.append((len(toks) - 1) / max(st["decode_secs"], 1e-9))
    sample = (f"decode of {n_tok} tokens (of {cfg['max_new']}) from the prefilled {plen}-token prompt, "
              f"{cfg['drafter']} drafter, k={k}, {steps} timed samples")
    if keep is not None:
        T.truncate(plen)
        keep.update(model=T, first=first, prompt=prompt)
    return float(np.mean(rates)), rates, sample, threads


def file_digest(path):
    import hashlib

    if os.path.isdir(path):  # an unquantized safetensors model directory
        path = os.path.join(path, "model.safetensors")
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 24), b""):
            h.update(b)
    return h.hexdigest()


def dtype_note(bits):
    """The arithmetic the verify pass computes in."""
    if bits == 16:
        return ("bf16 weights converted exactly to f16 MMA operands (|w| >= 2^-17); activations rounded to f16 MMA "
                "operands; f32 accumulation; f16 KV cache")
    w = (f"int{bits} weights dequantized exactly to f16 ((q - 8) * scale)" if bits == 4 else
         "int8 weights split exactly into two f16 MMA operands (hi + lo = q * scale)")
    return f"u{bits}/bf16-scale weights; {w}; activations rounded to f16 MMA operands; f32 accumulation; f16 KV cache"


def cpu_parity(keep, gpu_tokens, n, tol=2e-2):
    """Token parity of the GPU's decode with the CPU path on the same prompt and model bytes,
    teacher-forced on the GPU's tokens: the CPU model (prefilled) runs one pass over the GPU's
    first n tokens and takes its own greedy choice at every position. A position is checked when
    the CPU path's top-2 logit margin there exceeds tol (the north star's logit tolerance), and
    skipped as a near-tie otherwise."""
    from oracle import oracle as O

    T, first = keep["model"], keep["first"]
    toks = [int(t) for t in gpu_tokens[:n]]
    rows = T.forward_multi(toks[:-1], len(toks) - 1) if len(toks) > 1 else np.zeros((0, T.vocab), np.float32)
    choice = [first] + [int(O.argmax(r)) for r in rows]
    # the margin of the first choice needs the prefill logits: recompute the last prompt position
    T.truncate(len(keep["prompt"]) - 1)
    margins = [0.0] * len(toks)
    lc0 = T.forward(keep["prompt"][-1:])
    for i, r in enumerate([lc0] + list(rows)):
        top2 = np.partition(r, -2)[-2:]
        margins[i] = float(top2[1] - top2[0])
    checked = agreed = skipped = 0
    mismatches = []
    for i, t in enumerate(toks):
        if margins[i] > tol:
            checked += 1
            if choice[i] == t:
                agreed += 1
            else:
                mismatches.append(i)
        else:
            skipped += 1
    return {"checked": checked, "agreed": agreed, "skipped_near_ties": skipped, "positions": len(toks),
            "tolerance": tol, "mismatch_positions": mismatches[:8],
            "method": "teacher-forced on the GPU's decode tokens; CPU restatement on the same .lsq bytes"}


# ------------------------------------------------------------------------------------------------
# CUDA path
# ------------------------------------------------------------------------------------------------


def stored_rows(bits, group, rows, cols, seed):
    """Random stored rows (.lsq row format) with bf16 group scales near 1e-2."""
    rb = cols * bits // 8 + cols // group * 2
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(rows, rb), dtype=np.uint8)
    sc = raw[:, cols * bits // 8:].view(np.uint16)
    sc[:] = (0x3C23 + rng.integers(-64, 64, size=sc.shape)).astype(np.uint16)
    return np.ascontiguousarray(raw.reshape(-1))


def ref_batch(args, cfg):
    """Config 4 on the CPU restatement: a reduced sample (one sequence's prefill and a short
    decode), extrapolated to the batch as per-sequence throughput x 1 (the reference runs sequences
    one after another)."""
    rank, world, local, dist = setup_dist(args)
    if rank != 0:
        barrier(dist)
        return
    c2 = dict(cfg)
    c2["max_new"] = 16
    t_path, _ = cpu_files(args, c2, rank, None)
    v, rates, sample, cores = cpu_sample(args, c2, t_path, None, max(args.steps, 1), 0)
    sample = "reduced sample: one sequence of the batch, " + sample
    line = {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 activations, int8 weights", "data": "synthetic", "config": {"workload": "config4", "config": 4},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    barrier(dist)


def microbench(args):
    """Config 3: the verify-path kernels one at a time on one 0.5B layer's shapes, timed with CUDA
    events two ways. "Stream": back-to-back launches captured in one CUDA graph, each over its own
    replica of the weights (or of the K/V cache), the replicas together at least 256 MB (twice L2),
    so every launch reads from HBM as the layers of a pass do; time = span / launches. "Cold": one launch alone after a 256 MB
    read that evicts L2 (and the TLB), median of the repeats. GEMV: each projection shape x M;
    attention (tensor-core kernel, context split over up to 160 CTAs per kv head, a many-CTA merge):
    KV length sweep 512 .. 32768 with its roofline per length."""
    import torch

    import layerstream_b200 as ls

    rank, world, local, dist = setup_dist(args)
    torch.cuda.set_device(local)
    peak, peak_kind = peaks()
    # L2 eviction before every timed launch by READING 256 MB (a write would leave dirty lines whose
    # write-back the timed kernel would pay for)
    flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()
    gemv = []
    reps = max(args.steps, 3)
    for bits, group in ((8, 64), (4, 32)):
        for name, (rows, cols) in MICRO_SHAPES.items():
            raw = stored_rows(bits, group, rows, cols, seed=rows)
            w = ls.QWeights(bits, group, raw, rows, cols, device=local)
            nrep = int(min(4096, max(2, (256 << 20) // qmat_bytes(rows, cols, bits, group) + 1)))  # as the library picks
            for M in (1, 2, 4, 8, 16):
                xh = np.random.default_rng(M).standard_normal((M, cols)).astype(np.float32)
                # stream: the library's host entry times one CUDA graph of launches over device
                # replicas of the planes (>= 256 MB together)
                _, ms = ls.qgemv(bits, group, raw, rows, cols, xh, iters=2)
                us = ms * 1e3
                x = torch.from_numpy(xh).cuda()
                y = torch.empty(M, rows, device="cuda")
                for _ in range(args.warmup):
                    w.gemv(x.data_ptr(), M, y.data_ptr(), s.cuda_stream)
                ts = []
                for _ in range(reps):
                    flush.sum()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(s)
                    w.gemv(x.data_ptr(), M, y.data_ptr(), s.cuda_stream)
                    e1.record(s)
                    torch.cuda.synchronize()
                    ts.append(e0.elapsed_time(e1))
                us_cold = float(np.median(ts)) * 1e3
                b = w.bytes(M)
                gemv.append({"fmt": f"int{bits}-g{group}", "shape": name, "rows": rows, "cols": cols, "M": M, "us": us,
                             "bytes": b, "gbs": b / us / 1e3, "frac": b / us / 1e3 / peak, "replicas": nrep,
                             "us_cold": us_cold, "gbs_cold": b / us_cold / 1e3})
            del w
    att = []
    heads, kvh, hd, M = 14, 2, 64, 9
    rng = np.random.default_rng(5)
    for L in [512 << i for i in range(7)]:
        pos0 = L - M
        qkv = rng.standard_normal((M, (heads + 2 * kvh) * hd)).astype(np.float32)
        kc = rng.standard_normal((kvh, pos0, hd)).astype(np.float16)
        vc = rng.standard_normal((kvh, pos0, hd)).astype(np.float16)
        _, ms = ls.attention(heads, kvh, hd, pos0, qkv, kc, vc, iters=max(20, reps))
        b = L * kvh * hd * 2 * 2 + M * (heads + 2 * kvh) * hd * 4 + M * heads * hd * 4
        att.append({"kv_len": L, "M": M, "us": ms * 1e3, "bytes": b, "gbs": b / (ms * 1e3) / 1e3,
                    "frac": b / (ms * 1e3) / 1e3 / peak})
    head8 = [g for g in gemv if g["shape"] == "head" and g["fmt"] == "int8-g64" and g["M"] == 8][0]
    line = {"metric": "verify-kernel microbench: LM-head GEMV HBM GB/s (int8 g64, M = 8)", "value": head8["gbs"],
            "unit": "GB/s", "n_gpus": 1, "steps": reps, "warmup": args.warmup, "ms_per_step": head8["us"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/int4 weights, f32 x, f16 KV",
            "data": "synthetic",
            "config": {"workload": "config3: one 0.5B layer's GEMV shapes x M in 1..16, int8 g64 and int4 g32; GQA "
                                   "attention 14/2 heads, hd 64, M = 9, KV 512..32768",
                       "l2": "stream: back-to-back launches (one CUDA graph) over weight / K-V replicas totalling "
                             ">= 256 MB (twice L2), every launch reads HBM; cold (GEMV us_cold): one launch after a "
                             "256 MB read"},
            "roofline": {"bound": "hbm", "kernel": "gemv_tc_kernel (LM head, int8 g64, M = 8)", "achieved": head8["gbs"],
                         "peak": peak, "unit": "GB/s", "frac": head8["gbs"] / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": None},
            "gemv": gemv, "attention": att,
            "gpu_launches": sum(2 * g["replicas"] + 1 + args.warmup + reps for g in gemv)}
    if rank == 0:
        print(json.dumps(line), flush=True)


def qmat_bytes(rows, cols, bits, group):
    """Stored bytes of a group-quantized matrix: packed codes + one bf16 scale per group."""
    return rows * cols * bits // 8 + rows * (cols // group) * 2


def tp_rank_bytes(info, world, rank):
    """Weight bytes one verify pass reads on `rank` of a tensor-parallel split (the library's
    split: q heads evenly, each rank's kv heads, the intermediate dimension in 64-row blocks, the
    head's vocabulary in 32-row tiles); norms are counted whole on every rank."""
    h, hd, L = info.hidden, info.head_dim, info.layers
    hl = info.heads // world
    kvl = info.kv_heads // world if world <= info.kv_heads else 1
    nb = info.inter // 64
    il = 64 * ((rank + 1) * nb // world) - 64 * (rank * nb // world)
    b, g = info.bits, info.group
    layer = (qmat_bytes((hl + 2 * kvl) * hd, h, b, g) + qmat_bytes(h, hl * hd, b, g) + qmat_bytes(2 * il, h, b, g)
             + qmat_bytes(h, il, b, g) + 2 * h * 2 + (hl + 2 * kvl) * hd * 2)
    tiles = (info.vocab + 31) // 32
    t0, t1 = rank * tiles // world, (rank + 1) * tiles // world
    rows = min(info.vocab, 32 * t1) - 32 * t0
    return L * layer + qmat_bytes(rows, h, info.embed_bits, info.embed_group) + h * 4


def class_split(prof):
    """Per launch class of a profiled batch run: share of the pass time and achieved GB/s."""
    tot = prof["pass"]["ms"] or 1e-9
    out = {}
    for c, v in prof.items():
        if c == "pass" or not v["launches"]:
            continue
        out[c] = {"share": v["ms"] / tot, "ms": v["ms"], "launches": v["launches"],
                  "gbs": v["bytes"] / (v["ms"] * 1e-3) / 1e9 if v["ms"] else None}
    out["pass_ms_total"] = prof["pass"]["ms"]
    out["passes"] = prof["pass"]["launches"]
    return out


def batch_bench(args, cfg):
    """Config 4: B independent sequences per GPU through one batched verify pass per decode step
    (ls_batch_spec, prompt-lookup drafter). value = tokens generated after the first, all
    sequences, all ranks, / the slowest rank's decode-loop time; prefill is reported apart."""
    import torch

    import layerstream_b200 as ls
    from layerstream_b200 import synth

    rank, world, local, dist = setup_dist(args)
    torch.cuda.set_device(local)
    os.makedirs(args.root, exist_ok=True)
    if rank == 0:
        path = synth.ensure_lsq(args.root, cfg["shape"], 0, cfg["body"], cfg["embed"], clip=True, device=local)
    barrier(dist)
    if rank != 0:
        path = synth.ensure_lsq(args.root, cfg["shape"], 0, cfg["body"], cfg["embed"], clip=True, device=local)
    B, plen, max_new, k = cfg["batch"], cfg["prompt"], cfg["max_new"], cfg["k"]
    tp = bool(args.tp and cfg.get("stream_slots"))
    slots = None if tp else cfg.get("stream_slots")
    sealed = bool(args.sealed and slots)
    if sealed:
        # the bench model sealed once with the reference's default chunking (1 MiB layer chunks,
        # 512-row table chunks) under a fixed bench key; the file is reused between runs
        key = bytes(range(32))
        spath = path[:-4] + ".sealed"
        if rank == 0 and not os.path.exists(spath):
            ls.seal_model(path, spath + ".tmp", key, b"benchsea", device=local)
            os.replace(spath + ".tmp", spath)
        barrier(dist)
        model = ls.Model(spath, device=local, max_ctx=plen + 64, mode="stream", slots=slots, key=key)
    elif slots:
        model = ls.Model(path, device=local, max_ctx=plen + 64, mode="stream", slots=slots)
    else:
        model = ls.Model(path, device=local, max_ctx=plen + 64)
    V = model.vocab
    # data parallel: every rank decodes its own copy of the same B seeded sequences (identical
    # work per GPU); tensor parallel: the same B sequences split over the ranks' weight shards
    prompts = np.array([prompt_for(cfg, V, i) for i in range(B)], np.uint32)
    tp_arg = None
    if tp and world > 1:
        box = [ls.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tp_arg = (rank, world, box[0])
    batch = ls.Batch(model, B, max_ctx=plen + max_new + k + 16, max_block=k + 1, tp=tp_arg)
    for _ in range(max(args.warmup, 1)):
        batch.spec(prompts, 8, k)
    clocks = Clocks(local)
    barrier(dist)
    clocks.start()
    tokens, decode_s, first_s, passes, acc, dr = 0, 0.0, 0.0, 0, 0, 0
    r0 = model.report()
    for _ in range(max(args.steps, 1)):
        outs, st = batch.spec(prompts, max_new, k)
        tokens += sum(len(o) - 1 for o in outs)
        decode_s += st["decode_secs"]
        first_s += st["first_secs"]
        passes += st["target_passes"]
        acc += st["accepted"]
        dr += st["drafted"]
    clk = clocks.stop()
    r1 = model.report()
    # per-class split of verify passes after the timed region (events add a little time): every
    # sequence prefilled, then 32 (k+1)-row passes of all sequences
    nxt = []
    for i in range(B):
        batch.truncate(i, 0)
        nxt.append(batch.prefill(i, prompts[i]))
    batch.profile_enable(1)
    for _ in range(32):
        _, nxt = batch.verify(np.array([[t] * (k + 1) for t in nxt], np.uint32))
    prof = batch.profile()
    batch.profile_enable(0)
    peer = tp and world > 1 and batch.tp_peer()
    barrier(dist)
    # tensor parallel: every rank emits the same tokens, counted once
    ms_max, tok_all = reduce_over_ranks(dist, decode_s * 1e3, tokens if (rank == 0 or not tp) else 0, device="cuda")
    value = tok_all / (ms_max / 1e3)
    info = model.info
    avg_ctx = plen + max_new / 2
    kv = avg_ctx * info.layers * info.kv_heads * info.head_dim * 2 * 2 * B
    pass_s = decode_s / max(passes, 1)
    peak, peak_kind = peaks()
    streamed = None
    if slots:
        # bytes moved host -> device for weights over the whole run (prefill chunks + verify passes)
        run_s = decode_s + first_s
        streamed = {"slots": slots, "h2d_weight_bytes": r1["bytes_read"] - r0["bytes_read"],
                    "h2d_gbs": (r1["bytes_read"] - r0["bytes_read"]) / max(run_s, 1e-9) / 1e9,
                    "bytes_per_pass": info.weight_bytes, "note": "every pass streams all layers and the head over PCIe"}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / max(args.steps, 1), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": dtype_note(cfg["body"][0]), "data": "synthetic",
            "config": {"workload": f"config4: 0.5b Qwen2 random-init int8 g64, {B} sequences per GPU, {plen}-token prompts, "
                                   f"{max_new} new tokens each, k={k}, lookup drafter, batched verify",
                       "config": 4, "batch_per_gpu": B, "global_batch": B * world,
                       "parallelism": f"dp{world} (independent sequences, no collective)",
                       "timing": "host wall time of the decode loop (all sequences), prefill excluded"},
            "clocks": clk,
            "e2e": {"value": tok_all / ((ms_max / 1e3) + first_s / max(args.steps, 1)), "unit": UNIT,
                    "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                    "includes": "prefill of all sequences + decode through ls_batch_spec, host buffers"},
            "gpu_launches": int(passes * (2 + 5 * info.layers + 2)),
            "roofline": {"bound": "hbm", "kernel": "batched verify pass (separate kernels, KV-bound attention)",
                         "achieved": (info.weight_bytes + kv) / pass_s / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": (info.weight_bytes + kv) / pass_s / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": None, "algorithmic_bytes_per_launch": info.weight_bytes + kv,
                         "avg_launch_us": pass_s * 1e6, "launches_per_pass": 2 + 5 * info.layers + 2},
            "spec": {"tokens_per_pass": tokens / max(passes, 1) / B, "accepted_over_drafted": acc / max(dr, 1),
                     "target_passes": passes, "prefill_s": first_s / max(args.steps, 1)},
            "streaming": streamed, "per_rank_ms": reduce_over_ranks.per_rank_ms,
            "classes": class_split(prof)}
    if slots:
        # streamed weights: the bound is the host-to-device link, not HBM
        pcie = 64.0  # GB/s, nominal PCIe 5.0 x16 per direction (no measured figure on this pool)
        line["roofline"] = {"bound": "h2d", "kernel": "weight stream (cudaMemcpyAsync of layers and head chunks, 2 slots)",
                            "achieved": streamed["h2d_gbs"], "peak": pcie, "unit": "GB/s", "frac": streamed["h2d_gbs"] / pcie,
                            "peak_source": "nominal PCIe 5.0 x16", "traffic": None,
                            "algorithmic_bytes_per_launch": info.weight_bytes, "avg_launch_us": pass_s * 1e6}
        line["config"]["workload"] = (f"config5: 3b Qwen2 random-init int4 g32, {B} sequences, {plen}-token prompts, "
                                      f"{max_new} new tokens, k={k}, lookup drafter, {slots}-slot layer streaming from pinned host"
                                      + (", sealed file (ChaCha20-Poly1305 1 MiB chunks, opened on the GPU after each copy)"
                                         if sealed else ""))
        if sealed:
            line["sealed"] = {"cipher": "ChaCha20-Poly1305 (RFC 8439), chunks opened on the GPU", "layer_chunk": 1 << 20,
                              "embed_chunk_rows": 512}
        line["config"]["config"] = 5
        line["dtype"] = dtype_note(4)
    if tp:
        # per rank: its shard of the weights and the K/V of its kv heads; the pass also carries
        # 2 all-reduces per layer and one all-gather over NVLink (NCCL)
        kvl = info.kv_heads // world if world <= info.kv_heads else 1
        kv_r = avg_ctx * info.layers * kvl * info.head_dim * 2 * 2 * B
        w_r = max(tp_rank_bytes(info, world, r) for r in range(world))
        ar_bytes = 2 * info.layers * B * (k + 1) * info.hidden * 4
        line["scaling"] = "strong"
        line["config"].update({
            "workload": (f"config5b: 3b Qwen2 random-init int4 g32, {B} sequences, {plen}-token prompts, {max_new} new "
                         f"tokens, k={k}, lookup drafter, resident, tensor parallel over {world} GPU(s)"),
            "config": 5, "global_batch": B, "batch_per_gpu": B,
            "parallelism": (f"tp{world}: column-parallel QKV (q heads) and gate/up, row-parallel O and down summed "
                            + ("through the peers' memory over NVLink (reduction fused into the next RMSNorm/operand kernel)"
                               if peer else "with NCCL all-reduce")
                            + ", vocabulary-parallel head with an all-gather of per-rank maxima")
                           if world > 1 else "single GPU (tp1)"})
        line["dtype"] = dtype_note(4)
        # per layer: prep, QKV, attention, O, prep, gate/up, down (+ 2 adds with NCCL); per pass:
        # embedding, head prep, head, row maxima, acceptance
        per_layer = 7 if (world == 1 or peer) else 9
        line["gpu_launches"] = int(passes * (per_layer * info.layers + 5))
        line["roofline"] = {"bound": "hbm", "kernel": "tensor-parallel verify pass on the busiest rank (separate kernels)",
                            "achieved": (w_r + kv_r) / pass_s / 1e9, "peak": peak, "unit": "GB/s",
                            "frac": (w_r + kv_r) / pass_s / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
                            "traffic": None, "algorithmic_bytes_per_launch": w_r + kv_r, "avg_launch_us": pass_s * 1e6,
                            "allreduce_bytes_per_pass": ar_bytes if world > 1 else 0,
                            "collectives_per_pass": 2 * info.layers + 1 if world > 1 else 0}
    if rank == 0:
        print(json.dumps(line), flush=True)
    batch.close()
    model.close()


def main():
    args = parse()
    cfg = dict(CONFIGS[args.config])
    if cfg.get("batch"):
        if args.impl == "reference":
            ref_batch(args, cfg)
            return
        batch_bench(args, cfg)
        return
    if cfg.get("micro"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "config 3 is a GPU kernel microbenchmark; the reference's "
                                                                  "CPU kernels are timed through configs 1 and 2"}))
            return
        microbench(args)
        return
    if args.drafter:
        cfg["drafter"] = args.drafter
    if args.target == "bf16":
        cfg["bf16_target"] = True
        cfg["body"] = cfg["embed"] = (16, 0)
    if args.ncu_case:
        ncu_case(args, cfg)
        return
    rank, world, local, dist = setup_dist(args)
    wname = "bf16 (unquantized)" if cfg.get("bf16_target") else f"int{cfg['body'][0]} g{cfg['body'][1]}"
    workload = (f"config{args.config}: {cfg['shape']} Qwen2 random-init {wname}, "
                f"{cfg['prompt']}-token prompt, {cfg['max_new']} new tokens, k={cfg['k']}, batch 1 per GPU, "
                f"{cfg['drafter']} drafter")
    base_cfg = {"workload": workload, "config": args.config, "model": f"qwen2-{cfg['shape']}-arch random-init",
                "weights": "bf16" if cfg.get("bf16_target") else f"int{cfg['body'][0]}-g{cfg['body'][1]}",
                "embed": "bf16" if cfg.get("bf16_target") else f"int{cfg['embed'][0]}-g{cfg['embed'][1]}",
                "prompt_tokens": cfg["prompt"], "max_new": cfg["max_new"], "k": cfg["k"], "drafter": cfg["drafter"],
                "global_batch": world, "parallelism": f"dp{world} (independent sequences, no collective)",
                "l2": "inputs larger than L2 (weights streamed from HBM every pass)"}

    if args.impl == "reference":
        if rank != 0:
            barrier(dist)
            return
        t_path, d_path = cpu_files(args, cfg, rank, None)
        v, rates, sample, cores = cpu_sample(args, cfg, t_path, d_path, args.steps, args.warmup)
        line = {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 activations, int4/int8 weights", "data": "synthetic", "config": base_cfg,
                "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
                "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        barrier(dist)
        return

    import torch

    import layerstream_b200 as ls
    from layerstream_b200 import synth

    torch.cuda.set_device(local)
    os.makedirs(args.root, exist_ok=True)
    if rank == 0:
        t_path = (synth.ensure_model(args.root, cfg["shape"], 0) if cfg.get("bf16_target") else
                  synth.ensure_lsq(args.root, cfg["shape"], 0, cfg["body"], cfg["embed"], clip=True, device=local))
        d_path = synth.ensure_lsq(args.root, cfg["shape"], 0, cfg["draft"], cfg["draft"], clip=True,
                                  device=local) if cfg["drafter"] == "model" else None
    barrier(dist)
    if rank != 0:
        t_path = (synth.ensure_model(args.root, cfg["shape"], 0) if cfg.get("bf16_target") else
                  synth.ensure_lsq(args.root, cfg["shape"], 0, cfg["body"], cfg["embed"], clip=True, device=local))
        d_path = synth.ensure_lsq(args.root, cfg["shape"], 0, cfg["draft"], cfg["draft"], clip=True,
                                  device=local) if cfg["drafter"] == "model" else None

    plen, k, max_new = cfg["prompt"], cfg["k"], cfg["max_new"]
    max_ctx = plen + max_new + k + 16
    target = ls.Model(t_path, device=local, max_ctx=max_ctx)
    draft = ls.Model(d_path, device=local, max_ctx=max_ctx) if d_path else None
    V = target.vocab
    info = target.info
    prompt = prompt_for(cfg, V, 0)
    stream = torch.cuda.ExternalStream(target.stream, device=torch.device("cuda", local))

    first = target.forward(prompt, want_logits=False)
    if draft is not None:
        draft.forward(prompt, want_logits=False)

    def step():
        target.truncate(plen)
        if draft is not None:
            draft.truncate(plen)
        toks, st = ls.spec_continue(target, draft, prompt, first, max_new, k)
        last_tokens[:] = toks
        return len(toks) - 1, st

    last_tokens = []
    for _ in range(args.warmup):
        step()

    passes0 = target.report()["passes"] + (draft.report()["passes"] if draft else 0)
    clocks = Clocks(local)
    barrier(dist)
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    tokens, stats = 0, []
    for _ in range(args.steps):
        n, st = step()
        tokens += n
        stats.append(st)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier(dist)
    ms = e0.elapsed_time(e1)
    passes = target.report()["passes"] + (draft.report()["passes"] if draft else 0) - passes0
    # profiled samples after the timed region: CUDA events around every launch (roofline), then
    # the persistent pass kernel's barrier timeline (per-phase split; it slows the pass a little)
    target.profile_enable(1)
    step()
    prof = target.profile()
    prof_tl = None
    if info.persistent_pass:
        target.profile_enable(2)
        step()
        prof_tl = target.profile()
    target.profile_enable(0)
    ms_max, tok_all = reduce_over_ranks(dist, ms, tokens, device="cuda")
    value = tok_all / (ms_max / 1e3)

    # e2e: the whole public call (prefill + decode) from host buffers
    e2e_ms, e2e_tok = 0.0, 0
    r0 = target.report()
    for _ in range(args.e2e_steps):
        target.reset()
        if draft is not None:
            draft.reset()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        toks, _ = ls.speculative_greedy(target, draft, prompt, max_new, k)
        e2e_ms += (time.perf_counter() - t0) * 1e3
        e2e_tok += len(toks) - 1
    r1 = target.report()
    t2 = torch.tensor([e2e_ms, float(e2e_tok)], device="cuda")
    if dist is not None:
        mx = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t2, op=dist.ReduceOp.SUM)
        e2e_ms = float(mx.item())
    e2e_val = float(t2[1].item()) / (e2e_ms / 1e3) if e2e_ms > 0 else None
    h2d = (r1["h2d_bytes"] - r0["h2d_bytes"]) // max(args.e2e_steps, 1)
    d2h = (r1["d2h_bytes"] - r0["d2h_bytes"]) // max(args.e2e_steps, 1)

    # roofline of the dominant kernel (live CUDA-event timing of its launches). With the persistent
    # pass kernel a verify pass is one launch: algorithmic bytes = weights + the K/V rows read and
    # written at that pass's context. Otherwise the tensor-core GEMV launches dominate: QKV, O,
    # gate/up and down on every layer (timed on one sampled layer, times L) plus the LM head.
    peak, peak_kind = peaks()
    L = info.layers
    per_pass = {}
    for c, p in prof.items():
        if c == "pass" or not p["launches"]:
            continue
        mult = 1 if c == "head" else L
        per_pass[c] = (p["bytes"] / p["launches"] * mult, p["ms"] / p["launches"] * mult, mult)
    roof = None
    gemv_c = [c for c in ("qkv", "o", "gate_up", "down", "head") if c in per_pass]
    if info.persistent_pass and prof["pass"]["launches"]:
        pp = prof["pass"]
        b, t_ms = pp["bytes"] / pp["launches"], pp["ms"] / pp["launches"]
        achieved = b / (t_ms / 1e3) / 1e9
        phases = {}
        if prof_tl is not None:
            for c in ("qkv", "attention", "o", "gate_up", "down", "head"):
                q = prof_tl[c]
                if q["launches"]:
                    phases[c] = {"us": q["ms"] * 1e3 / q["launches"], "busy_us": q["busy_ms"] * 1e3 / q["launches"],
                                 "gbs": q["bytes"] / q["ms"] * 1e3 / 1e9 if q["ms"] > 0 else None,
                                 "per": "layer" if c != "head" else "pass",
                                 "critical_cta_us": dict(zip(CRIT_SEGMENTS, (v * 1e3 / q["launches"] for v in q["crit_ms"])))}
        roof = {"bound": "hbm", "kernel": "pass_kernel (one persistent launch per verify pass)", "achieved": achieved,
                "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": profile_traffic(f"pass_kernel-config{args.config}"), "algorithmic_bytes_per_launch": b,
                "avg_launch_us": t_ms * 1e3,
                "launches_per_pass": 1, "phases": phases}
        gemv_c = []
    if gemv_c:
        b = sum(per_pass[c][0] for c in gemv_c)
        t_ms = sum(per_pass[c][1] for c in gemv_c)
        n = sum(per_pass[c][2] for c in gemv_c)
        achieved = b / (t_ms / 1e3) / 1e9
        traffic = profile_traffic("gemv-pass")
        roof = {"bound": "hbm", "kernel": "gemv_tc_kernel (all launches of a verify pass)", "achieved": achieved,
                "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": traffic, "algorithmic_bytes_per_launch": b / n, "avg_launch_us": t_ms * 1e3 / n,
                "launches_per_pass": n,
                "per_class": {c: {"gbs": per_pass[c][0] / (per_pass[c][1] / 1e3) / 1e9,
                                  "us_per_launch": per_pass[c][1] * 1e3 / per_pass[c][2]} for c in per_pass}}
    vstep = None
    pp = prof["pass"]
    if pp["launches"]:
        avg_ctx = plen + max_new / 2
        wbytes = info.weight_bytes
        kvbytes = avg_ctx * L * info.kv_heads * info.head_dim * 2 * 2
        pass_s = pp["ms"] / pp["launches"] / 1e3
        vstep = {"bytes_per_pass": wbytes + kvbytes, "avg_pass_us": pass_s * 1e6, "achieved_gbs": (wbytes + kvbytes) / pass_s / 1e9,
                 "frac": (wbytes + kvbytes) / pass_s / 1e9 / peak,
                 "kernel_share_est": ({c: per_pass[c][1] / (pp["ms"] / pp["launches"]) for c in per_pass}
                                      if not info.persistent_pass else None)}
    acc = sum(s["accepted"] for s in stats)
    dr = sum(s["drafted"] for s in stats)
    tp = sum(s["target_passes"] for s in stats)

    cpu, parity = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            tpc, dpc = cpu_files(args, cfg, rank, None)
            keep = {}
            v, _, sample, cores = cpu_sample(args, cfg, tpc, dpc, steps=10, warmup=1, keep=keep)
            cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
            # outside every timed region: the GPU's decoded tokens against the CPU path's choices
            parity = cpu_parity(keep, last_tokens, min(len(last_tokens), 48))
            parity["model_bytes_identical"] = file_digest(tpc) == file_digest(t_path)
        except Exception as e:  # the baseline is reported, never required
            cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {e}"}

    kernels_per_pass = 2 + 5 * L
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype_note(cfg["body"][0]), "data": "synthetic",
        "config": base_cfg, "clocks": clk, "parity": parity,
        "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "steps": args.e2e_steps, "includes": "prefill + decode through ls_speculative_greedy, host buffers"},
        "gpu_launches": int(passes * (1 if info.persistent_pass else kernels_per_pass)),
        "roofline": roof, "verify_step": vstep,
        "spec": {"tokens_per_pass": tokens / max(tp, 1), "accepted_over_drafted": acc / max(dr, 1), "target_passes": tp},
        "per_rank_ms": reduce_over_ranks.per_rank_ms,
        "cpu_baseline": cpu,
    }
    if args.profile and rank == 0:
        print(json.dumps(prof, indent=1), file=sys.stderr)
    if rank == 0:
        print(json.dumps(line), flush=True)
    target.close()
    if draft is not None:
        draft.close()
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
