"""Tensor-parallel batch (config 5b) on two GPUs against the CPU path (needs 2 B200s).

Each rank holds its q heads (and their kv head), half of the intermediate dimension and half of
the vocabulary; O and down are summed over the ranks (by default through the peers' memory over
NVLink, with LS_TP_P2P=0 by the NCCL all-reduce) and the LM head's per-rank first maxima are
gathered. Every rank must emit the same tokens, and they must match the CPU path
wherever the top-2 logit margin exceeds the north-star tolerance.
"""
import os

import numpy as np
import pytest

import fixtures as F
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2
WORLD = 2


def _rank(rank, world, path, uid_q, out_q, prompts, max_new, k, peer):
    os.environ["LS_TP_P2P"] = "1" if peer else "0"
    import torch

    import layerstream_b200 as ls

    torch.cuda.set_device(rank)
    if rank == 0:
        uid = ls.tp_unique_id()
        for _ in range(world - 1):
            uid_q.put(uid)
    else:
        uid = uid_q.get(timeout=120)
    try:
        m = ls.Model(path, device=rank, max_ctx=64)
        b = ls.Batch(m, len(prompts), max_ctx=64, max_block=k + 1, tp=(rank, world, uid))
        if b.tp_peer() != peer:
            raise AssertionError(f"peer reduction {'off' if peer else 'on'} against LS_TP_P2P")
        got, st = b.spec(np.array(prompts, np.uint32), max_new, k)
        out_q.put((rank, got, None))
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, None, repr(e)))


def _cpu_tokens(path, prompt, n):
    c = O.Model(path, quantized=True, threads=4, max_ctx=64)
    logits = c.forward(prompt)
    toks, margins = [], []
    for i in range(n):
        srt = np.sort(logits)
        toks.append(int(np.argmax(logits)))
        margins.append(float(srt[-1] - srt[-2]))
        if i + 1 < n:
            logits = c.forward([toks[-1]])
    return toks, margins


def _run_tp(path, prompts, max_new, k, peer):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, WORLD, path, uid_q, out_q, prompts, max_new, k, peer)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            r, got, err = out_q.get(timeout=600)
            res[r] = (got, err)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(WORLD):
        assert res[r][1] is None, res[r][1]
    assert res[0][0] == res[1][0]  # every rank emits the same tokens
    return res[0][0]


def test_two_rank_tensor_parallel_batch_matches_the_cpu_path():
    import torch

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    from layerstream_b200 import synth

    synth.SHAPES["tp-test"] = dict(hidden_size=2048, num_attention_heads=16, num_key_value_heads=2,
                                   intermediate_size=256, num_hidden_layers=2, vocab_size=1000, rope_theta=1e6,
                                   max_position_embeddings=4096)
    d = F.TempDir("gpu-tp").path
    synth.write_random_model(d, "tp-test", 5)
    path = os.path.join(d, "tp.lsq")
    O.quantize_model(d, path, (4, 32), (4, 32), clip=True)
    prompts = [[(11 * i + 17 * s + 3) % 1000 for i in range(10)] for s in range(4)]
    max_new, k = 12, 4
    peer = _run_tp(path, prompts, max_new, k, True)
    nccl = _run_tp(path, prompts, max_new, k, False)
    # two ranks: the peer sum y0 + y1 and the fused norm equal NCCL's sum and the separate prep
    assert peer == nccl
    for pr, g in zip(prompts, peer):
        toks, margins = _cpu_tokens(path, pr, max_new)
        for i, (t, mg) in enumerate(zip(toks, margins)):
            if mg <= TOL:
                break
            assert g[i] == t, (pr, i)


def _rank_fail(rank, world, path, uid_q, out_q, inject_rank):
    # failure-path test: NVLS off (a rank that stops must not leave multicast objects behind)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    import layerstream_b200 as ls

    torch.cuda.set_device(rank)
    if rank == 0:
        uid = ls.tp_unique_id()
        for _ in range(world - 1):
            uid_q.put(uid)
    else:
        uid = uid_q.get(timeout=120)
    try:
        m = ls.Model(path, device=rank, max_ctx=64)
        b = ls.Batch(m, 2, max_ctx=64, max_block=5, tp=(rank, world, uid))
        firsts = [b.prefill(i, [(7 * i + j) % 1000 for j in range(9)]) for i in range(2)]
        blocks = np.array([[f, 1, 2, 3, 4] for f in firsts], np.uint32)
        want = b.verify(blocks)
        for i in range(2):
            b.truncate(i, 9)
        if rank == inject_rank:
            b.inject_error()
        codes = []
        for _ in range(2):  # the injected pass, then one more: the ranks stayed in step
            try:
                codes.append(("ok", b.verify(blocks)))
            except ls.LayerstreamError as e:
                codes.append((e.code, None))
        b.close()  # the failed communicator is aborted, not drained
        m.close()
        out_q.put((rank, (want, codes), None))
    except Exception as e:
        out_q.put((rank, None, repr(e)))


def test_an_error_on_one_rank_stops_every_rank_on_the_same_pass():
    # one rank's device error must not leave its peer waiting in the next collective
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    from layerstream_b200 import synth

    synth.SHAPES["tp-fail"] = dict(hidden_size=512, num_attention_heads=8, num_key_value_heads=2,
                                   intermediate_size=256, num_hidden_layers=2, vocab_size=1000, rope_theta=1e6,
                                   max_position_embeddings=4096)
    d = F.TempDir("gpu-tp-fail").path
    synth.write_random_model(d, "tp-fail", 6)
    path = os.path.join(d, "tp.lsq")
    O.quantize_model(d, path, (4, 32), (4, 32), clip=True)
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_fail, args=(r, WORLD, path, uid_q, out_q, 1)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            r, got, err = out_q.get(timeout=300)
            res[r] = (got, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(WORLD):
        assert res[r][1] is None, res[r][1]
        want, codes = res[r][0]
        assert codes[0] == (-4, None), (r, codes)  # LS_ERR_DEVICE on both ranks, same pass
        assert codes[1] == ("ok", want), (r, codes)
