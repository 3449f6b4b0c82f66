"""Byte accounting of the tensor-parallel bench line (CPU, no GPU).

`bench.tp_rank_bytes` gives the weight bytes one rank reads per verify pass; the TP line's roofline
divides the busiest rank's bytes by the pass time. Its shards must add up, over the ranks, to the
single-GPU bytes plus exactly what every rank holds a copy of: the norms (whole on every rank) and,
when there are more ranks than kv heads, the replicated kv heads' K/V rows and biases.
"""
import os
import sys
from types import SimpleNamespace

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def shape_3b(bits=4, group=32):
    return SimpleNamespace(hidden=2048, head_dim=128, layers=36, heads=16, kv_heads=2, inter=11008, bits=bits, group=group,
                           vocab=151936, embed_bits=bits, embed_group=group)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("fmt", [(4, 32), (8, 64)])
def test_rank_shards_add_up_to_the_single_gpu_bytes(world, fmt):
    info = shape_3b(*fmt)
    one = bench.tp_rank_bytes(info, 1, 0)
    total = sum(bench.tp_rank_bytes(info, world, r) for r in range(world))
    h, hd, L = info.hidden, info.head_dim, info.layers
    kvl = info.kv_heads // world if world <= info.kv_heads else 1
    extra_kv_rows = 2 * (world * kvl - info.kv_heads) * hd  # replicated K and V rows per layer
    replicated = (world - 1) * (L * 2 * h * 2 + h * 4)  # both RMSNorm weights per layer, the final norm
    replicated += L * (bench.qmat_bytes(extra_kv_rows, h, *fmt) + extra_kv_rows * 2)
    assert total == one + replicated


def test_single_gpu_bytes_are_the_model_matrices():
    info = shape_3b()
    h, hd, L, I = info.hidden, info.head_dim, info.layers, info.inter
    q = bench.qmat_bytes
    layer = (q((info.heads + 2 * info.kv_heads) * hd, h, 4, 32) + q(h, info.heads * hd, 4, 32) + q(2 * I, h, 4, 32)
             + q(h, I, 4, 32) + 2 * h * 2 + (info.heads + 2 * info.kv_heads) * hd * 2)
    assert bench.tp_rank_bytes(info, 1, 0) == L * layer + q(info.vocab, h, 4, 32) + h * 4
    # int4 g32 stores 0.5 byte per weight plus a bf16 scale per 32: 0.5625 byte per weight
    assert q(32, 2048, 4, 32) == 32 * 2048 * 9 // 16


def test_the_busiest_rank_sets_the_roofline_bytes():
    info = shape_3b()
    for world in (2, 4, 8):
        per = [bench.tp_rank_bytes(info, world, r) for r in range(world)]
        # the split is near even: the largest shard is within one 64-row block and one 32-row head
        # tile of the smallest
        slack = info.layers * (bench.qmat_bytes(128, info.hidden, 4, 32) + bench.qmat_bytes(info.hidden, 64, 4, 32))
        slack += bench.qmat_bytes(32, info.hidden, 4, 32)
        assert max(per) - min(per) <= slack
