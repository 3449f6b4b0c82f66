"""The paged K/V cache (needs a B200).

The reference keeps one dense [max_ctx x kv_dim] cache per layer and rolls it back by a length
(src/model.rs:67-68,137-140). Here each layer has a pool of fixed-size pages shared by the
sequences of a model or batch, and each sequence a page table; pages are taken as a sequence grows
and returned when it is truncated or reset. Checked here:

* the attention kernels read K/V through an arbitrary (shuffled) page table, with page sizes that
  do not divide the context, and match the float64 restatement of src/model.rs:261-282 at contexts
  of about 512, 4096 and 32768; the block's new rows land in the right pages;
* the page size never changes a model's results (bit-identical logits and tokens);
* rollbacks return pages to the pool, and a batch whose sequences reuse each other's freed pages
  (a fragmented table) decodes exactly like fresh single-sequence models.
"""

import os

import numpy as np
import pytest

import fixtures as F
import layerstream_b200 as ls
from oracle import oracle as O
from test_gpu_attention import reference, rope_tab, rotate

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("heads,kvh,hd,pos0,M,page", [(14, 2, 64, 507, 5, 16), (14, 2, 64, 4091, 9, 64),
                                                       (14, 2, 64, 32763, 5, 256), (16, 2, 128, 1000, 5, 32),
                                                       (4, 2, 16, 65, 33, 8)])
def test_attention_through_a_shuffled_page_table(heads, kvh, hd, pos0, M, page):
    rng = np.random.default_rng(pos0 + page)
    ctx = pos0 + M
    need = -(-ctx // page)
    num_pages = need + 5  # pages the table never names hold garbage
    table = rng.permutation(num_pages)[:need].astype(np.int32)
    qkv = rng.standard_normal((M, (heads + 2 * kvh) * hd)).astype(np.float32)
    k_pool = rng.standard_normal((kvh, num_pages, page, hd)).astype(np.float16)
    v_pool = rng.standard_normal((kvh, num_pages, page, hd)).astype(np.float16)
    k_before = k_pool.copy()
    p = np.arange(pos0)
    kc = k_pool[:, table[p // page], p % page]  # the dense cache the table describes
    vc = v_pool[:, table[p // page], p % page]
    got, _ = ls.attention_paged(heads, kvh, hd, pos0, qkv, k_pool, v_pool, page, table)
    want = reference(heads, kvh, hd, pos0, qkv, kc, vc)
    assert np.max(np.abs(got - want)) < 2e-4 * (1 + np.max(np.abs(want)))
    # the block's rows (K rotated, both rounded to f16) were written into their pages
    H, KV = heads * hd, kvh * hd
    pos = pos0 + np.arange(M)
    cos, sin = rope_tab(hd, ctx)
    k = qkv[:, H:H + KV].astype(np.float64).reshape(M, kvh, hd)
    k = rotate(k, cos[pos][:, None, :], sin[pos][:, None, :]).astype(np.float32).astype(np.float16).transpose(1, 0, 2)
    v = qkv[:, H + KV:].reshape(M, kvh, hd).astype(np.float16).transpose(1, 0, 2)
    kw = k_pool[:, table[pos // page], pos % page]
    vw = v_pool[:, table[pos // page], pos % page]
    assert np.array_equal(vw, v)
    assert np.max(np.abs(kw.astype(np.float32) - k.astype(np.float32))) <= 2e-3 * np.max(np.abs(k.astype(np.float32)))
    # pages outside the context are untouched
    unused = np.setdiff1d(np.arange(num_pages), table)
    assert np.array_equal(k_pool[:, unused], k_before[:, unused])


@pytest.fixture(scope="module")
def tiny():
    d = F.TempDir("gpu-paged").path
    F.write_tiny_model(d, 13)
    p = os.path.join(d, "q8g32.lsq")
    O.quantize_model(d, p, (8, 32), (8, 32), clip=True)
    yield p


def open_with_page(path, page, **kw):
    old = os.environ.get("LS_KV_PAGE")
    os.environ["LS_KV_PAGE"] = str(page)
    try:
        return ls.Model(path, **kw)
    finally:
        if old is None:
            del os.environ["LS_KV_PAGE"]
        else:
            os.environ["LS_KV_PAGE"] = old


def run_script(m):
    """Prefill, verify blocks with rejections, truncate, decode: logits and tokens of every step."""
    outs = [m.forward(F.PROMPT + list(range(40, 140)))]
    a = m.last_argmax
    for blk in ([a, 5, 6, 7, 8], [9, 10, 11], [12] * 9):
        m.verify(blk)
        outs.append(m.forward([3]))
    m.truncate(m.pos - 7)
    outs.append(m.forward_multi([1, 2, 3, 4], 4))
    return outs


def test_the_page_size_does_not_change_the_results(tiny):
    ref = None
    for page in (64, 8, 16, 256):
        m = open_with_page(tiny, page, max_ctx=300)
        assert m.info.kv_page == page
        outs = run_script(m)
        m.close()
        flat = np.concatenate([o.reshape(-1) for o in outs]).view(np.uint32)
        if ref is None:
            ref = flat
        else:
            assert np.array_equal(flat, ref), page


def test_speculative_decoding_is_unchanged_by_the_page_size(tiny):
    want = None
    for page in (8, 64):
        t = open_with_page(tiny, page, max_ctx=200)
        got, _ = ls.speculative_greedy(t, None, F.PROMPT, 40, 4)
        t.close()
        if want is None:
            want = got
        assert got == want, page


def test_rollbacks_return_pages_to_the_pool(tiny):
    m = open_with_page(tiny, 16, max_ctx=300)
    assert m.info.kv_pages_total == -(-300 // 16)
    assert m.info.kv_pages_used == 0
    m.forward(list(range(1, 50)))  # 49 positions: 4 pages
    assert m.info.kv_pages_used == 4
    m.verify([7] + [1] * 20)  # pages for 70 positions while verifying, then pos = 49 + m + 1
    assert m.info.kv_pages_used == -(-m.pos // 16)
    m.truncate(16)
    assert m.info.kv_pages_used == 1
    m.reset()
    assert m.info.kv_pages_used == 0
    m.close()


def test_a_batch_reusing_freed_pages_decodes_like_a_fresh_batch(tiny):
    # sequence 0 grows and is rolled back; its freed pages go to sequences 1 and 2, and sequence 0
    # then takes whatever is left: the tables end up out of order, the results must not change
    prompts = [F.PROMPT + list(range(200, 260)), [9, 8, 7, 6, 5, 4] * 7, [100, 200, 300, 400, 500, 1] * 5]
    old = os.environ.get("LS_KV_PAGE")
    os.environ["LS_KV_PAGE"] = "8"
    try:
        base = ls.Model(tiny, max_ctx=256)
        frag = ls.Batch(base, 3, max_ctx=160, max_block=9)
        fresh = ls.Batch(base, 3, max_ctx=160, max_block=9)
    finally:
        if old is None:
            del os.environ["LS_KV_PAGE"]
        else:
            os.environ["LS_KV_PAGE"] = old
    frag.prefill(0, prompts[0])
    frag.truncate(0, 3)
    f1, f2 = frag.prefill(1, prompts[1]), frag.prefill(2, prompts[2])
    frag.truncate(0, 0)
    got_first = [frag.prefill(0, prompts[0]), f1, f2]
    want_first = [fresh.prefill(i, pr) for i, pr in enumerate(prompts)]
    assert got_first == want_first
    for step in range(3):
        blocks = np.array([[f] + [1, 2, 3, (4 + step) % 600] for f in want_first], np.uint32)
        got = frag.verify(blocks)
        want = fresh.verify(blocks)
        assert got == want, step
        assert [frag.pos(i) for i in range(3)] == [fresh.pos(i) for i in range(3)]
        want_first = list(want[1])
    frag.close()
    fresh.close()
    base.close()
