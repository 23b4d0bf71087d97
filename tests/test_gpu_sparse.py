"""GPU: page-sparse decode over the codes (LC_STORE_DIGEST + LC_SPARSE_PAGES).

The oracle restates the policy of sdpa_page_sparse
(native_attention.rs:217-329) on the stored codes (pyoracle.quest_select):
digest = min / max of f32(c[code]) * sigma per 64-token page, bound = max
over the query group of sum_d max(q'_d max_d, q'_d min_d), first page and 4
most recent full pages pinned, keep = max(pages / 8, 64), plus the
undigested tail. The GPU output must match the oracle's attention over that
token set (orc_sc_attend_mask) at the decode tolerance. The data is checked
to leave no near-tie at the selection boundary. Queries use the configs'
scale (std 1/sqrt(128)), and one test the peaked regime of the reference's
Gemma call (q ~ N(0, 1), scale 1). A sequence below 16384 keys in the same
call is dense. Config 2's geometry (3-bit K / 2-bit V, head_dim 256) runs
through the general digest and the tensor-core kernel's tile map.
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu

DIM, HKV, HQ = 128, 8, 32


def _cache(lc, orc, lens, flags=None, max_size=0, dim=DIM, kb=4, vb=4, hkv=HKV):
    """The cache and the K codec's tables (the V codec's too when the bit
    widths differ: returned as t.v)."""
    t = orc.Tables.generate(dim, kb, 64, 42)
    c = lc.TurboQuantCompressor.from_tables(t.R, t.bounds, t.cents, t.proj)
    tv, cv = t, None
    if vb != kb:
        tv = orc.Tables.generate(dim, vb, 64, 42)
        cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    t.v, t.bits, t.dim, t.hkv = tv, kb, dim, hkv
    pages = (max(lens) + 400 + 255) // 256 + 2
    cache = lc.CudaKvCache(1, hkv, dim, c, cv, max_seqs=len(lens), max_pages=len(lens) * pages + 8,
                           max_pages_per_seq=pages,
                           store_flags=lc.LC_STORE_DIGEST if flags is None else flags,
                           layer_max_size=[max_size], layer_keep=[0])
    return t, cache


def _fill(cache, orc, t, lens, seed):
    """Random keys with 120 pages per head scaled by distinct factors 2 + 0.05 k:
    scaling a key scales its sigma and keeps its codes, so those pages' bounds
    separate cleanly and the selection boundary has no near-tie."""
    refs, kv = [], []
    rng = np.random.default_rng(seed)
    hkv, dim = t.hkv, t.dim
    for b, n in enumerate(lens):
        K = helpers.kv(orc, seed + 2 * b, 1, hkv, n, dim)
        V = helpers.kv(orc, seed + 2 * b + 1, 1, hkv, n, dim)
        P = n // 64
        if P > 130:
            for h in range(hkv):
                for k, p in enumerate(rng.choice(np.arange(1, P - 4), size=120, replace=False)):
                    K[0, h, p * 64:(p + 1) * 64] *= np.float32(2.0 + 0.05 * k)
        for c0 in range(0, n, 4096):
            c1 = min(n, c0 + 4096)
            cache.append(0, [b], np.ascontiguousarray(K[:, :, c0:c1]), np.ascontiguousarray(V[:, :, c0:c1]))
        ref = orc.SimpleCache(orc.Compressor(t), orc.Compressor(t.v), 1, hkv, dim)
        for h in range(hkv):
            ref.store(0, h, K[0, h], V[0, h], n)
        refs.append(ref)
        kv.append((K, V))
    return refs, kv


def _oracle(orc, t, refs, q, scale, hq=HQ):
    hkv, dim = t.hkv, t.dim
    G = hq // hkv
    out = np.zeros((len(refs), hq, dim), np.float32)
    min_gap = float("inf")
    R = t.R.astype(np.float64)
    for b, ref in enumerate(refs):
        for kvh in range(hkv):
            words, _, _, sigma = ref.read(0, kvh, 0)
            qr = q[b, kvh * G:(kvh + 1) * G].astype(np.float64) @ R.T
            mask, gap = orc.quest_select(words, sigma, t.cents, t.bits, dim, qr)
            min_gap = min(min_gap, gap)
            for g in range(G):
                out[b, kvh * G + g] = ref.attend_mask(0, kvh, q[b, kvh * G + g], scale, mask)
    return out, min_gap


def test_sparse_decode_matches_oracle(lc, orc, gpu):
    lens = [20000, 5000]
    t, cache = _cache(lc, orc, lens)
    refs, _ = _fill(cache, orc, t, lens, 300)
    q = helpers.queries(orc, 301, len(lens), HQ, DIM, std=DIM ** -0.5)
    scale = 1.0 / np.sqrt(DIM)
    got = cache.decode_attn(0, [0, 1], q, HQ, scale, flags=lc.LC_SPARSE_PAGES)
    ref, gap = _oracle(orc, t, refs, q, scale)
    assert gap > 1e-4, gap  # no near-tie at the selection boundary
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    dense = cache.decode_attn(0, [0, 1], q, HQ, scale)
    assert np.abs(dense[0] - got[0]).max() > 1e-4  # the long sequence really went sparse
    ok, msg = helpers.attn_close(got[1:], dense[1:])  # the short one stayed dense
    assert ok, msg
    cache.close()


def test_sparse_decode_peaked(lc, orc, gpu):
    """q ~ N(0, 1) at scale 1: the sparse decode's tiles take the K table's
    f16 residuals like the dense ones, and the selection is unchanged."""
    lens = [20000]
    t, cache = _cache(lc, orc, lens)
    # the keys and query directions of test_sparse_decode_matches_oracle (its
    # selection boundary has no near-tie; scaling q keeps the page order)
    refs, _ = _fill(cache, orc, t, lens, 300)
    q = helpers.queries(orc, 301, 1, HQ, DIM)
    got = cache.decode_attn(0, [0], q, HQ, 1.0, flags=lc.LC_SPARSE_PAGES)
    ref, gap = _oracle(orc, t, refs, q, 1.0)
    assert gap > 1e-4, gap
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    cache.close()


def test_sparse_digest_follows_appends(lc, orc, gpu):
    lens = [17000]
    t, cache = _cache(lc, orc, lens)
    refs, kv = _fill(cache, orc, t, lens, 400)
    scale = 1.0 / np.sqrt(DIM)
    q = helpers.queries(orc, 401, 1, HQ, DIM, std=DIM ** -0.5)
    cache.decode_attn(0, [0], q, HQ, scale, flags=lc.LC_SPARSE_PAGES)  # digests the first pages
    K = helpers.kv(orc, 402, 1, HKV, 300, DIM)
    V = helpers.kv(orc, 403, 1, HKV, 300, DIM)
    for s0 in range(0, 300, 100):  # 300 more tokens: new full pages to digest
        cache.append(0, [0], np.ascontiguousarray(K[:, :, s0:s0 + 100]), np.ascontiguousarray(V[:, :, s0:s0 + 100]))
    for h in range(HKV):
        refs[0].store(0, h, K[0, h], V[0, h], 300)
    got = cache.decode_attn(0, [0], q, HQ, scale, flags=lc.LC_SPARSE_PAGES)
    ref, gap = _oracle(orc, t, refs, q, scale)
    assert gap > 1e-4, gap
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    cache.close()


@pytest.mark.parametrize("std,scale,spread", [(1e-3, 256 ** -0.5, True), (256 ** -0.5, 256 ** -0.5, False),
                                              (1.0, 1.0, False)])
def test_sparse_decode_config2_geometry(lc, orc, gpu, std, scale, spread):
    """3-bit K / 2-bit V at head_dim 256 (config 2's global layer, GQA 2):
    the general digest, the head_dim-256 selection and the tensor-core
    kernel through the tile map, against the oracle's selection + masked
    attention; near-zero queries (nearly uniform weights, so the dropped
    pages show in the output), the configs' query scale and the peaked
    regime (where the chosen high-sigma pages hold the softmax mass)."""
    lens = [20000, 5000]
    t, cache = _cache(lc, orc, lens, dim=256, kb=3, vb=2, hkv=8)
    refs, _ = _fill(cache, orc, t, lens, 500)
    q = helpers.queries(orc, 501, len(lens), 16, 256, std=std)
    got = cache.decode_attn(0, [0, 1], q, 16, scale, flags=lc.LC_SPARSE_PAGES)
    ref, gap = _oracle(orc, t, refs, q, scale, hq=16)
    assert gap > 1e-4, gap
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    if spread:
        dense = cache.decode_attn(0, [0, 1], q, 16, scale)
        assert np.abs(dense[0] - got[0]).max() > 1e-3  # the long sequence really went sparse
    cache.close()


def test_sparse_refusals(lc, orc, gpu):
    q = helpers.queries(orc, 9, 1, HQ, DIM)
    t, cache = _cache(lc, orc, [100], flags=0)
    _fill(cache, orc, t, [100], 1)
    with pytest.raises(lc.LumenError) as e:
        cache.decode_attn(0, [0], q, HQ, 0.1, flags=lc.LC_SPARSE_PAGES)
    assert e.value.code == lc.LC_ERR_STATE
    cache.close()
    t, cache = _cache(lc, orc, [100], max_size=1024)  # a sliding layer
    _fill(cache, orc, t, [100], 2)
    with pytest.raises(lc.LumenError) as e:
        cache.decode_attn(0, [0], q, HQ, 0.1, flags=lc.LC_SPARSE_PAGES)
    assert e.value.code == lc.LC_ERR_INVALID
    cache.close()


@pytest.mark.parametrize("hq,qkind", [(8, "f32"), (16, "f16"), (16, "rotated"), (24, "f32")])
def test_sparse_group_sizes_and_query_forms(lc, orc, gpu, hq, qkind):
    """GQA 1, 2 and 3 (the select kernel's head loop and the fused decode's
    G instantiations), f16 queries, and queries passed already rotated
    (LC_Q_ROTATED), against the same oracle selection."""
    lens = [18000]
    t, cache = _cache(lc, orc, lens)
    refs, _ = _fill(cache, orc, t, lens, 500 + hq)
    q = helpers.queries(orc, 501 + hq, len(lens), hq, DIM, std=DIM ** -0.5)
    scale = 1.0 / np.sqrt(DIM)
    flags = lc.LC_SPARSE_PAGES
    if qkind == "f16":
        q = q.astype(np.float16).astype(np.float32)  # the oracle sees the f16 values
        qg = q.astype(np.float16)
    elif qkind == "rotated":
        qg = (q.astype(np.float64) @ t.R.astype(np.float64).T).astype(np.float32)
        flags |= lc.LC_Q_ROTATED
    else:
        qg = q
    got = cache.decode_attn(0, [0], qg, hq, scale, flags=flags)
    ref, gap = _oracle(orc, t, refs, q, scale, hq)
    assert gap > 1e-4, gap
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    cache.close()


def test_sparse_partials_path(lc, orc, gpu):
    """lc_decode_attn_partials with LC_SPARSE_PAGES (the unfused decode over
    the tile map plus the slot merge) finishes to the fused call's output."""
    lens = [20000, 17000]
    t, cache = _cache(lc, orc, lens)
    _fill(cache, orc, t, lens, 700)
    q = helpers.queries(orc, 701, len(lens), HQ, DIM, std=DIM ** -0.5)
    scale = 1.0 / np.sqrt(DIM)
    fused = cache.decode_attn(0, [0, 1], q, HQ, scale, flags=lc.LC_SPARSE_PAGES)
    m, l, o = cache.decode_partials(0, [0, 1], q, HQ, scale, flags=lc.LC_SPARSE_PAGES)
    out = cache.merge_partials(m[None], l[None], o[None]).reshape(fused.shape)
    np.testing.assert_allclose(out, fused, rtol=0, atol=2e-5)
    cache.close()


def test_sparse_after_lkv2_reload_and_fork(lc, orc, gpu, tmp_path):
    """A sequence loaded from an LKV2 snapshot re-digests its pages, and a
    request forked from a long sequence (pages shared copy-on-write) digests
    the shared pages again: both decode page-sparse exactly like the source."""
    lens = [18000, 0, 0]
    t, cache = _cache(lc, orc, lens)
    refs, _ = _fill(cache, orc, t, lens[:1], 800)
    q = helpers.queries(orc, 801, 1, HQ, DIM, std=DIM ** -0.5)
    scale = 1.0 / np.sqrt(DIM)
    src = cache.decode_attn(0, [0], q, HQ, scale, flags=lc.LC_SPARSE_PAGES)
    p = tmp_path / "sparse.lkv"
    cache.save_lkv2(0, p)
    cache.load_lkv2(1, p)
    loaded = cache.decode_attn(0, [1], q, HQ, scale, flags=lc.LC_SPARSE_PAGES)
    np.testing.assert_array_equal(loaded, src)
    cache.fork(0, 2, lens[0])
    forked = cache.decode_attn(0, [2], q, HQ, scale, flags=lc.LC_SPARSE_PAGES)
    np.testing.assert_array_equal(forked, src)
    again = cache.decode_attn(0, [0], q, HQ, scale, flags=lc.LC_SPARSE_PAGES)
    np.testing.assert_array_equal(again, src)  # the source is untouched by the fork's digests
    cache.close()
