"""GPU: the device ring and block table.

1. NativeRotatingKvCacheTurboQuant driven on the device reproduces the twelve
   digests recorded from the reference (golden_tests.rs:465-497): growth,
   one-time trim, wrap, temporal reorder, rewinds and refusals, bit for bit.
2. A sliding-window layer of the cache holds exactly the tokens the ring
   model says it holds, each compressed bit-exactly, and decode over it
   matches the oracle.
3. Prefix reuse through the block table shares pages and copies on write.
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


class GpuCase:
    """golden_tests.rs:372-411 on the device ring."""

    def __init__(self, lc, max_size, keep, qjl):
        self.qjl = qjl
        self.c = lc.NativeRotatingKvCacheTurboQuant(max_size, keep, 4)
        if qjl:
            self.c.with_qjl(64)

    def update(self, s, rng, d, prealloc):
        import ring_model as rm

        arrs = rm.tq_inputs(rng, s, self.qjl)
        if self.qjl:
            (kc, ks, ksg, krn), (vc, vs) = self.c.update_and_fetch_qjl(*arrs, prealloc=prealloc)
            out = [kc, ks, ksg, krn, vc, vs]
        else:
            (kc, ks), (vc, vs) = self.c.update_and_fetch(*arrs, prealloc=prealloc)
            out = [kc, ks, vc, vs]
        for a in out:
            d.array(a)

    def rewind(self, target):
        return self.c.truncate_to(target)

    def buffers(self):
        b = [self.c.backing(i) for i in range(6 if self.qjl else 4)]
        if self.qjl:
            return b[0], b[1], b[4], b[5], b[2], b[3]
        return b[0], b[1], b[2], b[3], None, None

    def counters(self):
        c = self.c.counters()
        return c["offset"], c["idx"], c["buf_len"]


@pytest.mark.parametrize("qjl", [False, True], ids=["stage1", "qjl"])
def test_device_ring_matches_recorded_digests(lc, orc, gpu, qjl):
    import ring_model as rm

    got = rm.digests(lambda ms, kp, q: GpuCase(lc, ms, kp, q), qjl)
    rec = rm.RECORDED_TQ_QJL if qjl else rm.RECORDED_TQ
    assert {k: hex(v) for k, v in got.items()} == {k: hex(v) for k, v in rec.items()}


def test_ring_deep_clone_and_clear(lc, gpu):
    c = lc.RawRing(2, 12, 2, [4, 8])
    for t in range(5):
        c.update([np.full((2, 1, 4), t, np.uint8), np.full((2, 1, 8), t, np.uint8)], True)
    d = c.deep_clone()
    c.update([np.full((2, 1, 4), 9, np.uint8), np.full((2, 1, 8), 9, np.uint8)], True)
    assert d.counters()["offset"] == 5 and c.counters()["offset"] == 6
    assert d.read(0, lc.LC_FETCH_BACKING) != c.read(0, lc.LC_FETCH_BACKING)
    c.clear()
    assert c.counters() == dict(offset=0, idx=0, buf_len=0, view_len=0)
    assert c.read(0, lc.LC_FETCH_BACKING) is None


@pytest.mark.parametrize("prealloc", [True, False])
def test_sliding_layer_holds_the_window(lc, orc, gpu, prealloc):
    """Config 2's sliding layers in miniature: window 64 with 4 sinks, wrapped
    several times by decode steps and chunks."""
    import ring_model as rm

    dim, hkv, hq, window, keep = 256, 2, 4, 64, 4
    tk = orc.Tables.generate(dim, 3, 64, 42)
    tv = orc.Tables.generate(dim, 2, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    cache = lc.CudaKvCache(2, hkv, dim, ck, cv, max_seqs=1, max_pages=16, max_pages_per_seq=4,
                           layer_max_size=[window, 0], layer_keep=[keep, 0], step_prealloc=prealloc)
    model = rm.RingModel(1, window, keep)
    total = 300
    K = helpers.kv(orc, 1234, 1, hkv, total, dim)
    V = helpers.kv(orc, 4321, 1, hkv, total, dim)
    ok, ov = orc.Compressor(tk), orc.Compressor(tv)
    kref = [ok.compress(K[0, h]) for h in range(hkv)]
    vref = [ov.compress(V[0, h]) for h in range(hkv)]
    plan = [1] * 40 + [20] + [1] * 70 + [90] + [1] * 80
    assert sum(plan) == total
    t0 = 0
    for s in plan:
        ids = np.arange(t0, t0 + s, dtype=np.int64).view(np.uint8).reshape(1, 1, s, 8)
        view = model.update([ids], prealloc)[0]
        cache.append(0, [0], np.ascontiguousarray(K[:, :, t0:t0 + s]), np.ascontiguousarray(V[:, :, t0:t0 + s]))
        t0 += s
        toks = view.reshape(-1, 8).copy().view(np.int64).ravel()
        st = cache.ring_state(0, 0)
        assert (st["offset"], st["idx"], st["view_len"]) == (model.offset, model.idx, len(toks))
    got = cache.fetch(0, 0)
    for h in range(hkv):
        np.testing.assert_array_equal(got["k_words"][h], kref[h][0][toks])
        np.testing.assert_array_equal(got["v_words"][h], vref[h][0][toks])
        np.testing.assert_array_equal(got["k_sigma"][h], kref[h][3][toks])
    # decode over the window == oracle attention over exactly those tokens
    ref = orc.SimpleCache(ok, ov, 1, hkv, dim)
    for h in range(hkv):
        ref.store(0, h, K[0, h, toks], V[0, h, toks], len(toks))
    q = helpers.queries(orc, 77, 1, hq, dim)
    scale = 1.0 / np.sqrt(dim)
    out = cache.decode_attn(0, [0], q, hq, scale)
    exp = np.stack([ref.attend(0, h // 2, q[0, h], scale) for h in range(hq)])
    ok, msg = helpers.attn_close(out[0], exp)
    assert ok, msg
    # post-rotation rollback refused (native_cache.rs:318-327)
    with pytest.raises(lc.LumenError) as e:
        cache.truncate_to(0, 0, 10)
    assert e.value.code == lc.LC_ERR_REFUSED


def test_prefix_fork_copy_on_write(lc, orc, gpu):
    dim, hkv, hq = 128, 8, 32
    tk = orc.Tables.generate(dim, 4, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cache = lc.CudaKvCache(2, hkv, dim, ck, max_seqs=3, max_pages=40, max_pages_per_seq=8)
    K = helpers.kv(orc, 50, 1, hkv, 1100, dim)
    V = helpers.kv(orc, 51, 1, hkv, 1100, dim)
    for layer in range(2):
        cache.append(layer, [0], np.ascontiguousarray(K[:, :, :1000]), np.ascontiguousarray(V[:, :, :1000]))
    before = cache.fetch(0, 1)
    cache.fork(0, 1, 600)                      # shares pages 0..2, page 2 partially
    assert cache.ring_state(1, 1)["view_len"] == 600
    # diverge: seq 1 appends its own tokens, seq 0 keeps decoding
    for layer in range(2):
        cache.append(layer, [1], np.ascontiguousarray(K[:, :, 1000:1050]), np.ascontiguousarray(V[:, :, 1000:1050]))
        for t in range(1000, 1010):
            cache.append(layer, [0], np.ascontiguousarray(K[:, :, t:t + 1]), np.ascontiguousarray(V[:, :, t:t + 1]))
    a = cache.fetch(0, 1)
    b = cache.fetch(1, 1)
    np.testing.assert_array_equal(a["k_words"][:, :1000], before["k_words"])
    np.testing.assert_array_equal(b["k_words"][:, :600], before["k_words"][:, :600])
    # seq 1 == a sequence built from the same 650 tokens without sharing
    idx = np.r_[0:600, 1000:1050]
    cache.append(1, [2], np.ascontiguousarray(K[:, :, idx]), np.ascontiguousarray(V[:, :, idx]))
    c = cache.fetch(2, 1)
    np.testing.assert_array_equal(b["k_words"], c["k_words"])
    np.testing.assert_array_equal(b["v_sigma"], c["v_sigma"])
    q = helpers.queries(orc, 3, 2, hq, dim)
    qq = np.ascontiguousarray(np.stack([q[0], q[0]]))
    o1 = cache.decode_attn(1, [1, 2], qq, hq, 1.0 / np.sqrt(dim))
    np.testing.assert_array_equal(o1[0], o1[1])  # shared pages read exactly like private ones
    # fork past what the source holds is refused
    with pytest.raises(lc.LumenError):
        cache.fork(0, 2, 5000)
    cache.release(1)
    assert cache.ring_state(1, 0)["view_len"] == 0


def test_truncate_to_refusals(lc, orc, gpu):
    tk = orc.Tables.generate(128, 4, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cache = lc.CudaKvCache(1, 2, 128, ck, max_seqs=1, max_pages=8, max_pages_per_seq=4)
    x = helpers.kv(orc, 1, 1, 2, 10, 128)
    cache.append(0, [0], x, x)
    with pytest.raises(lc.LumenError) as e:
        cache.truncate_to(0, 0, 11)
    assert e.value.code == lc.LC_ERR_REFUSED
    cache.truncate_to(0, 0, 10)
    cache.truncate_to(0, 0, 4)
    st = cache.ring_state(0, 0)
    assert st["offset"] == 4 and st["idx"] == 4 and st["view_len"] == 4
