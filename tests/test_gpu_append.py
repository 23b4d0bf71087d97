"""GPU: quantize-append and the trait hooks, bit-exact against the oracle.

The CUDA append kernel must reproduce compress_one (compressor.rs:61-107)
bit for bit: packed code words, sigma, QJL words and residual norm.
attend_keys / attend_values must reproduce SimpleCache (simple.rs:137-155)
bit for bit. Everything goes through the C ABI.
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu

CASES = [  # (head_dim, k_bits, v_bits, qjl_m)
    (128, 4, 4, 64),
    (128, 3, 3, 64),
    (64, 3, 2, 32),
    (256, 3, 2, 128),
    (128, 8, 2, 65),
]


def _codecs(lc, orc, dim, kb, vb, m, seed=42):
    tk = orc.Tables.generate(dim, kb, m, seed)
    tv = orc.Tables.generate(dim, vb, m, seed)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    return tk, tv, ck, cv


@pytest.mark.parametrize("dim,kb,vb,m", CASES)
def test_store_bit_exact(lc, orc, gpu, dim, kb, vb, m):
    tk, tv, ck, cv = _codecs(lc, orc, dim, kb, vb, m)
    H, n = 3, 300
    X = helpers.kv(orc, 1000 + dim + kb, 2, H, n, dim)
    X[0, 1, 5] = 0.0  # degenerate zero vector (compressor.rs:73-75)
    X[1, 2, 7] *= np.float32(1e4)
    cache = lc.SimpleCache(ck, 1, H, dim, v_compressor=cv, max_tokens=1024)
    ref = orc.SimpleCache(orc.Compressor(tk), orc.Compressor(tv), 1, H, dim)
    for h in range(H):
        # ragged: heads store different chunkings
        cuts = [0, 1, 17, 150, n] if h % 2 == 0 else [0, n]
        for a, b in zip(cuts[:-1], cuts[1:]):
            cache.store(0, h, X[0, h, a:b], X[1, h, a:b], b - a)
            ref.store(0, h, X[0, h, a:b], X[1, h, a:b], b - a)
    got = cache.fetch(0)
    for h in range(H):
        assert cache.seq_len(0, h) == ref.seq_len(0, h) == n
        for side, (w, s, q, r) in enumerate([("k_words", "k_sigma", "k_qjl", "k_rnorm"),
                                              ("v_words", "v_sigma", "v_qjl", "v_rnorm")]):
            s1, s2, rn, sc = ref.read(0, h, side)
            np.testing.assert_array_equal(got[w][h], s1)
            np.testing.assert_array_equal(got[s][h].view(np.uint32), sc.view(np.uint32))
            np.testing.assert_array_equal(got[q][h], s2)
            np.testing.assert_array_equal(got[r][h].view(np.uint32), rn.view(np.uint32))


@pytest.mark.parametrize("dim,kb,vb,m", CASES[:4])
def test_attend_hooks_bit_exact(lc, orc, gpu, dim, kb, vb, m):
    tk, tv, ck, cv = _codecs(lc, orc, dim, kb, vb, m)
    H, n = 2, 200
    X = helpers.kv(orc, 77 + dim, 2, H, n, dim)
    cache = lc.SimpleCache(ck, 2, H, dim, v_compressor=cv, max_tokens=512)
    ref = orc.SimpleCache(orc.Compressor(tk), orc.Compressor(tv), 2, H, dim)
    for h in range(H):
        cache.store(1, h, X[0, h], X[1, h], n)
        ref.store(1, h, X[0, h], X[1, h], n)
    q = orc.gauss_f32(5, dim)
    for h in range(H):
        a = cache.attend_keys(1, h, q)
        b = ref.attend_keys(1, h, q)
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
        w = np.exp((b - b.max()).astype(np.float64))
        w = (w / w.sum()).astype(np.float32)
        w[3] = 0.0  # below the 1e-10 skip threshold (simple.rs:149)
        va = cache.attend_values(1, h, w)
        vb_ = ref.attend_values(1, h, w)
        np.testing.assert_array_equal(va.view(np.uint32), vb_.view(np.uint32))
    # empty head
    assert len(cache.attend_keys(0, 0, q)) == 0
    np.testing.assert_array_equal(cache.attend_values(0, 0, np.zeros(0, np.float32)), np.zeros(dim, np.float32))


def test_truncate_and_clear_trait(lc, orc, gpu):
    tk, tv, ck, cv = _codecs(lc, orc, 128, 3, 3, 64)
    cache = lc.SimpleCache(ck, 1, 2, 128, max_tokens=64)
    X = helpers.kv(orc, 7, 2, 2, 6, 128)
    for t in range(6):
        for h in range(2):
            cache.store(0, h, X[0, h, t], X[1, h, t], 1)
    assert cache.seq_len(0, 0) == 6 and cache.seq_len(0, 1) == 6
    cache.truncate(0, 4)
    assert cache.seq_len(0, 0) == 4 and cache.seq_len(0, 1) == 4
    cache.truncate(0, 10)
    assert cache.seq_len(0, 0) == 4
    cache.truncate(0, 0)
    assert cache.seq_len(0, 0) == 0 and cache.seq_len(0, 1) == 0
    cache.store(0, 0, X[0, 0, 0], X[1, 0, 0], 1)
    assert cache.seq_len(0, 0) == 1
    cache.clear()
    assert cache.seq_len(0, 0) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_append_batched_bit_exact(lc, orc, gpu, dtype):
    """lc_append over several sequences at once: the kernel sees bf16 (or f32)
    inputs; the oracle compresses the same values widened to f32."""
    import torch

    dim, H, S, n = 128, 8, 3, 40
    tk, tv, ck, cv = _codecs(lc, orc, dim, 4, 4, 64)
    cache = lc.CudaKvCache(2, H, dim, ck, cv, max_seqs=4, max_pages=64, max_pages_per_seq=8,
                           store_flags=lc.LC_STORE_K_QJL)
    K = helpers.kv(orc, 11, S, H, n, dim)
    V = helpers.kv(orc, 12, S, H, n, dim)
    if dtype == "bf16":
        Kt, K = helpers.to_bf16(K)
        Vt, V = helpers.to_bf16(V)
        Kt, Vt = Kt.cuda(), Vt.cuda()
    else:
        Kt, Vt = torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda()
    ids = [2, 0, 3]
    # prefill in two chunks then 3 decode steps (S=1)
    cache.append(1, ids, Kt[:, :, :30].contiguous(), Vt[:, :, :30].contiguous())
    for t in range(30, n):
        cache.append(1, ids, Kt[:, :, t:t + 1].contiguous(), Vt[:, :, t:t + 1].contiguous())
    ok, ov = orc.Compressor(tk), orc.Compressor(tv)
    for b, seq in enumerate(ids):
        got = cache.fetch(seq, 1)
        assert cache.ring_state(seq, 1)["view_len"] == n
        for h in range(H):
            s1, s2, rn, sc = ok.compress(K[b, h])
            np.testing.assert_array_equal(got["k_words"][h], s1)
            np.testing.assert_array_equal(got["k_sigma"][h].view(np.uint32), sc.view(np.uint32))
            np.testing.assert_array_equal(got["k_qjl"][h], s2)
            np.testing.assert_array_equal(got["k_rnorm"][h].view(np.uint32), rn.view(np.uint32))
            s1, _, _, sc = ov.compress(V[b, h])
            np.testing.assert_array_equal(got["v_words"][h], s1)
            np.testing.assert_array_equal(got["v_sigma"][h].view(np.uint32), sc.view(np.uint32))
    assert cache.ring_state(1, 1)["view_len"] == 0


@pytest.mark.parametrize("dim,kb,vb,qjl,dtype,offset", [
    (128, 4, 4, False, "bf16", 0),  # config 3's chunk append: the register-blocked tile kernel
    (128, 4, 4, False, "f32", 0),
    (64, 2, 3, False, "bf16", 0),   # d 64, 2-bit K / 3-bit V (3-bit words hold 21 codes)
    (128, 4, 4, True, "bf16", 0),   # QJL stage 2: the batched strict kernel
    (128, 4, 4, False, "bf16", 1),  # inputs off the 8-byte boundary: the strict kernel takes them
])
def test_append_large_bit_exact(lc, orc, gpu, dim, kb, vb, qjl, dtype, offset):
    """One append of more than 16384 vectors per side (3 x 8 x 801 = 19224,
    not a multiple of any batch): codes, sigmas (and QJL bits, residual
    norms) bit-identical to the oracle's compress of the same values."""
    import torch

    H, S, n = 8, 3, 801
    tk, tv, ck, cv = _codecs(lc, orc, dim, kb, vb, 64)
    pages = (n + 255) // 256 + 2
    cache = lc.CudaKvCache(1, H, dim, ck, cv, max_seqs=S, max_pages=S * pages + 8, max_pages_per_seq=pages,
                           store_flags=(lc.LC_STORE_K_QJL | lc.LC_STORE_V_QJL) if qjl else 0)
    K = helpers.kv(orc, 21, S, H, n, dim)
    V = helpers.kv(orc, 22, S, H, n, dim)
    if dtype == "bf16":
        Kt, K = helpers.to_bf16(K)
        Vt, V = helpers.to_bf16(V)
        Kt, Vt = Kt.cuda(), Vt.cuda()
    else:
        Kt, Vt = torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda()
    if offset:  # the same values starting `offset` elements into a larger buffer
        def shift(t):
            buf = torch.zeros(t.numel() + offset, dtype=t.dtype, device=t.device)
            buf[offset:] = t.reshape(-1)
            return buf[offset:].view(t.shape)
        Kt, Vt = shift(Kt), shift(Vt)
    cache.append(0, [0, 1, 2], Kt, Vt)
    ok, ov = orc.Compressor(tk), orc.Compressor(tv)
    for b in range(S):
        got = cache.fetch(b, 0)
        for h in range(H):
            for p, x, comp in (("k", K[b, h], ok), ("v", V[b, h], ov)):
                s1, s2, rn, sc = comp.compress(x)
                np.testing.assert_array_equal(got[f"{p}_words"][h], s1, err_msg=f"{b} {h} {p}")
                np.testing.assert_array_equal(got[f"{p}_sigma"][h].view(np.uint32), sc.view(np.uint32))
                if qjl:
                    np.testing.assert_array_equal(got[f"{p}_qjl"][h], s2)
                    np.testing.assert_array_equal(got[f"{p}_rnorm"][h].view(np.uint32), rn.view(np.uint32))
    cache.close()


def test_append_errors(lc, orc, gpu):
    tk, tv, ck, cv = _codecs(lc, orc, 128, 4, 4, 64)
    cache = lc.CudaKvCache(1, 2, 128, ck, max_seqs=2, max_pages=4, max_pages_per_seq=2)
    x = np.zeros((1, 2, 1, 128), np.float32)
    with pytest.raises(lc.LumenError):
        cache.append(0, [5], x, x)  # bad sequence id
    with pytest.raises(lc.LumenError):
        cache.append(3, [0], x, x)  # bad layer
    big = np.zeros((1, 2, 1200, 128), np.float32)
    with pytest.raises(lc.LumenError) as e:
        cache.append(0, [0], big, big)  # more pages than the pool holds
    assert e.value.code == lc.LC_ERR_NOMEM
    assert cache.ring_state(0, 0) == dict(offset=0, idx=0, buf_len=0, view_len=0)  # refused before any change
    cache.append(0, [0], x, x)
    assert cache.ring_state(0, 0)["view_len"] == 1
