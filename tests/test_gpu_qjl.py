"""GPU: QJL stage-2 scores on the decode side.

- lc_attend_keys_qjl is estimate_inner_products (compressor.rs:122-159):
  stage-1 score plus ||r|| sqrt(pi/2)/sqrt(m) * sum_i sign_i (Phi q)_i, in
  the reference's f32 order, so it must equal the oracle bit for bit.
- lc_decode_attn with LC_QJL_SCORES scores every key with that estimate
  before softmax and attend_values; it is compared with the oracle's
  softmax(scale * two-stage scores) -> attend_values at the decode tolerance.
- Refusals: no stored K QJL bits, a pre-rotated query (the no-alloc entry's
  refusal is in test_zz_no_alloc.py).
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _codecs(lc, orc, dim, kb, vb, m):
    tk = orc.Tables.generate(dim, kb, m, 42)
    tv = orc.Tables.generate(dim, vb, m, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    return tk, tv, ck, cv


def _setup(lc, orc, dim, kb, vb, m, hkv, lens, seed, flags=None):
    tk, tv, ck, cv = _codecs(lc, orc, dim, kb, vb, m)
    B = len(lens)
    pages = (max(max(lens), 1) + 255) // 256 + 1
    cache = lc.CudaKvCache(1, hkv, dim, ck, cv, max_seqs=B, max_pages=B * pages + 8, max_pages_per_seq=pages,
                           store_flags=lc.LC_STORE_K_QJL if flags is None else flags)
    ok, ov = orc.Compressor(tk), orc.Compressor(tv)
    refs = []
    for b, n in enumerate(lens):
        ref = orc.SimpleCache(ok, ov, 1, hkv, dim)
        if n:
            K = helpers.kv(orc, seed + 2 * b, 1, hkv, n, dim)
            V = helpers.kv(orc, seed + 2 * b + 1, 1, hkv, n, dim)
            cache.append(0, [b], K, V)
            for h in range(hkv):
                ref.store(0, h, K[0, h], V[0, h], n)
        refs.append(ref)
    return cache, refs


@pytest.mark.parametrize("kb,m", [(3, 64), (2, 128), (4, 32), (3, 512)])
def test_attend_keys_qjl_bit_exact(lc, orc, gpu, kb, m):
    cache, refs = _setup(lc, orc, 128, kb, kb, m, 2, [300], 40 + kb)
    q = helpers.queries(orc, 41, 1, 1, 128)[0, 0]
    for h in range(2):
        got = cache.attend_keys_qjl(0, 0, h, q)
        ref = refs[0].attend_keys_qjl(0, h, q)
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
        # the correction is really there: stage-1 scores differ
        assert np.any(got != refs[0].attend_keys(0, h, q))
    cache.close()


def _oracle(refs, q, hkv, scale):
    B, hq, dim = q.shape
    G = hq // hkv
    out = np.zeros((B, hq, dim), np.float32)
    for b in range(B):
        if refs[b].seq_len(0, 0) == 0:
            continue
        for h in range(hq):
            out[b, h] = refs[b].attend(0, h // G, q[b, h], scale, qjl=True)
    return out


@pytest.mark.parametrize("dim,kb,vb,m,hkv,hq", [
    (128, 3, 2, 64, 8, 32),   # 3-bit K: where the correction matters
    (128, 4, 4, 64, 8, 32),   # the fast-path geometry, taken by the generic path here
    (256, 2, 2, 256, 4, 8),   # the largest qjl_m the decode takes
    (128, 3, 3, 32, 2, 6),    # m < 64, G = 3
])
def test_decode_qjl_scores(lc, orc, gpu, dim, kb, vb, m, hkv, hq):
    lens = [700, 33, 0, 1]
    cache, refs = _setup(lc, orc, dim, kb, vb, m, hkv, lens, 60 + kb + m)
    q = helpers.queries(orc, 61, len(lens), hq, dim)
    scale = 1.0 / np.sqrt(dim)
    got = cache.decode_attn(0, list(range(len(lens))), q, hq, scale, flags=lc.LC_QJL_SCORES)
    ok, msg = helpers.attn_close(got, _oracle(refs, q, hkv, scale))
    assert ok, msg
    np.testing.assert_array_equal(got[2], 0.0)
    # the stage-1 output differs: the flag changes the scores
    plain = cache.decode_attn(0, list(range(len(lens))), q, hq, scale)
    assert np.abs(plain - got).max() > 1e-4
    cache.close()


def test_decode_qjl_partials_merge(lc, orc, gpu):
    """Partials with QJL scores, merged, equal the one-call QJL decode."""
    import torch

    cache, refs = _setup(lc, orc, 128, 3, 3, 64, 8, [900], 77)
    q = torch.from_numpy(helpers.queries(orc, 78, 1, 32, 128)).cuda()
    scale = 1.0 / np.sqrt(128)
    buf = torch.empty(32 * 130, device="cuda")
    cache.decode_partials(0, [0], q, 32, scale, m=buf[:32], l=buf[32:64], o=buf[64:].view(32, 128),
                          flags=lc.LC_QJL_SCORES)
    merged = torch.empty((32, 128), device="cuda")
    cache.merge_partials(buf[:32].view(1, 32), buf[32:64].view(1, 32), buf[64:].view(1, 32, 128), out=merged)
    ref = torch.empty((1, 32, 128), device="cuda")
    cache.decode_attn(0, [0], q, 32, scale, flags=lc.LC_QJL_SCORES, out=ref)
    torch.cuda.synchronize()
    ok, msg = helpers.attn_close(merged.cpu().numpy().reshape(1, 32, 128), ref.cpu().numpy())
    assert ok, msg
    cache.close()


def test_qjl_refusals(lc, orc, gpu):
    cache, _ = _setup(lc, orc, 128, 3, 3, 64, 8, [40], 90, flags=0)
    q = helpers.queries(orc, 91, 1, 32, 128)
    with pytest.raises(lc.LumenError) as e:
        cache.decode_attn(0, [0], q, 32, 1.0, flags=lc.LC_QJL_SCORES)
    assert e.value.code == lc.LC_ERR_STATE
    with pytest.raises(lc.LumenError) as e:
        cache.attend_keys_qjl(0, 0, 0, q[0, 0])
    assert e.value.code == lc.LC_ERR_STATE
    cache.close()
    cache, _ = _setup(lc, orc, 128, 3, 3, 64, 8, [40], 90)
    with pytest.raises(lc.LumenError) as e:
        cache.decode_attn(0, [0], q, 32, 1.0, flags=lc.LC_QJL_SCORES | lc.LC_Q_ROTATED)
    assert e.value.code == lc.LC_ERR_INVALID
    cache.close()
