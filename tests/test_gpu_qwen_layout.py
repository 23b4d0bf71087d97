"""GPU: the Qwen TurboQuant layout, V stored un-rotated (LC_STORE_V_UNROTATED).

The reference's Qwen layers rotate K and Q but Lloyd-Max quantize V as it
is, and attend with the dequantized V directly, with no un-rotation on read
(crates/lumen-mlx/src/qwen3_5_moe.rs:2764-2790). The oracle restates that
with a V compressor whose rotation is the identity. Checks: the stored V
codes and sigmas equal the oracle's bit for bit (and K stays rotated), and
decode attention (fused, partials and generic kernels; queries rotated by
the cache or passed rotated, as the Qwen call does) matches the oracle's
attend_keys -> softmax -> attend_values at the decode tolerance.
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _setup(lc, orc, dim, kb, vb, hkv, lens, seed):
    tk = orc.Tables.generate(dim, kb, 64, 42)
    tv = orc.Tables.generate(dim, vb, 64, 42)
    tv_id = orc.Tables(dim, vb, 64, np.eye(dim, dtype=np.float32), tv.bounds, tv.cents, tv.proj)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)  # its R is not used
    pages = (max(lens) + 255) // 256 + 1
    cache = lc.CudaKvCache(1, hkv, dim, ck, cv, max_seqs=len(lens), max_pages=len(lens) * pages + 8,
                           max_pages_per_seq=pages, store_flags=lc.LC_STORE_V_UNROTATED)
    ok, ov = orc.Compressor(tk), orc.Compressor(tv_id)
    refs, vals = [], []
    for b, n in enumerate(lens):
        K = helpers.kv(orc, seed + 2 * b, 1, hkv, n, dim)
        V = helpers.kv(orc, seed + 2 * b + 1, 1, hkv, n, dim)
        cache.append(0, [b], K, V)
        ref = orc.SimpleCache(ok, ov, 1, hkv, dim)
        for h in range(hkv):
            ref.store(0, h, K[0, h], V[0, h], n)
        refs.append(ref)
        vals.append(V)
    return cache, refs, tk


def _oracle(refs, q, hkv, scale):
    B, hq, _ = q.shape
    G = hq // hkv
    return np.stack([np.stack([refs[b].attend(0, h // G, q[b, h], scale) for h in range(hq)]) for b in range(B)])


def test_v_codes_unrotated_bit_exact(lc, orc, gpu):
    cache, refs, _ = _setup(lc, orc, 128, 4, 4, 8, [300], 10)
    f = cache.fetch(0, 0)
    for h in (0, 5):
        kw, _, _, ks = refs[0].read(0, h, 0)
        vw, _, _, vs = refs[0].read(0, h, 1)
        np.testing.assert_array_equal(f["k_words"][h], kw)
        np.testing.assert_array_equal(f["v_words"][h], vw)
        np.testing.assert_array_equal(f["v_sigma"][h].view(np.uint32), vs.view(np.uint32))
    cache.close()


@pytest.mark.parametrize("dim,kb,vb,hkv,hq", [(128, 4, 4, 8, 32), (256, 3, 2, 8, 16), (128, 4, 4, 2, 16)])
def test_decode_unrotated_v(lc, orc, gpu, dim, kb, vb, hkv, hq):
    lens = [2000, 300]
    cache, refs, tk = _setup(lc, orc, dim, kb, vb, hkv, lens, 40 + dim)
    q = helpers.queries(orc, 41, len(lens), hq, dim, std=dim ** -0.5)
    ref = _oracle(refs, q, hkv, 1.0)
    got = cache.decode_attn(0, [0, 1], q, hq, 1.0)
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    # the Qwen call hands over q already rotated (q_rot = R q)
    q_rot = (q.astype(np.float64) @ tk.R.astype(np.float64).T).astype(np.float32)
    got = cache.decode_attn(0, [0, 1], q_rot, hq, 1.0, flags=lc.LC_Q_ROTATED)
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    m, l, o = cache.decode_partials(0, [0, 1], q, hq, 1.0)
    got = cache.merge_partials(m[None], l[None], o[None]).reshape(q.shape)
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    cache.close()
