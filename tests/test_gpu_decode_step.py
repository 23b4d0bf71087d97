"""GPU: lc_decode_step, one layer's decode step (append the new token of
every sequence, then attend; the reference's update_and_fetch followed by
turboquant_fused_attn, mlx/gemma4_moe.rs:4245-4797).

The queries are rotated by the append launch instead of inside the
attention kernel. Checked against the two calls it stands for, on a second
cache with the same contents (codes bit-exact, attention within 2e-5: only
the f32 rounding of the query rotation differs), and against the oracle at
the decode tolerance, in the configs' regime and the peaked one.
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _pair(lc, orc, dim, hkv, lens, seed):
    t = orc.Tables.generate(dim, 4, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(t.R, t.bounds, t.cents, t.proj)
    pages = (max(lens) + 8 + 255) // 256 + 1
    caches = [lc.CudaKvCache(1, hkv, dim, ck, max_seqs=len(lens), max_pages=len(lens) * pages + 8,
                             max_pages_per_seq=pages) for _ in range(2)]
    comp = orc.Compressor(t)
    refs, kvs = [], []
    for b, n in enumerate(lens):
        K = helpers.kv(orc, seed + 2 * b, 1, hkv, n + 1, dim)
        V = helpers.kv(orc, seed + 2 * b + 1, 1, hkv, n + 1, dim)
        for c in caches:
            c.append(0, [b], np.ascontiguousarray(K[:, :, :n]), np.ascontiguousarray(V[:, :, :n]))
        ref = orc.SimpleCache(comp, comp, 1, hkv, dim)
        for h in range(hkv):
            ref.store(0, h, K[0, h], V[0, h], n + 1)
        refs.append(ref)
        kvs.append((K[:, :, n:], V[:, :, n:]))
    k1 = np.ascontiguousarray(np.concatenate([k for k, _ in kvs]))
    v1 = np.ascontiguousarray(np.concatenate([v for _, v in kvs]))
    return caches, refs, k1, v1


@pytest.mark.parametrize("hkv,hq,std,scale", [(8, 32, 128 ** -0.5, 1.0), (8, 32, 1.0, 1.0), (8, 64, 1.0, 128 ** -0.5),
                                              (4, 8, 1.0, 1.0)])
def test_decode_step_equals_append_then_decode(lc, orc, gpu, hkv, hq, std, scale):
    import torch

    lens = [3000, 513, 64]
    (a, b), refs, k1, v1 = _pair(lc, orc, 128, hkv, lens, 70 + hq)
    q = helpers.queries(orc, 71, len(lens), hq, 128, std=std)
    ids = list(range(len(lens)))
    a.append(0, ids, k1, v1)
    want = a.decode_attn(0, ids, q, hq, scale)
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k1, v1))
    out = torch.empty((len(lens), hq, 128), device="cuda")
    b.decode_step(0, ids, kd, vd, qd, hq, scale, out=out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for s in ids:
        fa, fb = a.fetch(s, 0), b.fetch(s, 0)
        np.testing.assert_array_equal(fa["k_words"], fb["k_words"])
        np.testing.assert_array_equal(fa["v_sigma"].view(np.uint32), fb["v_sigma"].view(np.uint32))
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-5 * max(1.0, float(np.abs(want).max())))
    G = hq // hkv
    ref = np.stack([np.stack([refs[s].attend(0, h // G, q[s, h], scale) for h in range(hq)]) for s in ids])
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    a.close()
    b.close()


def test_decode_step_host_inputs_and_flags(lc, orc, gpu):
    """Host numpy inputs, and LC_Q_ROTATED (queries rotated by the caller: no
    rotation in the append launch)."""
    lens = [700]
    (a, b), refs, k1, v1 = _pair(lc, orc, 128, 8, lens, 90)
    q = helpers.queries(orc, 91, 1, 32, 128, std=128 ** -0.5)
    a.append(0, [0], k1, v1)
    want = a.decode_attn(0, [0], q, 32, 1.0)
    got = b.decode_step(0, [0], k1, v1, q, 32, 1.0)
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-5)
    a.close()
    b.close()
