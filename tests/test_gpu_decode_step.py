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


def _pair(lc, orc, dim, hkv, lens, seed, kbits=4, vbits=4):
    tk = orc.Tables.generate(dim, kbits, 64, 42)
    tv = orc.Tables.generate(dim, vbits, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    pages = (max(lens) + 8 + 255) // 256 + 1
    caches = [lc.CudaKvCache(1, hkv, dim, ck, cv, max_seqs=len(lens), max_pages=len(lens) * pages + 8,
                             max_pages_per_seq=pages) for _ in range(2)]
    comp, vcomp = orc.Compressor(tk), orc.Compressor(tv)
    refs, kvs = [], []
    for b, n in enumerate(lens):
        K = helpers.kv(orc, seed + 2 * b, 1, hkv, n + 1, dim)
        V = helpers.kv(orc, seed + 2 * b + 1, 1, hkv, n + 1, dim)
        for c in caches:
            c.append(0, [b], np.ascontiguousarray(K[:, :, :n]), np.ascontiguousarray(V[:, :, :n]))
        ref = orc.SimpleCache(comp, vcomp, 1, hkv, dim)
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


@pytest.mark.parametrize("hq,std", [(16, 256 ** -0.5), (16, 1.0), (8, 1.0), (32, 256 ** -0.5)])
def test_decode_step_config2_geometry(lc, orc, gpu, hq, std):
    """Config 2's geometry (head_dim 256, 3-bit K / 2-bit V, 8 KV heads, bf16
    queries): the append launch rotates the queries with R^T streamed through
    shared memory and the tensor-core kernel reads them as given (no rotation
    launch)."""
    import torch

    hkv, dim, scale = 8, 256, 256 ** -0.5
    lens = [2100, 300, 40]
    (a, b), refs, k1, v1 = _pair(lc, orc, dim, hkv, lens, 170 + hq, kbits=3, vbits=2)
    q = helpers.queries(orc, 171, len(lens), hq, dim, std=std)
    ids = list(range(len(lens)))
    qd = torch.from_numpy(q).cuda().to(torch.bfloat16)
    kd, vd = torch.from_numpy(k1).cuda(), torch.from_numpy(v1).cuda()
    a.append(0, ids, kd, vd)
    want = torch.empty((len(lens), hq, dim), device="cuda")
    a.decode_attn(0, ids, qd, hq, scale, out=want)
    got = torch.empty((len(lens), hq, dim), device="cuda")
    b.decode_step(0, ids, kd, vd, qd, hq, scale, out=got)
    torch.cuda.synchronize()
    want, got = want.cpu().numpy(), got.cpu().numpy()
    for s in ids:
        fa, fb = a.fetch(s, 0), b.fetch(s, 0)
        np.testing.assert_array_equal(fa["k_words"], fb["k_words"])
        np.testing.assert_array_equal(fa["v_words"], fb["v_words"])
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-5 * max(1.0, float(np.abs(want).max())))
    G = hq // hkv
    qb = qd.float().cpu().numpy()
    ref = np.stack([np.stack([refs[s].attend(0, h // G, qb[s, h], scale) for h in range(hq)]) for s in ids])
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg
    a.close()
    b.close()


def test_decode_step_layers_equals_per_layer_calls(lc, orc, gpu):
    """lc_decode_step_layers over 3 stacked layers gives the results of 3
    lc_decode_step calls (bit for bit: the same launches in the same order)."""
    import torch

    L, hkv, hq, dim, lens = 3, 8, 32, 128, [900, 300]
    t = orc.Tables.generate(dim, 4, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(t.R, t.bounds, t.cents, t.proj)
    pages = (max(lens) + 2 * 256 + 255) // 256 + 1  # room for the ring's 256-token growth steps
    caches = [lc.CudaKvCache(L, hkv, dim, ck, max_seqs=len(lens), max_pages=L * len(lens) * pages + 8,
                             max_pages_per_seq=pages) for _ in range(2)]
    ids = np.arange(len(lens), dtype=np.int32)
    for layer in range(L):
        for b, n in enumerate(lens):
            K = helpers.kv(orc, 300 + 10 * layer + 2 * b, 1, hkv, n, dim)
            V = helpers.kv(orc, 301 + 10 * layer + 2 * b, 1, hkv, n, dim)
            for c in caches:
                c.append(layer, [b], K, V)
    k1 = torch.from_numpy(np.stack([helpers.kv(orc, 400 + l, len(lens), hkv, 1, dim) for l in range(L)])).cuda()
    v1 = torch.from_numpy(np.stack([helpers.kv(orc, 500 + l, len(lens), hkv, 1, dim) for l in range(L)])).cuda()
    q = torch.from_numpy(np.stack([helpers.queries(orc, 600 + l, len(lens), hq, dim, std=dim ** -0.5)
                                   for l in range(L)])).cuda().to(torch.bfloat16)
    want = torch.empty((L, len(lens), hq, dim), device="cuda", dtype=torch.bfloat16)
    got = torch.empty_like(want)
    for layer in range(L):
        caches[0].decode_step(layer, ids, k1[layer], v1[layer], q[layer], hq, 1.0, out=want[layer],
                              out_dtype=lc.LC_BF16)
    caches[1].decode_step_layers(0, ids, k1, v1, q, hq, 1.0, out=got, out_dtype=lc.LC_BF16)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    for layer in range(L):
        for b in range(len(lens)):
            fa, fb = caches[0].fetch(b, layer), caches[1].fetch(b, layer)
            np.testing.assert_array_equal(fa["k_words"], fb["k_words"])
            np.testing.assert_array_equal(fa["v_sigma"].view(np.uint32), fb["v_sigma"].view(np.uint32))
    # host inputs and a sub-range of layers
    kh, vh = k1.cpu().numpy(), v1.cpu().numpy()
    qh = q.float().cpu().numpy()
    out_a = caches[0].decode_step(1, ids, kh[1], vh[1], qh[1], hq, 1.0)
    out_b = caches[1].decode_step_layers(1, ids, kh[1:2], vh[1:2], qh[1:2], hq, 1.0)
    np.testing.assert_array_equal(out_b[0], out_a)
    for c in caches:
        c.close()
