"""GPU: the path at BASELINE's full sizes, checked through size-independent
properties plus oracle slices.

Config 1 (32 sequences x 8192 tokens, 32 q / 8 kv heads, d 128, 4-bit K/V,
bf16 K/V with outlier channels, queries N(0, 1/sqrt(128)), scale 1):
- the one-launch fused decode equals the partials path (split-K partials,
  then the slot merge and un-rotation of lc_merge_partials);
- a sequence decoded alone equals its row of the batched decode;
- 8 full (sequence, kv head) slices spread over the batch and the heads:
  codes and sigmas bit-exact against the oracle's compressor, attention
  within the decode tolerance of the oracle's attend_keys -> softmax ->
  attend_values.

Config 2 (d 256, 3-bit K / 2-bit V, 16 q / 8 kv heads, a 1024-token sliding
ring wrapped 4x): decode over the wrapped ring equals decode over a fresh
full layer holding exactly the ring's 1024 tokens (attention does not
depend on key order, and quantization is per vector).
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _codecs(lc, orc, dim, kb, vb):
    tk = orc.Tables.generate(dim, kb, 64, 42)
    tv = orc.Tables.generate(dim, vb, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    return tk, tv, ck, cv


def _kv_dev(torch, gen, B, H, n, dim):
    """bf16 N(0, 1) with 4 channels per head scaled x8 (the configs' key outliers)."""
    x = torch.randn((B, H, n, dim), generator=gen, device="cuda", dtype=torch.float32)
    ch = torch.randint(0, dim, (H, 4), generator=gen, device="cuda")
    for h in range(H):
        x[:, h, :, ch[h]] *= 8.0
    return x.to(torch.bfloat16)


def test_config1_full_size(lc, orc, gpu):
    import torch

    B, HKV, HQ, D, N = 32, 8, 32, 128, 8192
    tk, tv, ck, cv = _codecs(lc, orc, D, 4, 4)
    pages = N // 256 + 2
    cache = lc.CudaKvCache(1, HKV, D, ck, cv, max_seqs=B, max_pages=B * pages + 8, max_pages_per_seq=pages)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1234)
    K = _kv_dev(torch, gen, B, HKV, N, D)
    V = _kv_dev(torch, gen, B, HKV, N, D)
    ids = list(range(B))
    for c0 in range(0, N, 2048):
        cache.append(0, ids, K[:, :, c0:c0 + 2048].contiguous(), V[:, :, c0:c0 + 2048].contiguous())
    q = (torch.randn((B, HQ, D), generator=gen, device="cuda") * D ** -0.5).to(torch.bfloat16)
    out = torch.empty((B, HQ, D), device="cuda", dtype=torch.float32)
    cache.decode_attn(0, ids, q, HQ, 1.0, out=out, out_dtype=lc.LC_F32)
    torch.cuda.synchronize()
    fused = out.cpu().numpy()
    assert np.isfinite(fused).all()

    # the partials path: split-K slots merged per row, then un-rotated
    m, l, o = cache.decode_partials(0, ids, q.float().cpu().numpy(), HQ, 1.0)
    merged = cache.merge_partials(m[None], l[None], o[None]).reshape(B, HQ, D)
    np.testing.assert_allclose(merged, fused, rtol=0, atol=2e-5)

    # one sequence alone against its row of the batch
    b = 5
    one = cache.decode_attn(0, [b], q[b:b + 1].float().cpu().numpy(), HQ, 1.0)
    np.testing.assert_allclose(one[0], fused[b], rtol=0, atol=2e-5)

    # the oracle on 8 full (sequence, kv head) slices spread over the batch
    # and the heads: codes and sigmas, then attention
    G = HQ // HKV
    ok_c, ok_v = orc.Compressor(tk), orc.Compressor(tv)
    for b, h in [(0, 0), (5, 3), (9, 7), (14, 1), (18, 4), (23, 6), (27, 2), (31, 5)]:
        Kh = K[b, h].float().cpu().numpy()
        Vh = V[b, h].float().cpu().numpy()
        ref = orc.SimpleCache(ok_c, ok_v, 1, 1, D)
        ref.store(0, 0, Kh, Vh, N)
        f = cache.fetch(b, 0)
        words, _, _, sigma = ref.read(0, 0, 0)
        np.testing.assert_array_equal(f["k_words"][h], words)
        np.testing.assert_array_equal(f["k_sigma"][h].view(np.uint32),
                                      np.asarray(sigma, np.float32).view(np.uint32))
        vwords, _, _, vsigma = ref.read(0, 0, 1)
        np.testing.assert_array_equal(f["v_words"][h], vwords)
        np.testing.assert_array_equal(f["v_sigma"][h].view(np.uint32),
                                      np.asarray(vsigma, np.float32).view(np.uint32))
        qb = q[b].float().cpu().numpy()
        want = np.stack([ref.attend(0, 0, qb[h * G + g], 1.0) for g in range(G)])
        ok, msg = helpers.attn_close(fused[b, h * G:(h + 1) * G], want)
        assert ok, f"slice ({b}, {h}): {msg}"
    cache.close()


def test_config2_wrapped_ring_equals_its_window(lc, orc, gpu):
    import torch

    B, HKV, HQ, D, W = 4, 8, 16, 256, 1024
    tk, tv, ck, cv = _codecs(lc, orc, D, 3, 2)
    pages = (W + 512) // 256 + 4
    ring = lc.CudaKvCache(1, HKV, D, ck, cv, max_seqs=B, max_pages=B * pages + 8, max_pages_per_seq=pages,
                          layer_max_size=[W], layer_keep=[0])
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77)
    n_chunked, n_single = 4 * W, W + 50  # wrapped 4x by 512-token chunks, then the in-place regime
    K = _kv_dev(torch, gen, B, HKV, n_chunked + n_single, D)
    V = _kv_dev(torch, gen, B, HKV, n_chunked + n_single, D)
    ids = list(range(B))
    for c0 in range(0, n_chunked, 512):
        ring.append(0, ids, K[:, :, c0:c0 + 512].contiguous(), V[:, :, c0:c0 + 512].contiguous())
    for t in range(n_chunked, n_chunked + n_single):
        ring.append(0, ids, K[:, :, t:t + 1].contiguous(), V[:, :, t:t + 1].contiguous())
    assert ring.seq_len(0, 0, 0) == W
    total = n_chunked + n_single
    fresh_pages = W // 256 + 2
    fresh = lc.CudaKvCache(1, HKV, D, ck, cv, max_seqs=B, max_pages=B * fresh_pages + 8,
                           max_pages_per_seq=fresh_pages)
    fresh.append(0, ids, K[:, :, total - W:].contiguous(), V[:, :, total - W:].contiguous())
    q = (torch.randn((B, HQ, D), generator=gen, device="cuda") * D ** -0.5).float().cpu().numpy()
    scale = D ** -0.5
    a = ring.decode_attn(0, ids, q, HQ, scale)
    b = fresh.decode_attn(0, ids, q, HQ, scale)
    assert np.isfinite(a).all()
    np.testing.assert_allclose(a, b, rtol=0, atol=2e-5)
    ring.close()
    fresh.close()
