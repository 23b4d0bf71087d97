"""GPU: fused split-K decode attention against the oracle.

The oracle composes the reference's trait calls exactly as a caller does:
attend_keys (compressor.rs:165-184) -> softmax(scale * s) -> attend_values
(simple.rs:76-99, 142-155). The GPU path computes the same function in the
rotated basis with f16 tensor-core tiles and f32 accumulation, so parity is
a tolerance (helpers.attn_close): for every output row (one query head)
    max |out - ref| <= 2e-3 + 1e-3 * max |ref row|   (2e-3 absolute, 1e-3 relative)
and over the whole output relative MSE (turboquant.rs:993-1003) <= 1e-3.
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu

ATOL = 2e-3
RTOL = 1e-3
REL_MSE = 1e-3


def _setup(lc, orc, dim, kb, vb, hkv, lens, seed, layers=1, m=64):
    tk = orc.Tables.generate(dim, kb, m, 42)
    tv = orc.Tables.generate(dim, vb, m, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    B = len(lens)
    nmax = max(max(lens), 1)
    pages = (nmax + 255) // 256 + 1
    cache = lc.CudaKvCache(layers, hkv, dim, ck, cv, max_seqs=B, max_pages=B * pages * layers + 8,
                           max_pages_per_seq=pages)
    ok, ov = orc.Compressor(tk), orc.Compressor(tv)
    refs = []
    for b, n in enumerate(lens):
        ref = orc.SimpleCache(ok, ov, 1, hkv, dim)
        if n:
            K = helpers.kv(orc, seed + 2 * b, 1, hkv, n, dim)
            V = helpers.kv(orc, seed + 2 * b + 1, 1, hkv, n, dim)
            cache.append(layers - 1, [b], K, V)
            for h in range(hkv):
                ref.store(0, h, K[0, h], V[0, h], n)
        refs.append(ref)
    return cache, refs, tk, tv


def _oracle(refs, q, hkv, scale):
    B, hq, dim = q.shape
    G = hq // hkv
    out = np.zeros((B, hq, dim), np.float32)
    for b in range(B):
        if refs[b].seq_len(0, 0) == 0:
            continue
        for h in range(hq):
            out[b, h] = refs[b].attend(0, h // G, q[b, h], scale)
    return out


def _assert_close(got, ref):
    ok, msg = helpers.attn_close(got, ref)
    assert ok, msg


def test_decode_config0(lc, orc, gpu):
    """1 layer, batch 1, 8 kv heads, d 128, 4096 tokens, 4-bit K/V, 32 q heads."""
    cache, refs, tk, tv = _setup(lc, orc, 128, 4, 4, 8, [4096], 100)
    q = helpers.queries(orc, 9, 1, 32, 128)
    scale = 1.0 / np.sqrt(128)
    got = cache.decode_attn(0, [0], q, 32, scale)
    _assert_close(got, _oracle(refs, q, 8, scale))


def test_decode_config1_shape_small_batch(lc, orc, gpu):
    """Config 1 geometry (GQA 32/8, d 128, 4-bit, q ~ N(0, 1/sqrt(128)), scale 1), ragged lengths."""
    lens = [1, 15, 16, 17, 255, 256, 257, 1000, 0, 2049]
    cache, refs, tk, tv = _setup(lc, orc, 128, 4, 4, 8, lens, 300)
    q = helpers.queries(orc, 10, len(lens), 32, 128, std=128 ** -0.5)
    got = cache.decode_attn(0, list(range(len(lens))), q, 32, 1.0)
    ref = _oracle(refs, q, 8, 1.0)
    _assert_close(got, ref)
    np.testing.assert_array_equal(got[8], 0.0)  # empty sequence


@pytest.mark.parametrize("dim,kb,vb,hkv,hq", [
    (256, 3, 2, 8, 16),   # config 2: 3-bit K / 2-bit V, d 256, 16 q / 8 kv
    (128, 4, 4, 8, 8),    # no GQA, fast path G=1
    (128, 4, 4, 2, 16),   # G=8
    (128, 3, 3, 4, 12),   # generic path, G=3
    (64, 2, 4, 2, 4),
])
def test_decode_other_geometries(lc, orc, gpu, dim, kb, vb, hkv, hq):
    lens = [700, 33]
    cache, refs, tk, tv = _setup(lc, orc, dim, kb, vb, hkv, lens, 500 + dim + kb)
    q = helpers.queries(orc, 11, len(lens), hq, dim)
    scale = 1.0 / np.sqrt(dim)
    got = cache.decode_attn(0, [0, 1], q, hq, scale)
    _assert_close(got, _oracle(refs, q, hkv, scale))


@pytest.mark.parametrize("hq", [32, 16, 8])
def test_decode_many_short_sequences(lc, orc, gpu, hq):
    """40 sequences of 33..64 tokens (two 32-token tiles per kv head): every
    CTA of the one-launch kernel covers 8 (sequence, kv head) segments, so
    its query rotation and output un-rotation handle 8 * G rows (32 at G=4:
    four 8-row blocks)."""
    rng = np.random.default_rng(5)
    lens = [int(x) for x in rng.integers(33, 65, size=40)]
    cache, refs, tk, tv = _setup(lc, orc, 128, 4, 4, 8, lens, 900)
    q = helpers.queries(orc, 13, len(lens), hq, 128)
    scale = 1.0 / np.sqrt(128)
    got = cache.decode_attn(0, list(range(len(lens))), q, hq, scale)
    _assert_close(got, _oracle(refs, q, 8, scale))


def test_decode_dtypes_and_flags(lc, orc, gpu):
    import torch

    cache, refs, tk, tv = _setup(lc, orc, 128, 4, 4, 8, [600, 300], 700)
    q = helpers.queries(orc, 12, 2, 32, 128)
    scale = 1.0 / np.sqrt(128)
    ref = _oracle(refs, q, 8, scale)
    # bf16 query on the device, bf16 output on the device
    qt, qv = helpers.to_bf16(q)
    out = torch.empty((2, 32, 128), dtype=torch.bfloat16, device="cuda")
    cache.decode_attn(0, [0, 1], qt.cuda(), 32, scale, out=out, out_dtype=lc.LC_BF16)
    ref_b = _oracle(refs, qv, 8, scale)
    got = out.float().cpu().numpy()
    # bf16 output: one rounding of 2^-9 relative on top of the f32 tolerance
    assert (np.abs(got - ref_b) - (ATOL + RTOL * np.abs(ref_b).max(-1, keepdims=True)
                                   + 2.0 ** -8 * np.abs(ref_b))).max() <= 0
    assert helpers.rel_mse(ref_b, got) <= REL_MSE
    # pre-rotated query and rotated output (R baked into Wo)
    R = tk.R.astype(np.float64)
    q_rot = (q.astype(np.float64) @ R.T).astype(np.float32)
    got_rot = cache.decode_attn(0, [0, 1], q_rot, 32, scale, flags=lc.LC_Q_ROTATED | lc.LC_OUT_ROTATED)
    back = (got_rot.astype(np.float64) @ tv.R.astype(np.float64))  # R^T applied: out = R^T o  =>  o R
    _assert_close(back.astype(np.float32), ref)


def test_partials_and_merge_split_sequence(lc, orc, gpu):
    """One context split by sequence over two shards, merged from (m, l, o) partials."""
    dim, hkv, hq, n = 128, 8, 32, 1500
    tk = orc.Tables.generate(dim, 4, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    K = helpers.kv(orc, 900, 1, hkv, n, dim)
    V = helpers.kv(orc, 901, 1, hkv, n, dim)
    cut = 700
    full = lc.CudaKvCache(1, hkv, dim, ck, max_seqs=3, max_pages=32, max_pages_per_seq=8)
    full.append(0, [0], K, V)
    full.append(0, [1], np.ascontiguousarray(K[:, :, :cut]), np.ascontiguousarray(V[:, :, :cut]))
    full.append(0, [2], np.ascontiguousarray(K[:, :, cut:]), np.ascontiguousarray(V[:, :, cut:]))
    q = helpers.queries(orc, 13, 1, hq, dim)
    scale = 1.0 / np.sqrt(dim)
    whole = full.decode_attn(0, [0], q, hq, scale)
    m1, l1, o1 = full.decode_partials(0, [1], q, hq, scale)
    m2, l2, o2 = full.decode_partials(0, [2], q, hq, scale)
    merged = full.merge_partials(np.stack([m1, m2]), np.stack([l1, l2]), np.stack([o1, o2]))
    # both are the same function; only the split-K boundaries (and so the f16
    # rounding of p) differ
    merged = merged.reshape(whole.shape)
    _assert_close(merged, whole)
    ref = orc.SimpleCache(orc.Compressor(tk), orc.Compressor(tk), 1, hkv, dim)
    for h in range(hkv):
        ref.store(0, h, K[0, h], V[0, h], n)
    _assert_close(merged, _oracle([ref], q, hkv, scale))


def test_decode_errors(lc, orc, gpu):
    cache, refs, tk, tv = _setup(lc, orc, 128, 4, 4, 8, [10], 1)
    q = helpers.queries(orc, 1, 1, 30, 128)
    with pytest.raises(lc.LumenError):
        cache.decode_attn(0, [0], q, 30, 1.0)  # 30 q heads not a multiple of 8 kv heads
    with pytest.raises(lc.LumenError):
        cache.decode_attn(0, [4], helpers.queries(orc, 1, 1, 32, 128), 32, 1.0)  # bad sequence id
