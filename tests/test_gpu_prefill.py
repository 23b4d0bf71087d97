"""GPU: causal prefill attention over the compressed cache (lc_prefill_attn).

After a chunk of L tokens has been appended, query i of the chunk attends to
the first view_len - L + i + 1 tokens (the masked prefill of
gemma4_moe.rs:4636-4660, on the codes). The oracle composes SimpleCache's
attend_keys -> softmax over that prefix -> attend_values
(orc_sc_attend_prefix); parity is the decode tolerance (helpers.attn_close).
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _setup(lc, orc, dim, kb, vb, hkv, prefix, chunk, seed, max_size=0, keep=0):
    tk = orc.Tables.generate(dim, kb, 64, 42)
    tv = orc.Tables.generate(dim, vb, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    n = prefix + chunk
    pages = (n + 255) // 256 + 1
    cache = lc.CudaKvCache(1, hkv, dim, ck, cv, max_seqs=1, max_pages=pages + 8, max_pages_per_seq=pages,
                           layer_max_size=[max_size], layer_keep=[keep])
    K = helpers.kv(orc, seed, 1, hkv, n, dim)
    V = helpers.kv(orc, seed + 1, 1, hkv, n, dim)
    if prefix:
        cache.append(0, [0], np.ascontiguousarray(K[:, :, :prefix]), np.ascontiguousarray(V[:, :, :prefix]))
    cache.append(0, [0], np.ascontiguousarray(K[:, :, prefix:]), np.ascontiguousarray(V[:, :, prefix:]))
    ref = orc.SimpleCache(orc.Compressor(tk), orc.Compressor(tv), 1, hkv, dim)
    for h in range(hkv):
        ref.store(0, h, K[0, h], V[0, h], n)
    return cache, ref


def _oracle(ref, q, hkv, scale, n_total):
    L, hq, dim = q.shape
    G = hq // hkv
    out = np.zeros((L, hq, dim), np.float32)
    for i in range(L):
        for h in range(hq):
            out[i, h] = ref.attend_prefix(0, h // G, q[i, h], scale, n_total - L + i + 1)
    return out


@pytest.mark.parametrize("dim,kb,vb,hkv,hq,prefix,chunk", [
    (128, 4, 4, 8, 32, 500, 40),   # fast path geometry (config 1 heads)
    (128, 4, 4, 8, 32, 0, 300),    # the chunk is the whole sequence
    (128, 3, 2, 4, 8, 300, 24),    # generic path
])
def test_prefill_matches_oracle(lc, orc, gpu, dim, kb, vb, hkv, hq, prefix, chunk):
    cache, ref = _setup(lc, orc, dim, kb, vb, hkv, prefix, chunk, 100 + prefix + chunk)
    q = helpers.queries(orc, 7, chunk, hq, dim)
    scale = 1.0 / np.sqrt(dim)
    got = cache.prefill_attn(0, 0, q, hq, scale)
    ok, msg = helpers.attn_close(got, _oracle(ref, q, hkv, scale, prefix + chunk))
    assert ok, msg
    cache.close()


def test_prefill_one_token_is_decode(lc, orc, gpu):
    """A one-token chunk is a decode step of that token (the tiled prefill
    kernel and the decode kernel agree within the decode tolerance)."""
    cache, ref = _setup(lc, orc, 128, 4, 4, 8, 700, 1, 5)
    q = helpers.queries(orc, 8, 1, 32, 128)
    a = cache.prefill_attn(0, 0, q, 32, 0.1)
    b = cache.decode_attn(0, [0], q, 32, 0.1)
    ok, msg = helpers.attn_close(a, b)
    assert ok, msg
    ok, msg = helpers.attn_close(a, _oracle(ref, q, 8, 0.1, 701))
    assert ok, msg
    cache.close()


@pytest.mark.parametrize("hkv,hq,prefix,chunk", [
    (4, 4, 700, 130),    # G 1: 128 tokens per block, two blocks
    (8, 24, 3000, 64),   # G 3: 42 tokens per block, 2 rows per block unused
    (2, 12, 1000, 77),   # G 6: 21 tokens per block
    (2, 16, 256, 200),   # G 8: 16 tokens per block, a page-aligned prefix
    (8, 32, 63, 65),     # G 4: the chunk straddles key tiles
])
def test_prefill_tiled_group_sizes(lc, orc, gpu, hkv, hq, prefix, chunk):
    """The tensor-core prefill kernel (4-bit, d 128) over GQA 1-8, ragged
    chunks and prefixes that do not align with the 64-key tiles."""
    cache, ref = _setup(lc, orc, 128, 4, 4, hkv, prefix, chunk, 300 + hq + chunk)
    q = helpers.queries(orc, 11 + hq, chunk, hq, 128)
    scale = 1.0 / np.sqrt(128)
    got = cache.prefill_attn(0, 0, q, hq, scale)
    ok, msg = helpers.attn_close(got, _oracle(ref, q, hkv, scale, prefix + chunk))
    assert ok, msg
    cache.close()


def _unit_rms(q):
    return (q / np.sqrt(np.mean(q.astype(np.float64) ** 2, axis=-1, keepdims=True))).astype(np.float32)


def test_prefill_tiled_peaked_scale1(lc, orc, gpu):
    """The reference's production regime (scale 1.0 on unit-RMS queries,
    gemma4_moe.rs:4642-4660): peaked softmax, where the kernel's precise
    tiles (K table residuals) must keep the decode tolerance. Device bf16
    queries, f32 output on the device."""
    import torch

    cache, ref = _setup(lc, orc, 128, 4, 4, 8, 2000, 96, 41)
    q = _unit_rms(helpers.queries(orc, 12, 96, 32, 128))
    qt, qv = helpers.to_bf16(q)
    out = torch.empty((96, 32, 128), dtype=torch.float32, device="cuda")
    cache.prefill_attn(0, 0, qt.cuda(), 32, 1.0, out=out, out_dtype=lc.LC_F32)
    torch.cuda.synchronize()
    ok, msg = helpers.attn_close(out.cpu().numpy(), _oracle(ref, qv, 8, 1.0, 2096))
    assert ok, msg
    cache.close()


def test_prefill_tiled_out_rotated(lc, orc, gpu):
    """LC_OUT_ROTATED leaves the tiled prefill's output in V's rotated basis:
    un-rotating it on the host gives the normal output."""
    cache, ref = _setup(lc, orc, 128, 4, 4, 8, 500, 40, 77)
    q = helpers.queries(orc, 13, 40, 32, 128)
    a = cache.prefill_attn(0, 0, q, 32, 0.1)
    b = cache.prefill_attn(0, 0, q, 32, 0.1, flags=lc.LC_OUT_ROTATED)
    tv = orc.Tables.generate(128, 4, 64, 42)
    R = np.asarray(tv.R, np.float64).reshape(128, 128)
    np.testing.assert_allclose(b.astype(np.float64) @ R, a, atol=2e-4)
    cache.close()


def test_prefill_sliding_window(lc, orc, gpu):
    # a ring of 1024 holding 600 tokens has not wrapped: plain causal prefill
    cache, ref = _setup(lc, orc, 128, 4, 4, 8, 560, 40, 9, max_size=1024, keep=4)
    q = helpers.queries(orc, 10, 40, 32, 128)
    got = cache.prefill_attn(0, 0, q, 32, 0.1)
    ok, msg = helpers.attn_close(got, _oracle(ref, q, 8, 0.1, 600))
    assert ok, msg
    cache.close()


def test_prefill_refusals(lc, orc, gpu):
    cache, _ = _setup(lc, orc, 128, 4, 4, 8, 300, 20, 11, max_size=256, keep=4)  # wrapped ring
    q = helpers.queries(orc, 12, 20, 32, 128)
    with pytest.raises(lc.LumenError) as e:
        cache.prefill_attn(0, 0, q, 32, 0.1)
    assert e.value.code == lc.LC_ERR_STATE
    cache.close()
    cache, _ = _setup(lc, orc, 128, 4, 4, 8, 0, 10, 13)
    with pytest.raises(lc.LumenError) as e:
        cache.prefill_attn(0, 0, helpers.queries(orc, 14, 11, 32, 128), 32, 0.1)
    assert e.value.code == lc.LC_ERR_INVALID
    cache.close()
