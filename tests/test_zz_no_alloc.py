"""GPU: lc_decode_attn_noalloc, the decode entry point whose scratch is a
fixed device array, against lc_decode_attn on the same cache and queries,
and against the oracle where the no-alloc call uploads block-table rows
itself.

Called through the C ABI with device tensors. The two entry points run the
same kernels, so the bar is the decode tolerance of helpers.attn_close
(per row 2e-3 absolute + 1e-3 of the row's scale, relative MSE 1e-3). Each
case makes two no-alloc calls in a row. The file is named to be collected
last, so the scratch set-up (first call on the device) is exercised both
after every other GPU test in one process and alone in a fresh one.
"""
import ctypes as C

import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _cache(lc, orc, dim, kb, vb, hkv, lens, seed):
    tk = orc.Tables.generate(dim, kb, 64, 42)
    tv = orc.Tables.generate(dim, vb, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    pages = (max(lens) + 255) // 256 + 2
    cache = lc.CudaKvCache(1, hkv, dim, ck, cv, max_seqs=len(lens), max_pages=len(lens) * pages + 8,
                           max_pages_per_seq=pages)
    for b, n in enumerate(lens):
        cache.append(0, [b], helpers.kv(orc, seed + 2 * b, 1, hkv, n, dim),
                     helpers.kv(orc, seed + 2 * b + 1, 1, hkv, n, dim))
    return cache


def _noalloc(lc, cache, ids, q, hq, scale, flags, out, out_dtype):
    import torch

    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream or lc.CUDA_STREAM_LEGACY)
    ids = np.ascontiguousarray(ids, np.int32)
    qd = lc.LC_BF16 if q.dtype == torch.bfloat16 else lc.LC_F32
    return lc.lib().lc_decode_attn_noalloc(cache._h, 0, len(ids), ids.ctypes.data, q.data_ptr(), qd, hq,
                                           C.c_float(scale), flags, out.data_ptr(), out_dtype, stream)


def _check_case(lc, orc, dim, kb, vb, hkv, hq, lens, flags, out_dtype):
    import torch

    cache = _cache(lc, orc, dim, kb, vb, hkv, lens, 900 + dim + kb)
    B = len(lens)
    ids = np.arange(B, dtype=np.int32)[::-1].copy()
    q = torch.from_numpy(helpers.queries(orc, 31, B, hq, dim, std=dim ** -0.5)).to(torch.bfloat16).cuda()
    scale = float(1.0 / np.sqrt(dim))
    tdt = torch.float32 if out_dtype == lc.LC_F32 else torch.bfloat16
    ref = torch.empty((B, hq, dim), dtype=tdt, device="cuda")
    cache.decode_attn(0, ids, q, hq, scale, flags, out=ref, out_dtype=out_dtype)
    torch.cuda.synchronize()
    ref = ref.float().cpu().numpy()
    for call in range(2):
        out = torch.full((B, hq, dim), float("nan"), dtype=tdt, device="cuda")
        st = _noalloc(lc, cache, ids, q, hq, scale, flags, out, out_dtype)
        assert st == lc.LC_OK, lc.lib().lc_last_error().decode()
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: unwritten output"
        ok, msg = helpers.attn_close(got, ref)
        assert ok, f"call {call}: {msg}"
    cache.close()


def test_noalloc_fast_path(lc, orc, gpu):
    """4-bit d=128 GQA 4 (the flat split-K kernel), ragged lengths."""
    _check_case(lc, orc, 128, 4, 4, 8, 32, [1000, 257, 33, 640], 0, lc.LC_F32)


def test_noalloc_generic_rotated_bf16(lc, orc, gpu):
    """3-bit K / 2-bit V, d=256 (the chunked kernel), rotated q and output, bf16 out."""
    _check_case(lc, orc, 256, 3, 2, 8, 16, [700, 1300], lc.LC_Q_ROTATED | lc.LC_OUT_ROTATED, lc.LC_BF16)


def test_noalloc_uploads_its_own_block_table(lc, orc, gpu):
    """Called straight after appends, with no lc_decode_attn before it: the
    block-table rows of the sequences are dirty, and lc_decode_attn_noalloc
    stages them through its fixed host array and uploads them itself (three
    rows, so the staging offset steps). Appending past a page boundary makes
    two rows dirty again for the second call. Both calls are checked against
    the oracle's attend_keys -> softmax -> attend_values, and the second also
    against lc_decode_attn, which runs only afterwards."""
    import torch

    dim, hkv, hq = 128, 8, 32
    t = orc.Tables.generate(dim, 4, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(t.R, t.bounds, t.cents, t.proj)
    lens = [250, 510, 100]
    cache = lc.CudaKvCache(1, hkv, dim, ck, max_seqs=3, max_pages=24, max_pages_per_seq=4)
    comp = orc.Compressor(t)
    refs = [orc.SimpleCache(comp, comp, 1, hkv, dim) for _ in lens]

    def add(b, n, seed):
        K = helpers.kv(orc, seed, 1, hkv, n, dim)
        V = helpers.kv(orc, seed + 1, 1, hkv, n, dim)
        cache.append(0, [b], K, V)
        for h in range(hkv):
            refs[b].store(0, h, K[0, h], V[0, h], n)

    for b, n in enumerate(lens):
        add(b, n, 40 + 2 * b)
    ids = np.array([2, 0, 1], np.int32)
    qn = helpers.queries(orc, 41, 3, hq, dim, std=dim ** -0.5)
    q = torch.from_numpy(qn).cuda()
    scale = float(dim ** -0.5)

    def oracle():
        return np.stack([np.stack([refs[b].attend(0, h // (hq // hkv), qn[i, h], scale) for h in range(hq)])
                         for i, b in enumerate(ids)])

    out = torch.full((3, hq, dim), float("nan"), device="cuda")
    st = _noalloc(lc, cache, ids, q, hq, scale, 0, out, lc.LC_F32)
    assert st == lc.LC_OK, lc.lib().lc_last_error().decode()
    torch.cuda.synchronize()
    ok, msg = helpers.attn_close(out.cpu().numpy(), oracle())
    assert ok, f"first call: {msg}"
    add(0, 20, 60)  # 250 -> 270 tokens: a second page
    add(1, 20, 62)  # 510 -> 530 tokens: a third page
    out2 = torch.full((3, hq, dim), float("nan"), device="cuda")
    st = _noalloc(lc, cache, ids, q, hq, scale, 0, out2, lc.LC_F32)
    assert st == lc.LC_OK, lc.lib().lc_last_error().decode()
    torch.cuda.synchronize()
    got2 = out2.cpu().numpy()
    ok, msg = helpers.attn_close(got2, oracle())
    assert ok, f"second call: {msg}"
    ref = torch.empty((3, hq, dim), device="cuda")
    cache.decode_attn(0, ids, q, hq, scale, out=ref, out_dtype=lc.LC_F32)
    torch.cuda.synchronize()
    ok, msg = helpers.attn_close(got2, ref.cpu().numpy())
    assert ok, f"second call vs lc_decode_attn: {msg}"
    cache.close()


def test_noalloc_refusals(lc, orc, gpu):
    """Host buffers and calls larger than the fixed scratch are refused with a
    clear error before any work is issued; the cache stays usable."""
    import torch

    hkv, dim = 8, 128
    cache = _cache(lc, orc, dim, 4, 4, hkv, [300, 300], 77)
    ids = np.arange(2, dtype=np.int32)
    q = torch.from_numpy(helpers.queries(orc, 5, 2, 32, dim)).to(torch.bfloat16).cuda()
    out = torch.empty((2, 32, dim), device="cuda")
    q_host = q.cpu()
    st = lc.lib().lc_decode_attn_noalloc(cache._h, 0, 2, ids.ctypes.data, q_host.data_ptr(), lc.LC_BF16, 32,
                                         C.c_float(1.0), 0, out.data_ptr(), lc.LC_F32, None)
    assert st == lc.LC_ERR_INVALID and b"device memory" in lc.lib().lc_last_error()
    # QJL scores are not taken here
    st = _noalloc(lc, cache, ids, q, 32, 1.0, lc.LC_QJL_SCORES, out, lc.LC_F32)
    assert st == lc.LC_ERR_INVALID and b"LC_QJL_SCORES" in lc.lib().lc_last_error()
    # 2 x 32768 query heads: rows * head_dim * 6 alone is 48 MiB > 32 MiB
    big_hq = 8 * 1024 * 4
    qb = torch.zeros((2, big_hq, dim), dtype=torch.bfloat16, device="cuda")
    ob = torch.empty((2, big_hq, dim), dtype=torch.bfloat16, device="cuda")
    st = _noalloc(lc, cache, ids, qb, big_hq, 1.0, 0, ob, lc.LC_BF16)
    assert st == lc.LC_ERR_NOMEM
    assert b"LC_NOALLOC_SCRATCH_BYTES" in lc.lib().lc_last_error()
    del qb, ob
    ref = torch.empty((2, 32, dim), device="cuda")
    cache.decode_attn(0, ids, q, 32, 0.1, out=ref, out_dtype=lc.LC_F32)
    st = _noalloc(lc, cache, ids, q, 32, 0.1, 0, out, lc.LC_F32)
    assert st == lc.LC_OK, lc.lib().lc_last_error().decode()
    torch.cuda.synchronize()
    ok, msg = helpers.attn_close(out.cpu().numpy(), ref.cpu().numpy())
    assert ok, msg
    cache.close()
