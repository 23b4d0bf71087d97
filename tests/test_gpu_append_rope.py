"""GPU: lc_append_rope, RoPE fused into quantize-append, bit-exact against the
oracle applying the same RoPE (orc_rope) and then compress_one.

Positions continue each sequence's layer: the sequences start at different
lengths, and the chunk sizes reach both append kernels (the warp kernel for
decode steps; past 16384 vectors the batched kernel with QJL stage 2, the
register-blocked tile kernel without). Both pair layouts and partial rotary
dims are covered. Values are not rotated.
"""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dim,kb,vb,m,rot,trad,chunks,qjl", [
    (128, 4, 4, 64, 128, False, [5, 1, 1], True),        # warp kernel, half-split pairs
    (128, 3, 2, 64, 64, True, [3, 1], True),             # partial rotary, traditional pairs
    (128, 4, 4, 64, 128, False, [2300], True),           # 2 x 8 x 2300 vectors: the batched kernel
    (128, 4, 4, 64, 96, True, [1100, 1201], False),      # no QJL: the register-blocked tile kernel
])
def test_append_rope_bit_exact(lc, orc, gpu, dim, kb, vb, m, rot, trad, chunks, qjl):
    tk = orc.Tables.generate(dim, kb, m, 42)
    tv = orc.Tables.generate(dim, vb, m, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    H, B, base = 8, 2, 10000.0
    start = [37, 300]  # tokens each sequence holds before the RoPE appends
    total = [start[b] + sum(chunks) for b in range(B)]
    pages = (max(total) + 255) // 256 + 3  # the append bounds prealloc growth up front
    cache = lc.CudaKvCache(1, H, dim, ck, cv, max_seqs=B, max_pages=B * pages + 8, max_pages_per_seq=pages,
                           store_flags=(lc.LC_STORE_K_QJL | lc.LC_STORE_V_QJL) if qjl else 0)
    K = [helpers.kv(orc, 500 + b, 1, H, total[b], dim)[0] for b in range(B)]
    V = [helpers.kv(orc, 600 + b, 1, H, total[b], dim)[0] for b in range(B)]
    for b in range(B):  # plain appends first: the prefix without RoPE
        cache.append(0, [b], np.ascontiguousarray(K[b][None, :, :start[b]]),
                     np.ascontiguousarray(V[b][None, :, :start[b]]))
    off = 0
    for n in chunks:
        k = np.stack([K[b][:, start[b] + off:start[b] + off + n] for b in range(B)])
        v = np.stack([V[b][:, start[b] + off:start[b] + off + n] for b in range(B)])
        cache.append_rope(0, list(range(B)), np.ascontiguousarray(k), np.ascontiguousarray(v), rot, base, trad)
        off += n
    kc, vc = orc.Compressor(tk), orc.Compressor(tv)
    for b in range(B):
        f = cache.fetch(b, 0)
        for h in range(H):
            kr = K[b][h].copy()
            kr[start[b]:] = orc.rope(kr[start[b]:], rot, start[b], base, trad)
            for side, (x, comp) in enumerate([(kr, kc), (V[b][h], vc)]):
                s1, s2, rn, sc = comp.compress(x)
                p = "kv"[side]
                np.testing.assert_array_equal(f[f"{p}_words"][h], s1, err_msg=f"{b} {h} {p}")
                np.testing.assert_array_equal(f[f"{p}_sigma"][h].view(np.uint32), sc.view(np.uint32))
                if qjl:
                    np.testing.assert_array_equal(f[f"{p}_qjl"][h], s2)
                    np.testing.assert_array_equal(f[f"{p}_rnorm"][h].view(np.uint32), rn.view(np.uint32))
    cache.close()


def test_append_rope_refusals(lc, orc, gpu):
    t = orc.Tables.generate(128, 4, 64, 42)
    c = lc.TurboQuantCompressor.from_tables(t.R, t.bounds, t.cents, t.proj)
    cache = lc.CudaKvCache(1, 2, 128, c, max_seqs=1, max_pages=4, max_pages_per_seq=2)
    k = helpers.kv(orc, 1, 1, 2, 3, 128)
    for dims in (0, 3, 130):
        with pytest.raises(lc.LumenError) as e:
            cache.append_rope(0, [0], k, k, dims)
        assert e.value.code == lc.LC_ERR_INVALID
    assert cache.seq_len(0, 0, 0) == 0  # nothing was appended
    cache.close()
