"""GPU: LKV2 snapshots of the cache (kv_disk.rs format), checked by the
independent restatement in oracle/lkv2.py.

- save -> the oracle parses the file: manifest JSON byte-identical to the
  oracle's serde_json restatement, ring bookkeeping per layer, arrays equal
  to the cache's backing rows (codes unpacked, QJL bits as +-1 bf16).
- save -> load into another sequence: identical backing rows and ring
  state, identical decode output (bit for bit), identical after both
  sequences take the same further appends (the ring continues as before).
- an oracle-written file loads into a fresh cache.
- refusals (fingerprint, bit widths, a corrupted byte) leave the target
  sequence as it was.
"""
import numpy as np
import pytest

import helpers
import lkv2

pytestmark = pytest.mark.gpu

HKV, DIM, KB, VB, M = 4, 128, 3, 2, 64
MAX_SIZE, KEEP = [0, 300], [0, 4]


def _cache(lc, orc, kb=KB, vb=VB, seqs=3):
    tk = orc.Tables.generate(DIM, kb, M, 42)
    tv = orc.Tables.generate(DIM, vb, M, 42)
    ck = lc.TurboQuantCompressor.from_tables(tk.R, tk.bounds, tk.cents, tk.proj)
    cv = lc.TurboQuantCompressor.from_tables(tv.R, tv.bounds, tv.cents, tv.proj)
    return lc.CudaKvCache(2, HKV, DIM, ck, cv, max_seqs=seqs, max_pages=seqs * 2 * 8 + 8, max_pages_per_seq=6,
                          store_flags=lc.LC_STORE_K_QJL | lc.LC_STORE_V_QJL,
                          layer_max_size=MAX_SIZE, layer_keep=KEEP)


def _fill(cache, orc, seq, seed):
    """Layer 0 (full): 700 tokens. Layer 1 (window 300, keep 4): 200 tokens,
    then 150 single-token steps, so the ring wraps."""
    K = helpers.kv(orc, seed, 1, HKV, 700, DIM)
    V = helpers.kv(orc, seed + 1, 1, HKV, 700, DIM)
    cache.append(0, [seq], K, V)
    cache.append(1, [seq], np.ascontiguousarray(K[:, :, :200]), np.ascontiguousarray(V[:, :, :200]))
    for t in range(200, 350):
        cache.append(1, [seq], np.ascontiguousarray(K[:, :, t:t + 1]), np.ascontiguousarray(V[:, :, t:t + 1]))


def _same_backing(lc, a, sa, b, sb):
    for layer in range(2):
        assert a.ring_state(sa, layer) == b.ring_state(sb, layer)
        fa, fb = a.fetch(sa, layer, lc.LC_FETCH_BACKING), b.fetch(sb, layer, lc.LC_FETCH_BACKING)
        for k in fa:
            np.testing.assert_array_equal(fa[k].view(np.uint8), fb[k].view(np.uint8), err_msg=f"{layer} {k}")


def test_save_matches_oracle_reader(lc, orc, gpu, tmp_path):
    cache = _cache(lc, orc)
    _fill(cache, orc, 0, 11)
    p = tmp_path / "a.lkv"
    cache.save_lkv2(0, p, "fp-test", prefix_tokens=[5, 6, 7])
    m, recs, js = lkv2.read(p)
    assert lkv2.manifest_json(m) == js  # the C writer's JSON is serde_json's compact form
    assert lc.lkv2_info(p) == {"layers": 2, "records": len(recs), "position": 700}
    assert m["model_fingerprint"] == "fp-test" and m["prefix_tokens"] == [5, 6, 7] and m["is_deep"]
    for layer, L in enumerate(m["layers"]):
        st = cache.ring_state(0, layer)
        assert L["kind"] == ("FullTurboquant" if layer == 0 else "SlidingTurboquant")
        assert (L["offset"], L["idx"], L["keep"], L["bits"], L["qjl_m"], L["v_bits"]) == \
            (st["offset"], st["idx"], KEEP[layer], KB, M, VB)
        f = cache.fetch(0, layer, lc.LC_FETCH_BACKING)
        S = st["buf_len"]
        arr = [recs[i].array() for i in L["arrays"]]
        np.testing.assert_array_equal(arr[0], lkv2.unpack_codes(f["k_words"], DIM, KB)[None])
        np.testing.assert_array_equal(arr[1].view(np.uint32), f["k_sigma"].reshape(1, HKV, S, 1).view(np.uint32))
        np.testing.assert_array_equal(arr[2], lkv2.unpack_codes(f["v_words"], DIM, VB)[None])
        np.testing.assert_array_equal(arr[3].view(np.uint32), f["v_sigma"].reshape(1, HKV, S, 1).view(np.uint32))
        np.testing.assert_array_equal(arr[4], lkv2.signs_pm1(f["k_qjl"], M)[None])
        np.testing.assert_array_equal(arr[5].view(np.uint32), f["k_rnorm"].reshape(1, HKV, S, 1).view(np.uint32))
        np.testing.assert_array_equal(arr[6], lkv2.signs_pm1(f["v_qjl"], M)[None])
        np.testing.assert_array_equal(arr[7].view(np.uint32), f["v_rnorm"].reshape(1, HKV, S, 1).view(np.uint32))
    assert m["layers"][1]["offset"] > MAX_SIZE[1]  # the window has wrapped
    cache.close()


def test_load_roundtrip_and_continue(lc, orc, gpu, tmp_path):
    cache = _cache(lc, orc)
    _fill(cache, orc, 0, 21)
    _fill(cache, orc, 1, 99)  # seq 1 holds other data before the load
    p = tmp_path / "b.lkv"
    cache.save_lkv2(0, p)
    cache.load_lkv2(1, p)
    _same_backing(lc, cache, 0, cache, 1)
    q = helpers.queries(orc, 23, 2, 16, DIM)
    for layer in range(2):
        out = cache.decode_attn(layer, [0, 1], q[[0, 0]], 16, DIM ** -0.5)
        np.testing.assert_array_equal(out[0], out[1])
    for t in range(5):  # the rings continue identically
        K = helpers.kv(orc, 300 + t, 1, HKV, 1, DIM)
        V = helpers.kv(orc, 400 + t, 1, HKV, 1, DIM)
        for layer in range(2):
            cache.append(layer, [0], K, V)
            cache.append(layer, [1], K, V)
    _same_backing(lc, cache, 0, cache, 1)
    cache.close()


def test_load_oracle_written_file(lc, orc, gpu, tmp_path):
    src = _cache(lc, orc)
    _fill(src, orc, 0, 31)
    src.save_lkv2(0, tmp_path / "c.lkv")
    m, _, _ = lkv2.read(tmp_path / "c.lkv")
    # rebuild the records from fetched rows with the oracle alone
    new_recs, layers = [], []
    for layer in range(2):
        st = src.ring_state(0, layer)
        f = src.fetch(0, layer, lc.LC_FETCH_BACKING)
        S = st["buf_len"]
        arrays = []
        for dt, a in [(lkv2.U8, lkv2.unpack_codes(f["k_words"], DIM, KB)[None]),
                      (lkv2.F32, f["k_sigma"].reshape(1, HKV, S, 1)),
                      (lkv2.U8, lkv2.unpack_codes(f["v_words"], DIM, VB)[None]),
                      (lkv2.F32, f["v_sigma"].reshape(1, HKV, S, 1)),
                      (lkv2.BF16, lkv2.signs_pm1(f["k_qjl"], M)[None]),
                      (lkv2.F32, f["k_rnorm"].reshape(1, HKV, S, 1)),
                      (lkv2.BF16, lkv2.signs_pm1(f["v_qjl"], M)[None]),
                      (lkv2.F32, f["v_rnorm"].reshape(1, HKV, S, 1))]:
            arrays.append(len(new_recs))
            new_recs.append(lkv2.record(dt, a))
        layers.append({"kind": "FullTurboquant" if layer == 0 else "SlidingTurboquant", "offset": st["offset"],
                       "base_offset": 0, "arrays": arrays, "max_size": m["layers"][layer]["max_size"],
                       "keep": KEEP[layer], "idx": st["idx"], "bits": KB, "qjl_m": M, "v_bits": VB})
    man = {"model_fingerprint": "", "created_at_unix": 1, "position": 700, "prefix_tokens": [], "is_deep": True,
           "layers": layers}
    p = tmp_path / "d.lkv"
    lkv2.write(p, man, new_recs)
    dst = _cache(lc, orc)
    dst.load_lkv2(2, p, "")
    _same_backing(lc, src, 0, dst, 2)
    src.close()
    dst.close()


def test_load_refusals_leave_the_sequence(lc, orc, gpu, tmp_path):
    cache = _cache(lc, orc)
    _fill(cache, orc, 0, 41)
    _fill(cache, orc, 1, 51)
    p = tmp_path / "e.lkv"
    cache.save_lkv2(0, p, "fp-1")
    before = [cache.ring_state(1, layer) for layer in range(2)]
    f_before = cache.fetch(1, 1, lc.LC_FETCH_BACKING)
    with pytest.raises(lc.LumenError) as e:
        cache.load_lkv2(1, p, "fp-2")
    assert e.value.code == lc.LC_ERR_STATE
    other = _cache(lc, orc, kb=4, vb=4)
    with pytest.raises(lc.LumenError) as e:
        other.load_lkv2(0, p)
    assert e.value.code == lc.LC_ERR_BITS
    other.close()
    b = bytearray(p.read_bytes())
    b[len(b) // 2] ^= 0x10
    bad = tmp_path / "f.lkv"
    bad.write_bytes(bytes(b))
    with pytest.raises(lc.LumenError) as e:
        cache.load_lkv2(1, bad)
    assert e.value.code == lc.LC_ERR_IO
    assert [cache.ring_state(1, layer) for layer in range(2)] == before
    f_after = cache.fetch(1, 1, lc.LC_FETCH_BACKING)
    for k in f_before:
        np.testing.assert_array_equal(f_before[k].view(np.uint8), f_after[k].view(np.uint8))
    cache.close()
