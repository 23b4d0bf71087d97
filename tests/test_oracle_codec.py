"""CPU: the oracle restatement against the reference's own unit tests.

Each test restates a test of rabbitson87/lumen-rs (file:line given) with the
same thresholds, driven by the oracle's seeded generator instead of Rust's
StdRng (whose stream is not available here).
"""
import numpy as np
import pytest


def cosine(a, b):
    """lumen-testkit cosine (crates/lumen-testkit/src/lib.rs:45-60): f64 accumulation."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    na, nb = (a * a).sum(), (b * b).sum()
    if na == 0 and nb == 0:
        return 1.0
    if na == 0 or nb == 0:
        return 0.0
    return float((a * b).sum() / (np.sqrt(na) * np.sqrt(nb)))


# ---------------------------------------------------------------- lloyd_max.rs
def test_codebook_3bit_mse(orc):  # lloyd_max.rs:220-227
    b, c = orc.lloyd_max(3)
    assert orc.codebook_mse(3, b, c) <= 0.035


def test_codebook_symmetry(orc):  # lloyd_max.rs:229-243
    _, c = orc.lloyd_max(3)
    for i in range(4):
        assert abs(c[i] + c[7 - i]) < 1e-10


def test_centroid_maps_to_own_code(orc):  # lloyd_max.rs:245-253
    b, c = orc.lloyd_max(3)
    for i, ci in enumerate(c):
        assert orc.quantize(b, 3, ci) == i


def test_vec_quantize_roundtrip(orc):  # lloyd_max.rs:255-265
    b, c = orc.lloyd_max(3)
    for x in (-2.0, -1.0, 0.0, 1.0, 2.0):
        assert abs(x - c[orc.quantize(b, 3, x)]) < 1.0


def test_empirical_mse_matches_analytical(orc):  # lloyd_max.rs:267-293
    b, c = orc.lloyd_max(3)
    xs = orc.gauss_f64(123, 100_000)
    codes = np.array([orc.quantize(b, 3, x) for x in xs])
    emp = float(np.mean((xs - c[codes]) ** 2))
    ana = orc.codebook_mse(3, b, c)
    assert abs(emp - ana) < 0.002
    assert emp <= 0.036


def test_codebook_2bit_and_4bit(orc):  # lloyd_max.rs:310-322
    for bits in (2, 4):
        b, c = orc.lloyd_max(bits)
        assert len(c) == 1 << bits
        if bits == 4:
            assert orc.codebook_mse(bits, b, c) < 0.01


def test_invalid_bits(orc):  # lloyd_max.rs:75-77
    for bits in (0, 9):
        with pytest.raises(ValueError):
            orc.lloyd_max(bits)


# Published optimum Lloyd-Max quantizer levels for a unit Gaussian (Max, 1960),
# positive half; the A&S 7.1.26 erf used by the reference moves them < 5e-4.
MAX_1960 = {
    1: [0.7979],
    2: [0.4528, 1.5104],
    3: [0.2451, 0.7560, 1.3439, 2.1520],
    4: [0.1284, 0.3881, 0.6568, 0.9424, 1.2562, 1.6181, 2.0690, 2.7326],
}


@pytest.mark.parametrize("bits", [1, 2, 3, 4])
def test_codebook_matches_published_levels(orc, bits):
    _, c = orc.lloyd_max(bits)
    n = 1 << bits
    np.testing.assert_allclose(c[n // 2:], MAX_1960[bits], atol=5e-4)


# ------------------------------------------------------------------ bitpack.rs
@pytest.mark.parametrize("bits,n,words", [(3, 256, 13), (2, 128, 4), (4, 64, 4)])
def test_pack_unpack_roundtrip(orc, bits, n, words):  # bitpack.rs:58-84
    codes = (np.arange(n) % (1 << bits)).astype(np.uint8)
    packed = orc.pack_codes(codes, bits)
    assert len(packed) == words
    np.testing.assert_array_equal(orc.unpack_codes(packed, n, bits), codes)


def test_packed_size_bytes(orc):  # bitpack.rs:86-94
    assert orc.packed_words(256, 3) * 8 == 104
    assert orc.packed_words(256, 2) * 8 == 64
    assert orc.packed_words(512, 3) * 8 == 200


def test_compression_ratio(orc):  # bitpack.rs:96-108
    assert 256 / (orc.packed_words(256, 3) * 8) > 2.0


def test_3bit_word_top_bit_unused(orc):  # bitpack.rs:4: 21 codes per u64, 1 bit unused
    codes = np.full(256, 7, np.uint8)
    packed = orc.pack_codes(codes, 3)
    assert all(int(w) >> 63 == 0 for w in packed)


# ---------------------------------------------------------------------- qjl.rs
def test_qjl_packed_len(orc):  # qjl.rs:403-412
    for m, w in [(0, 0), (1, 1), (63, 1), (64, 1), (65, 2), (128, 2), (129, 3)]:
        assert orc.qjl_packed_len(m) == w


def test_qjl_last_word_masking(orc):  # qjl.rs:414-429
    P = orc.qjl_generate(32, 65, 42)
    res = orc.gauss_f32(99, 32)
    packed = orc.qjl_project_and_pack(P, res)
    assert len(packed) == 2
    assert int(packed[1]) & ~1 == 0


def test_qjl_deterministic(orc):  # qjl.rs:279-293
    P = orc.qjl_generate(64, 128, 42)
    res = orc.gauss_f32(99, 64)
    a = orc.qjl_project_and_pack(P, res)
    assert len(a) == orc.qjl_packed_len(128)
    np.testing.assert_array_equal(a, orc.qjl_project_and_pack(P, res))


def test_qjl_unbiased(orc):  # qjl.rs:295-332
    dim, m = 128, 256
    P = orc.qjl_generate(dim, m, 42)
    total = 0.0
    g = orc.gauss_f32(99, 2000 * 2 * dim).reshape(2000, 2, dim)
    for k in range(2000):
        r, q = g[k, 0], g[k, 1]
        true = float(np.float32(np.dot(q.astype(np.float64), r.astype(np.float64))))
        rn = float(np.sqrt(np.sum(r.astype(np.float64) ** 2)))
        est = orc.qjl_estimate_correction(P, q, orc.qjl_project_and_pack(P, r), rn)
        total += est - true
    assert abs(total / 2000) < 1.0


# ----------------------------------------------------------------- rotation.rs
def test_rotation_orthogonality(orc):  # rotation.rs:157-173
    R = orc.rotation_generate(128, 42)
    err = np.abs(R.astype(np.float32) @ R.T.astype(np.float32) - np.eye(128, dtype=np.float32)).max()
    assert err < 1e-5


def test_rotation_inverse_roundtrip(orc):  # rotation.rs:175-193
    R = orc.rotation_generate(128, 42)
    x = orc.gauss_f32(99, 128)
    back = orc.rotation_apply_inverse(R, orc.rotation_apply(R, x))
    assert np.abs(back - x).max() < 1e-4


def test_rotation_norm_preservation(orc):  # rotation.rs:195-210
    R = orc.rotation_generate(128, 42)
    x = orc.gauss_f32(77, 128)
    y = orc.rotation_apply(R, x)
    nx, ny = np.sqrt(np.sum(x * x)), np.sqrt(np.sum(y * y))
    assert abs(nx - ny) / nx < 1e-5


def test_rotation_deterministic(orc):  # rotation.rs:212-217
    np.testing.assert_array_equal(orc.rotation_generate(64, 42), orc.rotation_generate(64, 42))
    assert not np.array_equal(orc.rotation_generate(64, 42), orc.rotation_generate(64, 43))


# --------------------------------------------------------------- compressor.rs
def _tables(orc, bits, m, dim=128, seed=42):
    return orc.Tables.generate(dim, bits, m, seed)


def test_stage1_only_3bit_cosine(orc):  # compressor.rs:242-277
    comp = orc.Compressor(_tables(orc, 3, 64))
    X = orc.gauss_f32(99, 200 * 128).reshape(200, 128)
    s1, s2, rn, sc = comp.compress(X)
    Q = orc.gauss_f32(1234, 50 * 128).reshape(50, 128)
    cs = [cosine(X @ q, comp.estimate_stage1(q, s1, sc)) for q in Q]
    assert np.mean(cs) >= 0.98


def test_two_stage_3bit_m512_cosine(orc):  # compressor.rs:279-293
    comp = orc.Compressor(_tables(orc, 3, 512))
    X = orc.gauss_f32(99, 200 * 128).reshape(200, 128)
    s1, s2, rn, sc = comp.compress(X)
    Q = orc.gauss_f32(4321, 50 * 128).reshape(50, 128)
    cs = [cosine(X @ q, comp.estimate(q, s1, sc, s2, rn)) for q in Q]
    assert np.mean(cs) >= 0.99
    assert np.min(cs) >= 0.95


def test_stage1_reconstruction_quality(orc):  # compressor.rs:295-324
    t = _tables(orc, 3, 64)
    comp = orc.Compressor(t)
    x = orc.gauss_f32(77, 128)
    cv = comp.compress_one(x)
    codes = orc.unpack_codes(cv["stage1"], 128, 3)
    recon = orc.rotation_apply_inverse(t.R, t.cents[codes].astype(np.float32))
    assert cosine(x, recon) >= 0.98


def test_zero_vector_guard(orc):  # compressor.rs:73-75
    comp = orc.Compressor(_tables(orc, 4, 64))
    cv = comp.compress_one(np.zeros(128, np.float32))
    assert cv["scale"] == 0.0
    assert not cv["codes"].any()


def test_compress_matches_compress_one(orc):  # compressor.rs:110-116
    comp = orc.Compressor(_tables(orc, 4, 64))
    X = orc.gauss_f32(5, 8 * 128).reshape(8, 128)
    s1, s2, rn, sc = comp.compress(X)
    for i in range(8):
        cv = comp.compress_one(X[i])
        np.testing.assert_array_equal(s1[i], cv["stage1"])
        np.testing.assert_array_equal(s2[i], cv["stage2"])
        assert rn[i] == cv["residual_norm"] and sc[i] == cv["scale"]


# ---------------------------------------------------------- turboquant-cache
def _cache(orc, bits=3, dim=64, layers=2, heads=4):
    comp = orc.Compressor(_tables(orc, bits, 64, dim))
    return comp, orc.SimpleCache(comp, comp, layers, heads, dim)


def test_simple_store_and_attend(orc):  # simple.rs:195-258
    comp, cache = _cache(orc)
    g = orc.gauss_f32(42, 10 * 64 * 2 + 64)
    keys, values, q = g[:640].reshape(10, 64), g[640:1280].reshape(10, 64), g[1280:]
    cache.store(0, 0, keys, values, 10)
    assert cache.seq_len(0, 0) == 10 and cache.seq_len(0, 1) == 0
    scores = cache.attend_keys(0, 0, q)
    assert len(scores) == 10
    w = np.exp(scores.astype(np.float64))
    w = (w / w.sum()).astype(np.float32)
    out = cache.attend_values(0, 0, w)
    expected = (w[:, None].astype(np.float64) * values).sum(0)
    assert cosine(out, expected) > 0.95


def test_simple_memory_ratio(orc):  # simple.rs:260-288
    comp, cache = _cache(orc, layers=1, heads=1)
    g = orc.gauss_f32(42, 100 * 64 * 2)
    cache.store(0, 0, g[:6400], g[6400:], 100)
    assert 100 * 64 * 4 * 2 / cache.memory_bytes() > 2.0


def test_simple_truncate(orc):  # simple.rs:290-322
    comp, cache = _cache(orc, bits=3, dim=128, layers=1, heads=2)
    g = orc.gauss_f32(7, 6 * 256)
    for i in range(6):
        cache.store(0, 0, g[i * 256:i * 256 + 128], g[i * 256 + 128:(i + 1) * 256], 1)
        cache.store(0, 1, g[i * 256:i * 256 + 128], g[i * 256 + 128:(i + 1) * 256], 1)
    assert cache.seq_len(0, 0) == 6 and cache.seq_len(0, 1) == 6
    cache.truncate(0, 4)
    assert cache.seq_len(0, 0) == 4 and cache.seq_len(0, 1) == 4
    cache.truncate(0, 10)
    assert cache.seq_len(0, 0) == 4
    cache.truncate(0, 0)
    assert cache.seq_len(0, 0) == 0 and cache.seq_len(0, 1) == 0


def test_simple_incremental_store_and_clear(orc):  # simple.rs:324-346
    comp, cache = _cache(orc, bits=3, dim=128, layers=1, heads=1)
    g = orc.gauss_f32(42, 5 * 256)
    for i in range(5):
        cache.store(0, 0, g[i * 256:i * 256 + 128], g[i * 256 + 128:(i + 1) * 256], 1)
    assert cache.seq_len(0, 0) == 5
    cache.clear()
    assert cache.seq_len(0, 0) == 0
