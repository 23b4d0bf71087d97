"""Golden fixtures (tests/golden/, written by tests/golden/make_golden.py).

CPU:
- the oracle reproduces every fixture bit for bit;
- the product codec reads the table files back exactly;
- the product generator (lc_codec_new) produces the same tables.

GPU:
- the device compressor reproduces the frozen compressed vectors bit for
  bit: stage-1 words, QJL words, residual norm and scale, for 2, 3 and 4
  bits;
- decode attention matches the frozen SimpleCache output to the decode
  tolerance.
"""
import importlib
import os
import sys

import numpy as np
import pytest

import helpers

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
ROT = os.path.join(GOLD, "tq_d128_s42.tqrm")
QJL = os.path.join(GOLD, "tq_d128_m64_s43.tqjl")


def _cb(bits):
    return os.path.join(GOLD, f"tq_b{bits}.tqcb")


def _make():
    sys.path.insert(0, GOLD)
    import make_golden

    return make_golden


def test_oracle_reproduces_golden(orc, tmp_path):
    mg = _make()
    f = mg.fixtures(orc)
    mg.write_tqrm(tmp_path / "r", f["R"])
    mg.write_tqjl(tmp_path / "p", f["P"])
    assert (tmp_path / "r").read_bytes() == open(ROT, "rb").read()
    assert (tmp_path / "p").read_bytes() == open(QJL, "rb").read()
    for b in (2, 3, 4):
        mg.write_tqcb(tmp_path / f"c{b}", b, f[f"bounds{b}"], f[f"cents{b}"])
        assert (tmp_path / f"c{b}").read_bytes() == open(_cb(b), "rb").read()
    comp = np.load(os.path.join(GOLD, "compress_d128.npz"))
    for k, v in f["compress"].items():
        np.testing.assert_array_equal(comp[k], v, err_msg=k)
    att = np.load(os.path.join(GOLD, "attend_d128_b4.npz"))
    np.testing.assert_array_equal(att["out"], f["attend"]["out"])


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_product_codec_reads_golden_files(lc, bits):
    c = lc.TurboQuantCompressor.from_files(_cb(bits), ROT, QJL)
    R, b, cents, P = c.tables()
    raw = open(ROT, "rb").read()
    np.testing.assert_array_equal(R.ravel(), np.frombuffer(raw[8:], "<f4"))
    raw = open(QJL, "rb").read()
    np.testing.assert_array_equal(P.ravel(), np.frombuffer(raw[12:], "<f4"))
    raw = open(_cb(bits), "rb").read()
    n = 1 << bits
    np.testing.assert_array_equal(b, np.frombuffer(raw[12:12 + 8 * (n + 1)], "<f8"))
    np.testing.assert_array_equal(cents, np.frombuffer(raw[12 + 8 * (n + 1):], "<f8"))


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_product_generator_matches_golden(lc, bits):
    gen = lc.TurboQuantCompressor(lc.TurboQuantConfig(bits, 64, 42, 1000, 128))
    ref = lc.TurboQuantCompressor.from_files(_cb(bits), ROT, QJL)
    for a, b in zip(gen.tables(), ref.tables()):
        np.testing.assert_array_equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [2, 3, 4])
def test_gpu_compress_matches_golden(lc, gpu, bits):
    codec = lc.TurboQuantCompressor.from_files(_cb(bits), ROT, QJL)
    cache = lc.CudaKvCache(1, 1, 128, codec, max_seqs=1, max_pages=4, max_pages_per_seq=2,
                           store_flags=lc.LC_STORE_K_QJL | lc.LC_STORE_V_QJL)
    comp = np.load(os.path.join(GOLD, "compress_d128.npz"))
    X = comp["x"]
    cache.store(0, 0, 0, X, X, len(X))
    f = cache.fetch(0, 0)
    for side in ("k", "v"):
        np.testing.assert_array_equal(f[f"{side}_words"][0], comp[f"stage1_b{bits}"])
        np.testing.assert_array_equal(f[f"{side}_qjl"][0], comp[f"stage2_b{bits}"])
        np.testing.assert_array_equal(f[f"{side}_rnorm"][0].view(np.uint32), comp[f"rnorm_b{bits}"].view(np.uint32))
        np.testing.assert_array_equal(f[f"{side}_sigma"][0].view(np.uint32), comp[f"scale_b{bits}"].view(np.uint32))
    cache.close()


@pytest.mark.gpu
def test_gpu_attend_matches_golden(lc, orc, gpu):
    att = np.load(os.path.join(GOLD, "attend_d128_b4.npz"))
    ks, vs, _ = (int(x) for x in att["kv_seeds"])
    n = int(att["n_tokens"])
    codec = lc.TurboQuantCompressor.from_files(_cb(4), ROT, QJL)
    cache = lc.CudaKvCache(1, 8, 128, codec, max_seqs=1, max_pages=4, max_pages_per_seq=3)
    K = helpers.kv(orc, ks, 1, 8, n, 128)
    V = helpers.kv(orc, vs, 1, 8, n, 128)
    cache.append(0, [0], K, V)
    got = cache.decode_attn(0, [0], att["q"][None], 32, 1.0 / np.sqrt(128))
    ok, msg = helpers.attn_close(got[0], att["out"])
    assert ok, msg
    cache.close()
