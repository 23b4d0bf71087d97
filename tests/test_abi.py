"""CPU: the C-ABI library loads and exports every declared symbol, and its
host-side codec setup (no GPU needed) agrees with the oracle."""
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "lumen_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(lc_[a-z_0-9]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(lc):
    L = lc.lib()
    declared = _declared_symbols()
    assert len(declared) >= 30
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    assert sorted(lc.ABI_SYMBOLS) == declared


def test_version(lc):
    assert "sm_100a" in lc.version()


def test_packed_words_matches_bitpack(lc, orc):  # bitpack.rs:11-14
    for n in (1, 64, 128, 256, 512):
        for bits in range(1, 9):
            assert lc.packed_words(n, bits) == orc.packed_words(n, bits)


@pytest.mark.parametrize("dim,bits,m,seed", [(128, 4, 64, 42), (64, 3, 32, 7), (256, 2, 128, 11)])
def test_codec_new_matches_oracle_tables(lc, orc, dim, bits, m, seed):
    """TurboQuantCompressor::new layout (compressor.rs:20-32): R from seed, Phi from seed+1."""
    comp = lc.TurboQuantCompressor(lc.TurboQuantConfig(bits, m, seed, 1000, dim))
    R, b, c, P = comp.tables()
    t = orc.Tables.generate(dim, bits, m, seed)
    np.testing.assert_array_equal(R, t.R)
    np.testing.assert_array_equal(b, t.bounds)
    np.testing.assert_array_equal(c, t.cents)
    np.testing.assert_array_equal(P, t.proj)


def test_codec_file_roundtrip(lc, tmp_path):  # rotation.rs:239-248, lloyd_max.rs:295-308, qjl.rs:391-401
    comp = lc.TurboQuantCompressor(lc.TurboQuantConfig(3, 64, 42, 1000, 64))
    paths = [str(tmp_path / n) for n in ("cb.bin", "rot.bin", "qjl.bin")]
    comp.save(*paths)
    back = lc.TurboQuantCompressor.from_files(*paths)
    for x, y in zip(comp.tables(), back.tables()):
        np.testing.assert_array_equal(x, y)
    assert (back.head_dim, back.bits, back.qjl_m) == (64, 3, 64)


def test_codec_file_layout(lc, tmp_path):
    """binfile.rs: 4-byte magic, u32 LE header fields, LE arrays."""
    comp = lc.TurboQuantCompressor(lc.TurboQuantConfig(2, 32, 1, 1000, 32))
    paths = [str(tmp_path / n) for n in ("cb.bin", "rot.bin", "qjl.bin")]
    comp.save(*paths)
    R, b, c, P = comp.tables()
    cb = open(paths[0], "rb").read()
    assert cb[:4] == b"TQCB" and np.frombuffer(cb[4:12], "<u4").tolist() == [2, 4]
    np.testing.assert_array_equal(np.frombuffer(cb[12:12 + 40], "<f8"), b)
    np.testing.assert_array_equal(np.frombuffer(cb[52:84], "<f8"), c)
    rot = open(paths[1], "rb").read()
    assert rot[:4] == b"TQRM" and np.frombuffer(rot[4:8], "<u4")[0] == 32 and len(rot) == 8 + 32 * 32 * 4
    qj = open(paths[2], "rb").read()
    assert qj[:4] == b"TQJL" and np.frombuffer(qj[4:12], "<u4").tolist() == [32, 32]


def test_codec_errors(lc, tmp_path):
    with pytest.raises(lc.LumenError) as e:
        lc.TurboQuantCompressor(lc.TurboQuantConfig(9, 64, 42, 10, 128))
    assert e.value.code == -2  # LC_ERR_BITS (lloyd_max.rs:75-77)
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"XXXX" + b"\0" * 64)
    with pytest.raises(lc.LumenError) as e:
        lc.TurboQuantCompressor.from_files(str(bad), str(bad), str(bad))
    assert e.value.code == -8  # LC_ERR_MAGIC (BadMagic)
    with pytest.raises(lc.LumenError) as e:
        lc.TurboQuantCompressor.from_files(str(tmp_path / "none"), str(bad), str(bad))
    assert e.value.code == -7  # LC_ERR_IO
    trunc = tmp_path / "trunc.bin"
    trunc.write_bytes(b"TQCB" + np.array([3, 8], "<u4").tobytes() + b"\0" * 10)
    with pytest.raises(lc.LumenError) as e:
        lc.TurboQuantCompressor.from_files(str(trunc), str(bad), str(bad))
    assert e.value.code == -7


def test_from_tables_roundtrip(lc, orc):
    t = orc.Tables.generate(128, 4, 64, 5)
    comp = lc.TurboQuantCompressor.from_tables(t.R, t.bounds, t.cents, t.proj)
    R, b, c, P = comp.tables()
    np.testing.assert_array_equal(R, t.R)
    np.testing.assert_array_equal(P, t.proj)
    assert comp.bits == 4 and comp.qjl_m == 64
