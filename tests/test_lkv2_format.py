"""CPU: the LKV2 snapshot format (crates/lumen-mlx/src/kv_disk.rs).

The oracle restatement (oracle/lkv2.py) writes the reference's own test
snapshot (sample_manifest and records of kv_disk.rs:2078-2125, 2157-2173);
the library's host-only reader (lc_lkv2_info, no device) must accept it and
reject every kind of corruption the reference's reader rejects
(kv_disk.rs:175-190 bad magic, :189-248 lengths, :414-446 CRCs and trailing
bytes).
"""
import struct
import zlib

import numpy as np
import pytest

import lkv2


def sample_manifest():
    """kv_disk.rs:2078-2102."""
    return {
        "model_fingerprint": "fp-abc123", "created_at_unix": 1_700_000_000, "position": 42,
        "prefix_tokens": [1, 2, 3, 4, 5], "last_token": 7, "is_deep": True,
        "layers": [
            {"kind": "Full", "offset": 42, "base_offset": 0, "arrays": [0, 1]},
            {"kind": "FullTurboquant", "offset": 42, "base_offset": 0, "arrays": [2, 3], "max_size": 1024,
             "keep": 0, "idx": 42, "bits": 3, "qjl_m": 64},
        ],
    }


def sample_records():
    """kv_disk.rs:2104-2125, 2160-2165."""
    def f32(shape, fill):
        return lkv2.record(lkv2.F32, (fill + np.arange(int(np.prod(shape)), dtype=np.float32)).reshape(shape))

    def u8(shape):
        return lkv2.record(lkv2.U8, (np.arange(int(np.prod(shape))) % 251).astype(np.uint8).reshape(shape))

    return [f32([1, 2, 4, 8], 0.0), f32([1, 2, 4, 8], 100.0), u8([1, 4, 16, 128]), f32([1, 4, 16, 1], 3.5)]


def test_crc_and_json_form():
    assert zlib.crc32(b"123456789") == 0xCBF43926  # CRC-32/IEEE check value
    js = lkv2.manifest_json(sample_manifest()).decode()
    # serde_json compact form: declaration order, absent Options left out
    assert js.startswith('{"model_fingerprint":"fp-abc123","created_at_unix":1700000000,"position":42,'
                         '"prefix_tokens":[1,2,3,4,5],"last_token":7,"is_deep":true,"layers":[')
    assert '{"kind":"Full","offset":42,"base_offset":0,"arrays":[0,1]}' in js
    assert '"arrays":[2,3],"max_size":1024,"keep":0,"idx":42,"bits":3,"qjl_m":64}' in js


def test_oracle_roundtrip_is_byte_faithful():
    b = lkv2.encode(sample_manifest(), sample_records())
    m, recs, js = lkv2.decode(b)
    assert m == sample_manifest()
    assert [(r.dtype, r.shape, r.data) for r in recs] == [(r.dtype, r.shape, r.data) for r in sample_records()]
    assert lkv2.encode(m, recs) == b


def test_library_reads_reference_sample(lc, tmp_path):
    p = tmp_path / "s.lkv"
    lkv2.write(p, sample_manifest(), sample_records())
    assert lc.lkv2_info(p) == {"layers": 2, "records": 4, "position": 42}


def _corrupt(b: bytes, at: int, delta: int = 1) -> bytes:
    x = bytearray(b)
    x[at] = (x[at] + delta) & 0xFF
    return bytes(x)


def test_library_rejects_corruption(lc, tmp_path):
    good = lkv2.encode(sample_manifest(), sample_records())
    (jl,) = struct.unpack_from("<I", good, 8)
    rec0 = 12 + jl + 8  # first record header
    cases = {
        "magic": (b"XXXX" + good[4:], lc.LC_ERR_MAGIC),
        "version": (good[:4] + struct.pack("<I", 3) + good[8:], lc.LC_ERR_MAGIC),
        "manifest byte": (_corrupt(good, 12 + 5), lc.LC_ERR_IO),
        "manifest CRC": (_corrupt(good, 12 + jl), lc.LC_ERR_IO),
        "manifest length": (good[:8] + struct.pack("<I", 1 << 30) + good[12:], lc.LC_ERR_IO),
        "dtype tag": (good[:rec0] + bytes([99]) + good[rec0 + 1:], lc.LC_ERR_IO),
        "payload length": (good[:rec0 + 5 + 16] + struct.pack("<Q", 1 << 40) + good[rec0 + 5 + 24:], lc.LC_ERR_IO),
        "payload byte": (_corrupt(good, rec0 + 5 + 16 + 8 + 3), lc.LC_ERR_IO),
        "record CRC": (_corrupt(good, len(good) - 1), lc.LC_ERR_IO),
        "trailing byte": (good + b"\0", lc.LC_ERR_IO),
        "truncated": (good[:-3], lc.LC_ERR_IO),
        "record count": (good[:12 + jl + 4] + struct.pack("<I", 5) + good[12 + jl + 8:], lc.LC_ERR_IO),
    }
    for name, (b, code) in cases.items():
        p = tmp_path / (name.replace(" ", "_") + ".lkv")
        p.write_bytes(b)
        with pytest.raises(lc.LumenError) as e:
            lc.lkv2_info(p)
        assert e.value.code == code, name
        with pytest.raises(lkv2.LkvError):
            lkv2.read(p)
    with pytest.raises(lc.LumenError) as e:
        lc.lkv2_info(tmp_path / "missing.lkv")
    assert e.value.code == lc.LC_ERR_IO
