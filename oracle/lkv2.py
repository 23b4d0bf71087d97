"""Test infrastructure: an independent restatement of the LKV2 snapshot
format of crates/lumen-mlx/src/kv_disk.rs, used only as the checker of the
library's lc_save_lkv2 / lc_load_lkv2 / lc_lkv2_info.

  layout      kv_disk.rs:285-323   "LKV2" | version u32 | JSON length u32 |
                                   JSON | CRC-32(JSON) | count u32 | records
  record      kv_disk.rs:155-168   dtype u8 | ndim u32 | shape i32[ndim] |
                                   len u64 | payload | CRC-32(all of it)
  checks      kv_disk.rs:189-248, 414-446 (ndim <= 8, len == shape x dtype,
                                   CRCs, no trailing bytes)
  manifest    kv_disk.rs:214-283   serde_json's compact output: fields in
                                   declaration order, Option fields with
                                   skip_serializing_if left out when None
  TQ layer    kv_disk.rs:2000-2024 arrays [keys_codes, keys_sigma,
                                   values_codes, values_sigma, keys_signs?,
                                   keys_residual_norm?]

CRC-32 is zlib's (the same CRC-32/IEEE as crc32fast).
"""
from __future__ import annotations

import json
import struct
import zlib
from dataclasses import dataclass

import numpy as np

MAGIC = b"LKV2"
VERSION = 2

# DtypeTag (kv_disk.rs:85-100): tag byte -> (numpy dtype, stored bytes)
DTYPES = {
    0: ("bool", 1), 1: ("uint8", 1), 2: ("<u2", 2), 3: ("<u4", 4), 4: ("<u8", 8), 5: ("int8", 1),
    6: ("<i2", 2), 7: ("<i4", 4), 8: ("<i8", 8), 9: ("<f2", 2), 10: ("<f4", 4), 11: ("<f8", 8),
    12: ("<u2", 2),  # bf16: raw 16-bit patterns
}
U8, F32, BF16 = 1, 10, 12
BF16_ONE, BF16_MINUS_ONE = 0x3F80, 0xBF80


class LkvError(Exception):
    pass


@dataclass
class Record:
    dtype: int
    shape: list
    data: bytes

    def array(self) -> np.ndarray:
        return np.frombuffer(self.data, DTYPES[self.dtype][0]).reshape(self.shape)


def record(dtype: int, arr: np.ndarray) -> Record:
    a = np.ascontiguousarray(arr, DTYPES[dtype][0])
    return Record(dtype, [int(d) for d in arr.shape], a.tobytes())


# LayerMeta / KvManifest fields in declaration order; the ones marked True
# are Option<...> with skip_serializing_if = "Option::is_none".
LAYER_FIELDS = [("kind", False), ("offset", False), ("base_offset", False), ("arrays", False),
                ("lengths_id", True), ("left_padding_id", True), ("max_size", True), ("keep", True),
                ("idx", True), ("bits", True), ("qjl_m", True), ("group_size", True)]
MANIFEST_FIELDS = [("model_fingerprint", False), ("created_at_unix", False), ("position", False),
                   ("prefix_tokens", False), ("last_token", True), ("is_deep", False), ("layers", False)]


def _ordered(d: dict, fields, extra=()) -> dict:
    out = {}
    for k, opt in fields:
        v = d.get(k)
        if opt and v is None:
            continue
        out[k] = v
    for k in extra:  # fields the reference's reader ignores (v_bits)
        if d.get(k) is not None:
            out[k] = d[k]
    return out


def manifest_json(m: dict) -> bytes:
    layers = [_ordered(L, LAYER_FIELDS, extra=("v_bits",)) for L in m["layers"]]
    top = _ordered(dict(m, layers=layers), MANIFEST_FIELDS)
    return json.dumps(top, separators=(",", ":"), ensure_ascii=False).encode()


def encode(m: dict, records: list) -> bytes:
    js = manifest_json(m)
    out = bytearray(MAGIC + struct.pack("<II", VERSION, len(js)) + js + struct.pack("<I", zlib.crc32(js)))
    out += struct.pack("<I", len(records))
    for r in records:
        n = int(np.prod(r.shape)) if r.shape else 0
        if len(r.data) != n * DTYPES[r.dtype][1]:
            raise LkvError("record length != shape x dtype")
        body = bytes([r.dtype]) + struct.pack("<I", len(r.shape)) + b"".join(struct.pack("<i", d) for d in r.shape)
        body += struct.pack("<Q", len(r.data)) + r.data
        out += body + struct.pack("<I", zlib.crc32(body))
    return bytes(out)


def write(path, m: dict, records: list) -> None:
    with open(path, "wb") as f:
        f.write(encode(m, records))


def decode(b: bytes):
    """(manifest dict, records, manifest JSON bytes); LkvError if malformed."""
    try:
        return _decode(b)
    except (struct.error, IndexError, ValueError) as e:  # ran off the end / bad JSON
        raise LkvError(f"truncated or malformed: {e}") from e


def _decode(b: bytes):
    if b[:4] != MAGIC:
        raise LkvError("bad magic")
    ver, jl = struct.unpack_from("<II", b, 4)
    if ver != VERSION:
        raise LkvError("unsupported version")
    p = 12
    js = b[p:p + jl]
    p += jl
    if len(js) != jl or struct.unpack_from("<I", b, p)[0] != zlib.crc32(js):
        raise LkvError("manifest CRC mismatch")
    p += 4
    m = json.loads(js)
    (n,) = struct.unpack_from("<I", b, p)
    p += 4
    recs = []
    for _ in range(n):
        q = p
        dt = b[p]
        (nd,) = struct.unpack_from("<I", b, p + 1)
        if nd > 8 or dt not in DTYPES:
            raise LkvError("bad record header")
        shape = list(struct.unpack_from("<%di" % nd, b, p + 5))
        (ln,) = struct.unpack_from("<Q", b, p + 5 + 4 * nd)
        want = (int(np.prod(shape)) if shape else 0) * DTYPES[dt][1]
        if ln != want:
            raise LkvError("record length disagrees with shape and dtype")
        p += 5 + 4 * nd + 8
        data = b[p:p + ln]
        p += ln
        if len(data) != ln or struct.unpack_from("<I", b, p)[0] != zlib.crc32(b[q:p]):
            raise LkvError("record CRC mismatch")
        p += 4
        recs.append(Record(dt, shape, data))
    if p != len(b):
        raise LkvError("trailing bytes")
    return m, recs, js


def read(path):
    with open(path, "rb") as f:
        return decode(f.read())


def unpack_codes(words: np.ndarray, dim: int, bits: int) -> np.ndarray:
    """bitpack::unpack_codes (bitpack.rs:35-52) over the last axis of u64 words."""
    cpw = 64 // bits
    j = np.arange(dim)
    w = words[..., j // cpw]
    return ((w >> ((j % cpw) * bits).astype(np.uint64)) & np.uint64((1 << bits) - 1)).astype(np.uint8)


def signs_pm1(words: np.ndarray, m: int) -> np.ndarray:
    """QJL sign words -> bf16 bit patterns of +1 (bit set) / -1."""
    i = np.arange(m)
    bit = (words[..., i // 64] >> (i % 64).astype(np.uint64)) & np.uint64(1)
    return np.where(bit == 1, BF16_ONE, BF16_MINUS_ONE).astype(np.uint16)
