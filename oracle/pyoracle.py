"""TEST INFRASTRUCTURE ONLY: ctypes bindings to the CPU oracle (oracle.cpp).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline leg may
import this module, and only as the checker. The product (lumen-rs_b200/)
never imports it.

Each function names the reference code it restates (paths inside
rabbitson87/lumen-rs). Tables (rotation R, QJL projection Phi, Lloyd-Max
codebook) are explicit inputs, exactly as the reference's
``TurboQuantCompressor::from_files`` (crates/lumen-core/src/compressor.rs:43-58)
takes them.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (g++, no FMA contraction)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "oracle.cpp"))
    ):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.orc_splitmix_next.restype = C.c_uint64
        L.orc_splitmix_next.argtypes = [C.POINTER(C.c_uint64)]
        L.orc_gauss_f64.argtypes = [C.c_uint64, _f64p, C.c_int64]
        L.orc_gauss_f32.argtypes = [C.c_uint64, _f32p, C.c_int64]
        L.orc_lloyd_max.restype = C.c_int
        L.orc_lloyd_max.argtypes = [C.c_int, C.c_int, _f64p, _f64p]
        L.orc_codebook_mse.restype = C.c_double
        L.orc_codebook_mse.argtypes = [C.c_int, _f64p, _f64p]
        L.orc_quantize.restype = C.c_int
        L.orc_quantize.argtypes = [_f64p, C.c_int, C.c_double]
        L.orc_rotation_from_gaussian.argtypes = [C.c_int, _f64p, _f32p]
        L.orc_rotation_generate.argtypes = [C.c_int, C.c_uint64, _f32p]
        L.orc_rotation_apply.argtypes = [_f32p, C.c_int, _f32p, _f32p]
        L.orc_rotation_apply_inverse.argtypes = [_f32p, C.c_int, _f32p, _f32p]
        L.orc_packed_words.restype = C.c_int
        L.orc_packed_words.argtypes = [C.c_int, C.c_int]
        L.orc_pack_codes.argtypes = [_u8p, C.c_int, C.c_int, _u64p]
        L.orc_unpack_codes.argtypes = [_u64p, C.c_int, C.c_int, _u8p]
        L.orc_qjl_packed_len.restype = C.c_int
        L.orc_qjl_packed_len.argtypes = [C.c_int]
        L.orc_qjl_generate.argtypes = [C.c_int, C.c_int, C.c_uint64, _f32p]
        L.orc_qjl_project_and_pack.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _u64p]
        L.orc_qjl_project_query.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _f32p]
        L.orc_qjl_correction_from_projection.restype = C.c_float
        L.orc_qjl_correction_from_projection.argtypes = [C.c_int, _f32p, _u64p, C.c_float]
        L.orc_compressor_new.restype = C.c_void_p
        L.orc_compressor_new.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, _f64p, _f64p, _f32p]
        L.orc_compressor_free.argtypes = [C.c_void_p]
        L.orc_compress_one.argtypes = [C.c_void_p, _f32p, _u64p, _u64p, C.POINTER(C.c_float),
                                       C.POINTER(C.c_float), _u8p]
        L.orc_compress.argtypes = [C.c_void_p, _f32p, C.c_int64, _u64p, _u64p, _f32p, _f32p]
        L.orc_estimate_stage1.argtypes = [C.c_void_p, _f32p, C.c_int64, _u64p, _f32p, _f32p]
        L.orc_estimate_two_stage.argtypes = [C.c_void_p, _f32p, C.c_int64, _u64p, _f32p, _u64p, _f32p, _f32p]
        L.orc_sc_new.restype = C.c_void_p
        L.orc_sc_new.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.orc_sc_free.argtypes = [C.c_void_p]
        L.orc_sc_store.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, _f32p, C.c_int64]
        L.orc_sc_seq_len.restype = C.c_int64
        L.orc_sc_seq_len.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.orc_sc_attend_keys.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, _f32p]
        L.orc_sc_attend_keys_qjl.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, _f32p]
        L.orc_sc_attend_ex.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, C.c_float, C.c_int, _f32p]
        L.orc_sc_attend_prefix.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, C.c_float, C.c_int64, _f32p]
        L.orc_rope.argtypes = [_f32p, C.c_int64, C.c_int, C.c_int, C.c_int64, C.c_double, C.c_int]
        L.orc_sc_attend_mask.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, C.c_float, _u8p, _f32p]
        L.orc_sc_attend_values.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, _f32p]
        L.orc_sc_attend.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, C.c_float, _f32p]
        L.orc_sc_clear.argtypes = [C.c_void_p]
        L.orc_sc_truncate.argtypes = [C.c_void_p, C.c_int, C.c_int64]
        L.orc_sc_memory_bytes.restype = C.c_int64
        L.orc_sc_memory_bytes.argtypes = [C.c_void_p]
        L.orc_sc_read.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                  C.c_void_p, C.c_void_p]
        L.orc_sc_load.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int64, C.c_void_p, C.c_void_p,
                                  C.c_void_p, C.c_void_p]
        L.orc_fnv1a.restype = C.c_uint64
        L.orc_fnv1a.argtypes = [C.c_uint64, C.c_char_p, C.c_int64]
        _lib = L
    return _lib


# ----------------------------------------------------------------------------
# Seeded inputs (SplitMix64 + Box-Muller), shared by tests and bench.
# ----------------------------------------------------------------------------
def gauss_f64(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float64)
    lib().orc_gauss_f64(seed & 0xFFFFFFFFFFFFFFFF, out, n)
    return out


def gauss_f32(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_gauss_f32(seed & 0xFFFFFFFFFFFFFFFF, out, n)
    return out


# ----------------------------------------------------------------------------
# Codec pieces (crates/lumen-core/src/*.rs)
# ----------------------------------------------------------------------------
def lloyd_max(bits: int, n_iter: int = 1000):
    """lloyd_max.rs:74-122 -> (boundaries[n+1] f64, centroids[n] f64)."""
    n = 1 << bits
    b = np.empty(n + 1, np.float64)
    c = np.empty(n, np.float64)
    if lib().orc_lloyd_max(bits, n_iter, b, c) != 0:
        raise ValueError(f"invalid bit width {bits}: must be 1..=8")
    return b, c


def codebook_mse(bits: int, b: np.ndarray, c: np.ndarray) -> float:
    return lib().orc_codebook_mse(bits, np.ascontiguousarray(b, np.float64), np.ascontiguousarray(c, np.float64))


def quantize(b: np.ndarray, bits: int, x: float) -> int:
    return lib().orc_quantize(np.ascontiguousarray(b, np.float64), bits, float(x))


def rotation_generate(dim: int, seed: int) -> np.ndarray:
    """Haar rotation (rotation.rs:47-87 construction) from the oracle's own stream."""
    R = np.empty(dim * dim, np.float32)
    lib().orc_rotation_generate(dim, seed, R)
    return R.reshape(dim, dim)


def rotation_apply(R: np.ndarray, x: np.ndarray) -> np.ndarray:
    d = R.shape[0]
    y = np.empty(d, np.float32)
    lib().orc_rotation_apply(np.ascontiguousarray(R, np.float32).ravel(), d, np.ascontiguousarray(x, np.float32), y)
    return y


def rotation_apply_inverse(R: np.ndarray, y: np.ndarray) -> np.ndarray:
    d = R.shape[0]
    x = np.empty(d, np.float32)
    lib().orc_rotation_apply_inverse(np.ascontiguousarray(R, np.float32).ravel(), d,
                                     np.ascontiguousarray(y, np.float32), x)
    return x


def packed_words(n: int, bits: int) -> int:
    return lib().orc_packed_words(n, bits)


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.uint8)
    out = np.empty(packed_words(len(codes), bits), np.uint64)
    lib().orc_pack_codes(codes, len(codes), bits, out)
    return out


def unpack_codes(packed: np.ndarray, n: int, bits: int) -> np.ndarray:
    out = np.empty(n, np.uint8)
    lib().orc_unpack_codes(np.ascontiguousarray(packed, np.uint64), n, bits, out)
    return out


def qjl_packed_len(m: int) -> int:
    return lib().orc_qjl_packed_len(m)


def qjl_generate(dim: int, m: int, seed: int) -> np.ndarray:
    P = np.empty(m * dim, np.float32)
    lib().orc_qjl_generate(dim, m, seed, P)
    return P.reshape(m, dim)


def qjl_project_and_pack(P: np.ndarray, res: np.ndarray) -> np.ndarray:
    m, d = P.shape
    out = np.empty(qjl_packed_len(m), np.uint64)
    lib().orc_qjl_project_and_pack(np.ascontiguousarray(P, np.float32).ravel(), m, d,
                                   np.ascontiguousarray(res, np.float32), out)
    return out


# Page-sparse decode (sdpa_page_sparse, native_attention.rs:217-329) over the
# codes: DIGEST_PAGE 64, SPARSE_SINK_PAGES 1, SPARSE_RECENT_PAGES 4,
# SPARSE_DECODE_MIN_KEYS 16384, keep = max(pages / 8, 64).
DIGEST_PAGE, SPARSE_SINK, SPARSE_RECENT, SPARSE_MIN_KEYS = 64, 1, 4, 16384


def quest_select(words, sigma, cents, bits, dim, q_rot):
    """Token mask of one (sequence, kv head) for page-sparse decode.

    words [n, W] u64 and sigma [n] f32: the stored keys; cents: the codebook;
    q_rot [G, dim]: the head group's rotated queries. The digest holds the
    min and max of the dequantized rotated keys, f32(c[code]) * sigma in f32,
    over each full 64-token page; a page's bound is the max over the group of
    sum_d max(q_d max_d, q_d min_d) (in f64 here); the first and the 4 last
    full pages are pinned; the keep largest bounds are chosen (lower page
    index first on ties) with the undigested tail. Returns (mask [n] u8,
    relative gap between the keep-th and the next unpinned bound, or inf)."""
    n = words.shape[0]
    P = n // DIGEST_PAGE
    keep = max(P // 8, 64)
    mask = np.ones(n, np.uint8)
    if n < SPARSE_MIN_KEYS or P <= keep:
        return mask, float("inf")
    codes = unpack_codes(words, dim, bits)
    kd = np.asarray(cents, np.float32)[codes] * sigma.astype(np.float32)[:, None]  # f32 products
    pages = kd[: P * DIGEST_PAGE].reshape(P, DIGEST_PAGE, dim)
    mn, mx = pages.min(1).astype(np.float64), pages.max(1).astype(np.float64)
    q = np.asarray(q_rot, np.float64)
    qp, qn = np.maximum(q, 0.0), np.minimum(q, 0.0)
    bound = (qp @ mx.T + qn @ mn.T).max(0)  # [P]
    pinned = (np.arange(P) < SPARSE_SINK) | (np.arange(P) >= P - SPARSE_RECENT)
    order = sorted(range(P), key=lambda p: (0 if pinned[p] else 1, -bound[p], p))
    chosen = order[:keep]
    free = [bound[p] for p in order[keep - 1: keep + 1] if not pinned[p]]
    gap = abs(free[0] - free[1]) / max(abs(free[0]), 1e-30) if len(free) == 2 else float("inf")
    mask[: P * DIGEST_PAGE] = 0
    for p in chosen:
        mask[p * DIGEST_PAGE:(p + 1) * DIGEST_PAGE] = 1
    return mask, gap


def unpack_codes(words: np.ndarray, dim: int, bits: int) -> np.ndarray:
    """bitpack::unpack_codes (bitpack.rs:35-52) over the last axis of u64 words."""
    cpw = 64 // bits
    j = np.arange(dim)
    w = words[..., j // cpw]
    return ((w >> ((j % cpw) * bits).astype(np.uint64)) & np.uint64((1 << bits) - 1)).astype(np.uint8)


def rope(x: np.ndarray, rot_dims: int, pos0: int, base: float = 10000.0, traditional: bool = False) -> np.ndarray:
    """RoPE of the rows of x [n, dim] at positions pos0.. (orc_rope)."""
    y = np.ascontiguousarray(x, np.float32).copy()
    n, dim = y.shape
    lib().orc_rope(y.ravel(), n, dim, rot_dims, pos0, base, 1 if traditional else 0)
    return y


def qjl_estimate_correction(P: np.ndarray, q: np.ndarray, packed: np.ndarray, rnorm: float) -> float:
    m, d = P.shape
    pq = np.empty(m, np.float32)
    lib().orc_qjl_project_query(np.ascontiguousarray(P, np.float32).ravel(), m, d,
                                np.ascontiguousarray(q, np.float32), pq)
    return lib().orc_qjl_correction_from_projection(m, pq, np.ascontiguousarray(packed, np.uint64), rnorm)


class Tables:
    """The explicit tables one compressor runs on (R, codebook, Phi)."""

    def __init__(self, dim: int, bits: int, m: int, R: np.ndarray, bounds: np.ndarray,
                 cents: np.ndarray, proj: np.ndarray):
        self.dim, self.bits, self.m = dim, bits, m
        self.R = np.ascontiguousarray(R, np.float32).reshape(dim, dim)
        self.bounds = np.ascontiguousarray(bounds, np.float64)
        self.cents = np.ascontiguousarray(cents, np.float64)
        self.proj = np.ascontiguousarray(proj, np.float32).reshape(m, dim)

    @classmethod
    def generate(cls, dim: int, bits: int, m: int = 64, seed: int = 42, n_iter: int = 1000):
        """compressor.rs:20-32 layout: R from `seed`, Phi from `seed + 1`."""
        b, c = lloyd_max(bits, n_iter)
        return cls(dim, bits, m, rotation_generate(dim, seed), b, c, qjl_generate(dim, m, seed + 1))


class Compressor:
    """TurboQuantCompressor (compressor.rs:11-184) over explicit tables."""

    def __init__(self, t: Tables):
        self.t = t
        self.dim, self.bits, self.m = t.dim, t.bits, t.m
        self.words = packed_words(t.dim, t.bits)
        self.qwords = qjl_packed_len(t.m)
        self._h = lib().orc_compressor_new(t.dim, t.bits, t.m, t.R.ravel(), t.bounds, t.cents, t.proj.ravel())

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.orc_compressor_free(h)
            self._h = None

    def compress_one(self, x: np.ndarray):
        s1 = np.empty(self.words, np.uint64)
        s2 = np.empty(self.qwords, np.uint64)
        rn, sc = C.c_float(), C.c_float()
        codes = np.empty(self.dim, np.uint8)
        lib().orc_compress_one(self._h, np.ascontiguousarray(x, np.float32), s1, s2, C.byref(rn), C.byref(sc), codes)
        return dict(stage1=s1, stage2=s2, residual_norm=np.float32(rn.value), scale=np.float32(sc.value), codes=codes)

    def compress(self, X: np.ndarray):
        X = np.ascontiguousarray(X, np.float32).reshape(-1, self.dim)
        n = X.shape[0]
        s1 = np.empty((n, self.words), np.uint64)
        s2 = np.empty((n, self.qwords), np.uint64)
        rn = np.empty(n, np.float32)
        sc = np.empty(n, np.float32)
        lib().orc_compress(self._h, X.ravel(), n, s1.ravel(), s2.ravel(), rn, sc)
        return s1, s2, rn, sc

    def estimate_stage1(self, q, s1, sc):
        n = s1.shape[0]
        out = np.empty(n, np.float32)
        lib().orc_estimate_stage1(self._h, np.ascontiguousarray(q, np.float32), n,
                                  np.ascontiguousarray(s1, np.uint64).ravel(), np.ascontiguousarray(sc, np.float32), out)
        return out

    def estimate(self, q, s1, sc, s2, rn):
        n = s1.shape[0]
        out = np.empty(n, np.float32)
        lib().orc_estimate_two_stage(self._h, np.ascontiguousarray(q, np.float32), n,
                                     np.ascontiguousarray(s1, np.uint64).ravel(), np.ascontiguousarray(sc, np.float32),
                                     np.ascontiguousarray(s2, np.uint64).ravel(), np.ascontiguousarray(rn, np.float32),
                                     out)
        return out


class SimpleCache:
    """turboquant-cache SimpleCache (simple.rs:13-185); K and V compressors may differ."""

    def __init__(self, kc: Compressor, vc: Compressor, n_layers: int, n_heads: int, dim: int):
        self.kc, self.vc = kc, vc
        self.n_layers, self.n_heads, self.dim = n_layers, n_heads, dim
        self._h = lib().orc_sc_new(kc._h, vc._h, n_layers, n_heads, dim)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.orc_sc_free(h)
            self._h = None

    def store(self, layer, head, keys, values, n_tokens):
        lib().orc_sc_store(self._h, layer, head, np.ascontiguousarray(keys, np.float32).ravel(),
                           np.ascontiguousarray(values, np.float32).ravel(), n_tokens)

    def seq_len(self, layer, head):
        return lib().orc_sc_seq_len(self._h, layer, head)

    def attend_keys(self, layer, head, q):
        out = np.empty(max(self.seq_len(layer, head), 1), np.float32)
        lib().orc_sc_attend_keys(self._h, layer, head, np.ascontiguousarray(q, np.float32), out)
        return out[: self.seq_len(layer, head)]

    def attend_keys_qjl(self, layer, head, q):
        """Two-stage scores: estimate_inner_products (compressor.rs:122-159)."""
        out = np.empty(max(self.seq_len(layer, head), 1), np.float32)
        lib().orc_sc_attend_keys_qjl(self._h, layer, head, np.ascontiguousarray(q, np.float32), out)
        return out[: self.seq_len(layer, head)]

    def attend_values(self, layer, head, w):
        out = np.empty(self.dim, np.float32)
        lib().orc_sc_attend_values(self._h, layer, head, np.ascontiguousarray(w, np.float32), out)
        return out

    def attend_prefix(self, layer, head, q, scale, n_keys):
        """Attention over the first n_keys stored tokens (causal prefill)."""
        out = np.empty(self.dim, np.float32)
        lib().orc_sc_attend_prefix(self._h, layer, head, np.ascontiguousarray(q, np.float32), float(scale),
                                   int(n_keys), out)
        return out

    def attend_mask(self, layer, head, q, scale, mask):
        """Attention over the stored tokens with mask[t] != 0."""
        out = np.empty(self.dim, np.float32)
        lib().orc_sc_attend_mask(self._h, layer, head, np.ascontiguousarray(q, np.float32), float(scale),
                                 np.ascontiguousarray(mask, np.uint8), out)
        return out

    def attend(self, layer, head, q, scale=1.0, qjl=False):
        """softmax(scale * scores) then attend_values; qjl: two-stage scores."""
        out = np.empty(self.dim, np.float32)
        lib().orc_sc_attend_ex(self._h, layer, head, np.ascontiguousarray(q, np.float32), float(scale),
                               1 if qjl else 0, out)
        return out

    def clear(self):
        lib().orc_sc_clear(self._h)

    def truncate(self, layer, n_keep):
        lib().orc_sc_truncate(self._h, layer, n_keep)

    def memory_bytes(self):
        return lib().orc_sc_memory_bytes(self._h)

    def load(self, layer, head, side, s1, scale, s2=None, rnorm=None):
        """Append already-compressed vectors (stage1 words [n, W], scale [n])."""
        s1 = np.ascontiguousarray(s1, np.uint64)
        scale = np.ascontiguousarray(scale, np.float32)
        s2 = None if s2 is None else np.ascontiguousarray(s2, np.uint64)
        rnorm = None if rnorm is None else np.ascontiguousarray(rnorm, np.float32)
        lib().orc_sc_load(self._h, layer, head, side, len(scale), s1.ctypes.data,
                          None if s2 is None else s2.ctypes.data, None if rnorm is None else rnorm.ctypes.data,
                          scale.ctypes.data)
        self._keep = getattr(self, "_keep", []) + [s1, scale, s2, rnorm]

    def read(self, layer, head, side):
        """(stage1 [n,W], stage2 [n,Q], residual_norm [n], scale [n]) of K (side 0) or V (side 1)."""
        c = self.vc if side else self.kc
        n = self.seq_len(layer, head)
        s1 = np.empty((n, c.words), np.uint64)
        s2 = np.empty((n, c.qwords), np.uint64)
        rn = np.empty(n, np.float32)
        sc = np.empty(n, np.float32)
        lib().orc_sc_read(self._h, layer, head, side, s1.ctypes.data, s2.ctypes.data, rn.ctypes.data, sc.ctypes.data)
        return s1, s2, rn, sc


def fnv1a(h: int, data: bytes) -> int:
    return lib().orc_fnv1a(h, data, len(data))
