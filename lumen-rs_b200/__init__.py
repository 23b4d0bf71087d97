"""lumen-rs_b200: the TurboQuant compressed-KV path of lumen-rs, B200-native.

Host-side mirror of the reference's API over the C ABI in
include/lumen_cuda.h (liblumen_cuda.so, built by build.py). Names, argument
meaning and error behaviour follow rabbitson87/lumen-rs:

  TurboQuantConfig / TurboQuantCompressor   crates/lumen-core/src/{config,compressor}.rs
  KVCache (trait) / SimpleCache             crates/turboquant-cache/src/{traits,simple}.rs
  NativeRotatingKvCacheTurboQuant           crates/lumen-mlx/src/native_cache.rs:1517-1862
  CudaKvCache                               the multi-sequence device cache the above sit on

There is no CPU fallback: every operation runs the sm_100a kernels through
the C ABI, and importing this package fails if the library is missing.
Array arguments are numpy arrays (host memory) or torch tensors (host or
device); the library stages host buffers itself.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

__all__ = [
    "LumenError", "lib", "TurboQuantConfig", "TurboQuantCompressor", "CudaKvCache", "KVCache", "SimpleCache",
    "NativeRotatingKvCacheTurboQuant", "RawRing", "SplitGroup", "packed_words", "LC_F32", "LC_BF16", "LC_F16",
    "LC_Q_ROTATED", "LC_OUT_ROTATED", "LC_STORE_K_QJL", "LC_STORE_V_QJL",
]

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblumen_cuda.so")

LC_OK, LC_ERR_INVALID, LC_ERR_BITS, LC_ERR_REFUSED, LC_ERR_CUDA = 0, -1, -2, -3, -4
LC_ERR_TIMEOUT, LC_ERR_NOMEM, LC_ERR_IO, LC_ERR_MAGIC, LC_ERR_STATE = -5, -6, -7, -8, -9
LC_F32, LC_BF16, LC_F16 = 0, 1, 2
LC_STORE_K_QJL, LC_STORE_V_QJL, LC_STORE_DIGEST, LC_STORE_V_UNROTATED = 1, 2, 4, 8
LC_FETCH_VIEW, LC_FETCH_BACKING = 0, 1
LC_Q_ROTATED, LC_OUT_ROTATED, LC_QJL_SCORES, LC_SPARSE_PAGES = 1, 2, 4, 8
LC_GROUP_ID_BYTES, LC_GROUP_NCCL = 128, 1
# cudaStreamLegacy: the legacy default stream (torch's default stream, handle 0).
# A NULL stream in the C ABI means the library's own stream instead.
CUDA_STREAM_LEGACY = 0x1

# Every symbol include/lumen_cuda.h declares.
ABI_SYMBOLS = [
    "lc_last_error", "lc_codec_new", "lc_codec_from_files", "lc_codec_from_tables", "lc_codec_save",
    "lc_codec_tables", "lc_codec_shape", "lc_codec_free", "lc_packed_words", "lc_cache_create",
    "lc_cache_destroy", "lc_store", "lc_attend_keys", "lc_attend_keys_qjl", "lc_attend_values", "lc_seq_len", "lc_clear",
    "lc_truncate", "lc_append", "lc_append_rope", "lc_truncate_to", "lc_fork", "lc_release", "lc_ring_state", "lc_fetch",
    "lc_decode_attn", "lc_decode_step", "lc_decode_step_layers", "lc_prefill_attn", "lc_decode_attn_noalloc", "lc_decode_attn_partials", "lc_merge_partials", "lc_cache_info", "lc_cache_timing",
    "lc_group_id", "lc_group_create", "lc_group_info", "lc_group_status", "lc_group_destroy", "lc_decode_attn_split",
    "lc_ring_create",
    "lc_ring_update", "lc_ring_truncate_to", "lc_ring_counters", "lc_ring_read", "lc_ring_clear",
    "lc_ring_deep_clone", "lc_ring_destroy", "lc_version", "lc_save_lkv2", "lc_load_lkv2", "lc_lkv2_info",
]


class LumenError(RuntimeError):
    """A failed C-ABI call: `code` is the LC_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class lc_cache_config(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int32), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("max_seqs", C.c_int32),
        ("max_pages", C.c_int64), ("max_pages_per_seq", C.c_int64), ("store_flags", C.c_uint32),
        ("device", C.c_int32), ("step_prealloc", C.c_int32), ("reserved", C.c_int32),
        ("layer_max_size", C.POINTER(C.c_int64)), ("layer_keep", C.POINTER(C.c_int64)),
    ]


class lc_fetch_out(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in
                ("k_words", "k_sigma", "v_words", "v_sigma", "k_qjl", "k_rnorm", "v_qjl", "v_rnorm")]


_lib = None


def lib():
    """Load liblumen_cuda.so; raises if it is missing (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python lumen-rs_b200/build.py`")
    L = C.CDLL(LIB_PATH)
    vp, i32, i64, u32, u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint32, C.c_uint64
    pp = C.POINTER(C.c_void_p)
    sig = {
        "lc_last_error": (C.c_char_p, []),
        "lc_version": (C.c_char_p, []),
        "lc_packed_words": (u64, [u64, u32]),
        "lc_codec_new": (C.c_int, [u32, u64, u64, u64, u64, pp]),
        "lc_codec_from_files": (C.c_int, [C.c_char_p, C.c_char_p, C.c_char_p, pp]),
        "lc_codec_from_tables": (C.c_int, [u64, u32, u64, vp, vp, vp, vp, pp]),
        "lc_codec_save": (C.c_int, [vp, C.c_char_p, C.c_char_p, C.c_char_p]),
        "lc_codec_tables": (C.c_int, [vp, vp, vp, vp, vp]),
        "lc_codec_shape": (C.c_int, [vp, C.POINTER(u64), C.POINTER(u32), C.POINTER(u64)]),
        "lc_codec_free": (None, [vp]),
        "lc_cache_create": (C.c_int, [C.POINTER(lc_cache_config), vp, vp, pp]),
        "lc_cache_destroy": (None, [vp]),
        "lc_cache_info": (C.c_int, [vp, C.POINTER(i32), pp, C.POINTER(u64)]),
        "lc_cache_timing": (C.c_int, [vp, i32, C.POINTER(C.c_double), C.POINTER(u64), C.POINTER(C.c_double),
                                      C.POINTER(u64), C.POINTER(C.c_double)]),
        "lc_store": (C.c_int, [vp, i32, i32, i32, vp, vp, i64]),
        "lc_attend_keys": (C.c_int, [vp, i32, i32, i32, vp, vp, i64]),
        "lc_attend_keys_qjl": (C.c_int, [vp, i32, i32, i32, vp, vp, i64]),
        "lc_attend_values": (C.c_int, [vp, i32, i32, i32, vp, i64, vp]),
        "lc_seq_len": (i64, [vp, i32, i32, i32]),
        "lc_clear": (C.c_int, [vp]),
        "lc_truncate": (C.c_int, [vp, i32, i32, i64]),
        "lc_append": (C.c_int, [vp, i32, i32, vp, vp, vp, i32, i64, vp]),
        "lc_append_rope": (C.c_int, [vp, i32, i32, vp, vp, vp, i32, i64, i32, C.c_double, i32, vp]),
        "lc_truncate_to": (C.c_int, [vp, i32, i32, i64]),
        "lc_fork": (C.c_int, [vp, i32, i32, i64]),
        "lc_release": (C.c_int, [vp, i32]),
        "lc_ring_state": (C.c_int, [vp, i32, i32, C.POINTER(i64), C.POINTER(i64), C.POINTER(i64), C.POINTER(i64)]),
        "lc_fetch": (C.c_int, [vp, i32, i32, i32, C.POINTER(lc_fetch_out), i64, C.POINTER(i64)]),
        "lc_save_lkv2": (C.c_int, [vp, i32, C.c_char_p, C.c_char_p, vp, i64]),
        "lc_load_lkv2": (C.c_int, [vp, i32, C.c_char_p, C.c_char_p]),
        "lc_lkv2_info": (C.c_int, [C.c_char_p, C.POINTER(i64), C.POINTER(i64), C.POINTER(C.c_uint64)]),
        "lc_decode_attn": (C.c_int, [vp, i32, i32, vp, vp, i32, i32, C.c_float, u32, vp, i32, vp]),
        "lc_decode_attn_noalloc": (C.c_int, [vp, i32, i32, vp, vp, i32, i32, C.c_float, u32, vp, i32, vp]),
        "lc_decode_step": (C.c_int, [vp, i32, i32, vp, vp, vp, i32, vp, i32, i32, C.c_float, u32, vp, i32, vp]),
        "lc_decode_step_layers": (C.c_int, [vp, i32, i32, i32, vp, vp, vp, i32, vp, i32, i32, C.c_float, u32, vp, i32,
                                            vp]),
        "lc_prefill_attn": (C.c_int, [vp, i32, i32, vp, i32, i32, i32, C.c_float, u32, vp, i32, vp]),
        "lc_decode_attn_partials": (C.c_int, [vp, i32, i32, vp, vp, i32, i32, C.c_float, u32, vp, vp, vp, vp]),
        "lc_merge_partials": (C.c_int, [vp, i32, i32, vp, vp, vp, u32, vp, i32, vp]),
        "lc_group_id": (C.c_int, [vp]),
        "lc_group_create": (C.c_int, [i32, i32, vp, i32, i32, i32, u32, pp]),
        "lc_group_info": (C.c_int, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)]),
        "lc_group_status": (C.c_int, [vp]),
        "lc_group_destroy": (C.c_int, [vp]),
        "lc_decode_attn_split": (C.c_int, [vp, vp, i32, i32, vp, vp, i32, i32, C.c_float, u32, vp, i32, vp]),
        "lc_ring_create": (C.c_int, [i32, i64, i64, i32, vp, i32, pp]),
        "lc_ring_update": (C.c_int, [vp, vp, i64, i32, vp]),
        "lc_ring_truncate_to": (C.c_int, [vp, i64]),
        "lc_ring_counters": (C.c_int, [vp, C.POINTER(i64), C.POINTER(i64), C.POINTER(i64), C.POINTER(i64)]),
        "lc_ring_read": (C.c_int, [vp, i32, i32, vp, i64, C.POINTER(i64)]),
        "lc_ring_clear": (C.c_int, [vp]),
        "lc_ring_deep_clone": (C.c_int, [vp, pp]),
        "lc_ring_destroy": (None, [vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def _check(status: int):
    if status != LC_OK:
        raise LumenError(status, lib().lc_last_error().decode())


def _ptr(x) -> Optional[int]:
    """Address of a numpy array or torch tensor (must be contiguous)."""
    if x is None:
        return None
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("array must be C-contiguous")
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        if not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return x.data_ptr()
    raise TypeError(f"unsupported buffer type {type(x)}")


def _dtype_code(x) -> int:
    if isinstance(x, np.ndarray):
        if x.dtype == np.float32:
            return LC_F32
        if x.dtype == np.float16:
            return LC_F16
        raise TypeError("numpy inputs must be float32 or float16")
    name = str(x.dtype)
    return {"torch.float32": LC_F32, "torch.bfloat16": LC_BF16, "torch.float16": LC_F16}[name]


def _auto_stream(stream, *tensors):
    """The stream to run on: the caller's, else torch's current stream when a
    CUDA tensor is passed (so torch's allocator and our kernels stay ordered),
    else the library's own stream (None)."""
    if stream is not None:
        s = getattr(stream, "cuda_stream", stream)
        return s if s else CUDA_STREAM_LEGACY
    for t in tensors:
        if t is not None and getattr(t, "is_cuda", False):
            import torch

            return torch.cuda.current_stream(t.device).cuda_stream or CUDA_STREAM_LEGACY
    return None


def lkv2_info(path) -> dict:
    """Host-only read and check of an LKV2 snapshot (kv_disk.rs format)."""
    nl, nr, pos = C.c_int64(), C.c_int64(), C.c_uint64()
    _check(lib().lc_lkv2_info(os.fsencode(path), C.byref(nl), C.byref(nr), C.byref(pos)))
    return {"layers": nl.value, "records": nr.value, "position": pos.value}


def packed_words(n: int, bits: int) -> int:
    """bitpack.rs:11-14"""
    return int(lib().lc_packed_words(n, bits))


def version() -> str:
    return lib().lc_version().decode()


# ---------------------------------------------------------------------------
# lumen-core: TurboQuantConfig / TurboQuantCompressor
# ---------------------------------------------------------------------------
@dataclass
class TurboQuantConfig:
    """config.rs:3-28 (defaults bits 3, qjl_m 64, seed 42, 1000 EM iterations, head_dim 128)."""

    bits: int = 3
    qjl_m: int = 64
    seed: int = 42
    lloyd_max_iter: int = 1000
    head_dim: int = 128


class TurboQuantCompressor:
    """The tables of one compressor (R, Lloyd-Max codebook, QJL projection).

    ``TurboQuantCompressor(config)`` builds them like compressor.rs:20-32 with
    this library's generator; ``from_files`` loads the reference's
    TQCB/TQRM/TQJL files (compressor.rs:43-58); ``from_tables`` takes arrays.
    """

    def __init__(self, config: Optional[TurboQuantConfig] = None, *, _handle=None):
        self.config = config or TurboQuantConfig()
        if _handle is None:
            h = C.c_void_p()
            c = self.config
            _check(lib().lc_codec_new(c.bits, c.qjl_m, c.seed, c.lloyd_max_iter, c.head_dim, C.byref(h)))
            _handle = h
        self._h = _handle
        d, b, m = C.c_uint64(), C.c_uint32(), C.c_uint64()
        _check(lib().lc_codec_shape(self._h, C.byref(d), C.byref(b), C.byref(m)))
        self.head_dim, self.bits, self.qjl_m = d.value, b.value, m.value
        self.config = TurboQuantConfig(self.bits, self.qjl_m, self.config.seed, self.config.lloyd_max_iter,
                                       self.head_dim)

    @classmethod
    def from_files(cls, codebook_path: str, rotation_path: str, qjl_path: str, config=None):
        h = C.c_void_p()
        _check(lib().lc_codec_from_files(codebook_path.encode(), rotation_path.encode(), qjl_path.encode(),
                                         C.byref(h)))
        return cls(config, _handle=h)

    @classmethod
    def from_tables(cls, rotation: np.ndarray, boundaries: np.ndarray, centroids: np.ndarray,
                    qjl_proj: Optional[np.ndarray]):
        R = np.ascontiguousarray(rotation, np.float32)
        b = np.ascontiguousarray(boundaries, np.float64)
        c = np.ascontiguousarray(centroids, np.float64)
        P = None if qjl_proj is None else np.ascontiguousarray(qjl_proj, np.float32)
        d = R.shape[0]
        bits = int(round(np.log2(len(c))))
        m = 0 if P is None else P.shape[0]
        h = C.c_void_p()
        _check(lib().lc_codec_from_tables(d, bits, m, _ptr(R), _ptr(b), _ptr(c), _ptr(P), C.byref(h)))
        return cls(TurboQuantConfig(bits, m, 0, 0, d), _handle=h)

    def save(self, codebook_path: str, rotation_path: str, qjl_path: str):
        _check(lib().lc_codec_save(self._h, codebook_path.encode(), rotation_path.encode(), qjl_path.encode()))

    def tables(self):
        """(rotation [d,d] f32, boundaries f64, centroids f64, qjl_proj [m,d] f32)."""
        d, n, m = self.head_dim, 1 << self.bits, self.qjl_m
        R = np.empty((d, d), np.float32)
        b = np.empty(n + 1, np.float64)
        c = np.empty(n, np.float64)
        P = np.empty((max(m, 1), d), np.float32)
        _check(lib().lc_codec_tables(self._h, _ptr(R), _ptr(b), _ptr(c), _ptr(P)))
        return R, b, c, P[:m]

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib is not None:
            _lib.lc_codec_free(h)
            self._h = None


# ---------------------------------------------------------------------------
# The device cache
# ---------------------------------------------------------------------------
class CudaKvCache:
    """Multi-sequence TurboQuant KV cache on one GPU (lc_cache)."""

    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, k_codec: TurboQuantCompressor,
                 v_codec: Optional[TurboQuantCompressor] = None, *, max_seqs: int = 1, max_pages: int = 1024,
                 max_pages_per_seq: int = 256, store_flags: int = 0, device: int = 0, step_prealloc: bool = True,
                 layer_max_size: Optional[Sequence[int]] = None, layer_keep: Optional[Sequence[int]] = None):
        self.k_codec = k_codec
        self.v_codec = v_codec or k_codec
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.max_seqs, self.store_flags, self.device = max_seqs, store_flags, device
        cfg = lc_cache_config()
        cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, cfg.max_seqs = n_layers, n_kv_heads, head_dim, max_seqs
        cfg.max_pages, cfg.max_pages_per_seq, cfg.store_flags = max_pages, max_pages_per_seq, store_flags
        cfg.device, cfg.step_prealloc = device, int(step_prealloc)
        self._ms = self._kp = None
        if layer_max_size is not None:
            self._ms = (C.c_int64 * n_layers)(*layer_max_size)
            self._kp = (C.c_int64 * n_layers)(*(layer_keep or [0] * n_layers))
            cfg.layer_max_size = C.cast(self._ms, C.POINTER(C.c_int64))
            cfg.layer_keep = C.cast(self._kp, C.POINTER(C.c_int64))
        h = C.c_void_p()
        _check(lib().lc_cache_create(C.byref(cfg), self.k_codec._h, self.v_codec._h, C.byref(h)))
        self._h = h

    def close(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib is not None:
            _lib.lc_cache_destroy(h)
            self._h = None

    __del__ = close

    # -- info --
    def kernel_launches(self) -> int:
        n = C.c_uint64()
        _check(lib().lc_cache_info(self._h, None, None, C.byref(n)))
        return n.value

    def timing(self, mode: int):
        """lc_cache_timing: 1 start, 0 stop+report, 2 report. Returns
        (decode_ms, decode_launches, append_ms, append_launches, other_ms)."""
        dm, dn, am, an, om = C.c_double(), C.c_uint64(), C.c_double(), C.c_uint64(), C.c_double()
        _check(lib().lc_cache_timing(self._h, mode, C.byref(dm), C.byref(dn), C.byref(am), C.byref(an), C.byref(om)))
        return dm.value, dn.value, am.value, an.value, om.value

    def stream(self) -> int:
        s = C.c_void_p()
        _check(lib().lc_cache_info(self._h, None, C.byref(s), None))
        return s.value or 0

    # -- ring / block table --
    def append(self, layer: int, seq_ids, keys, values, stream=None):
        """Quantize-append keys/values [n_seqs, n_kv_heads, n_tokens, head_dim] (un-rotated)."""
        ids = np.ascontiguousarray(seq_ids, np.int32)
        n_tok = keys.shape[2]
        stream = _auto_stream(stream, keys, values)
        _check(lib().lc_append(self._h, layer, len(ids), _ptr(ids), _ptr(keys), _ptr(values), _dtype_code(keys),
                               n_tok, stream))

    def append_rope(self, layer: int, seq_ids, keys, values, rope_dims: int, rope_base: float = 10000.0,
                    traditional: bool = False, stream=None):
        """append() with RoPE applied to the keys first (positions continue
        each sequence's layer)."""
        ids = np.ascontiguousarray(seq_ids, np.int32)
        n_tok = keys.shape[2]
        stream = _auto_stream(stream, keys, values)
        _check(lib().lc_append_rope(self._h, layer, len(ids), _ptr(ids), _ptr(keys), _ptr(values), _dtype_code(keys),
                                    n_tok, rope_dims, rope_base, 1 if traditional else 0, stream))

    def truncate_to(self, seq: int, layer: int, target: int):
        _check(lib().lc_truncate_to(self._h, seq, layer, target))

    def fork(self, src: int, dst: int, prefix_len: int):
        _check(lib().lc_fork(self._h, src, dst, prefix_len))

    def release(self, seq: int):
        _check(lib().lc_release(self._h, seq))

    def ring_state(self, seq: int, layer: int):
        o, i, b, v = C.c_int64(), C.c_int64(), C.c_int64(), C.c_int64()
        _check(lib().lc_ring_state(self._h, seq, layer, C.byref(o), C.byref(i), C.byref(b), C.byref(v)))
        return dict(offset=o.value, idx=i.value, buf_len=b.value, view_len=v.value)

    def save_lkv2(self, seq: int, path, model_fingerprint: Optional[str] = None, prefix_tokens=()):
        """Snapshot sequence `seq`'s layers to an LKV2 file (kv_disk.rs)."""
        toks = np.ascontiguousarray(prefix_tokens, np.uint32)
        fp = None if model_fingerprint is None else model_fingerprint.encode()
        _check(lib().lc_save_lkv2(self._h, seq, os.fsencode(path), fp, _ptr(toks) if len(toks) else None, len(toks)))

    def load_lkv2(self, seq: int, path, model_fingerprint: Optional[str] = None):
        """Replace sequence `seq`'s layers with an LKV2 snapshot."""
        fp = None if model_fingerprint is None else model_fingerprint.encode()
        _check(lib().lc_load_lkv2(self._h, seq, os.fsencode(path), fp))

    def fetch(self, seq: int, layer: int, which: int = LC_FETCH_VIEW):
        """Stored vectors of (seq, layer) in the reference's CompressedVector layout."""
        st = self.ring_state(seq, layer)
        n = st["buf_len"] if which == LC_FETCH_BACKING else st["view_len"]
        H = self.n_kv_heads
        kw = np.zeros((H, n, packed_words(self.head_dim, self.k_codec.bits)), np.uint64)
        vw = np.zeros((H, n, packed_words(self.head_dim, self.v_codec.bits)), np.uint64)
        ks = np.zeros((H, n), np.float32)
        vs = np.zeros((H, n), np.float32)
        out = dict(k_words=kw, k_sigma=ks, v_words=vw, v_sigma=vs)
        fo = lc_fetch_out()
        fo.k_words, fo.k_sigma, fo.v_words, fo.v_sigma = _ptr(kw), _ptr(ks), _ptr(vw), _ptr(vs)
        if self.store_flags & LC_STORE_K_QJL:
            out["k_qjl"] = np.zeros((H, n, (self.k_codec.qjl_m + 63) // 64), np.uint64)
            out["k_rnorm"] = np.zeros((H, n), np.float32)
            fo.k_qjl, fo.k_rnorm = _ptr(out["k_qjl"]), _ptr(out["k_rnorm"])
        if self.store_flags & LC_STORE_V_QJL:
            out["v_qjl"] = np.zeros((H, n, (self.v_codec.qjl_m + 63) // 64), np.uint64)
            out["v_rnorm"] = np.zeros((H, n), np.float32)
            fo.v_qjl, fo.v_rnorm = _ptr(out["v_qjl"]), _ptr(out["v_rnorm"])
        got = C.c_int64()
        _check(lib().lc_fetch(self._h, seq, layer, which, C.byref(fo), n, C.byref(got)))
        return out

    # -- decode --
    def decode_attn(self, layer: int, seq_ids, q, n_q_heads: int, scale: float = 1.0, flags: int = 0, out=None,
                    out_dtype: int = LC_F32, stream=None):
        """softmax(scale q K^T) V for one query token per sequence; q [n_seqs, n_q_heads, head_dim]."""
        ids = np.ascontiguousarray(seq_ids, np.int32)
        if out is None:
            out = np.empty((len(ids), n_q_heads, self.head_dim), np.float32)
            out_dtype = LC_F32
        stream = _auto_stream(stream, q, out)
        _check(lib().lc_decode_attn(self._h, layer, len(ids), _ptr(ids), _ptr(q), _dtype_code(q), n_q_heads,
                                    scale, flags, _ptr(out), out_dtype, stream))
        return out

    def decode_step(self, layer: int, seq_ids, keys, values, q, n_q_heads: int, scale: float = 1.0, flags: int = 0,
                    out=None, out_dtype: int = LC_F32, stream=None):
        """append each sequence's new token (keys / values [n_seqs, n_kv_heads, 1, head_dim]), then
        decode_attn; the queries are rotated by the append launch."""
        ids = np.ascontiguousarray(seq_ids, np.int32)
        if isinstance(keys, np.ndarray):
            keys = np.ascontiguousarray(keys, np.float32)
            values = np.ascontiguousarray(values, np.float32)
        if out is None:
            out = np.empty((len(ids), n_q_heads, self.head_dim), np.float32)
            out_dtype = LC_F32
        stream = _auto_stream(stream, q, keys, out)
        _check(lib().lc_decode_step(self._h, layer, len(ids), _ptr(ids), _ptr(keys), _ptr(values), _dtype_code(keys),
                                    _ptr(q), _dtype_code(q), n_q_heads, scale, flags, _ptr(out), out_dtype, stream))
        return out

    def decode_step_layers(self, layer0: int, seq_ids, keys, values, q, n_q_heads: int, scale: float = 1.0,
                           flags: int = 0, out=None, out_dtype: int = LC_F32, stream=None):
        """decode_step for layers layer0 .. layer0 + len(keys) - 1 from one
        native call: keys / values [n_layers, n_seqs, n_kv_heads, 1, head_dim],
        q [n_layers, n_seqs, n_q_heads, head_dim], out like q (all contiguous)."""
        ids = seq_ids if isinstance(seq_ids, np.ndarray) and seq_ids.dtype == np.int32 else \
            np.ascontiguousarray(seq_ids, np.int32)
        n_layers = keys.shape[0]
        if isinstance(keys, np.ndarray):
            keys = np.ascontiguousarray(keys, np.float32)
            values = np.ascontiguousarray(values, np.float32)
        if out is None:
            out = np.empty((n_layers, len(ids), n_q_heads, self.head_dim), np.float32)
            out_dtype = LC_F32
        stream = _auto_stream(stream, q, keys, out)
        _check(lib().lc_decode_step_layers(self._h, layer0, n_layers, len(ids), _ptr(ids), _ptr(keys), _ptr(values),
                                           _dtype_code(keys), _ptr(q), _dtype_code(q), n_q_heads, scale, flags,
                                           _ptr(out), out_dtype, stream))
        return out

    def prefill_attn(self, layer: int, seq: int, q, n_q_heads: int, scale: float = 1.0, flags: int = 0, out=None,
                     out_dtype: int = LC_F32, stream=None):
        """Causal attention of the last len(q) tokens of (seq, layer) over its
        view; q [n_q_tokens, n_q_heads, head_dim]."""
        n_tok = q.shape[0]
        if out is None:
            out = np.empty((n_tok, n_q_heads, self.head_dim), np.float32)
            out_dtype = LC_F32
        stream = _auto_stream(stream, q, out)
        _check(lib().lc_prefill_attn(self._h, layer, seq, _ptr(q), _dtype_code(q), n_tok, n_q_heads, scale, flags,
                                     _ptr(out), out_dtype, stream))
        return out

    def decode_partials(self, layer: int, seq_ids, q, n_q_heads: int, scale: float = 1.0, flags: int = 0,
                        m=None, l=None, o=None, stream=None):
        ids = np.ascontiguousarray(seq_ids, np.int32)
        rows = len(ids) * n_q_heads
        if m is None:
            m = np.empty(rows, np.float32)
            l = np.empty(rows, np.float32)
            o = np.empty((rows, self.head_dim), np.float32)
        stream = _auto_stream(stream, q, m)
        _check(lib().lc_decode_attn_partials(self._h, layer, len(ids), _ptr(ids), _ptr(q), _dtype_code(q), n_q_heads,
                                             scale, flags, _ptr(m), _ptr(l), _ptr(o), stream))
        return m, l, o

    def decode_attn_split(self, group: "SplitGroup", layer: int, seq_ids, q, n_q_heads: int, scale: float = 1.0,
                          flags: int = 0, out=None, out_dtype: int = LC_F32, stream=None):
        """decode_attn over sequences split by tokens across `group`'s ranks:
        this cache holds this rank's shard in seq_ids; every rank calls with
        the same queries and gets the attention over the whole context."""
        ids = np.ascontiguousarray(seq_ids, np.int32)
        if out is None:
            out = np.empty((len(ids), n_q_heads, self.head_dim), np.float32)
            out_dtype = LC_F32
        stream = _auto_stream(stream, q, out)
        _check(lib().lc_decode_attn_split(self._h, group._h, layer, len(ids), _ptr(ids), _ptr(q), _dtype_code(q),
                                          n_q_heads, scale, flags, _ptr(out), out_dtype, stream))
        return out

    def merge_partials(self, m, l, o, flags: int = 0, out=None, out_dtype: int = LC_F32, stream=None):
        """m, l [n_parts, n_rows]; o [n_parts, n_rows, head_dim] -> out [n_rows, head_dim]."""
        n_parts, n_rows = m.shape
        if out is None:
            out = np.empty((n_rows, self.head_dim), np.float32)
            out_dtype = LC_F32
        stream = _auto_stream(stream, m, out)
        _check(lib().lc_merge_partials(self._h, n_parts, n_rows, _ptr(m), _ptr(l), _ptr(o), flags, _ptr(out),
                                       out_dtype, stream))
        return out

    # -- KVCache trait calls on one sequence --
    def store(self, seq, layer, head, keys, values, n_tokens):
        k = np.ascontiguousarray(keys, np.float32).reshape(n_tokens, self.head_dim) if isinstance(keys, np.ndarray) else keys
        v = np.ascontiguousarray(values, np.float32).reshape(n_tokens, self.head_dim) if isinstance(values, np.ndarray) else values
        _check(lib().lc_store(self._h, seq, layer, head, _ptr(k), _ptr(v), n_tokens))

    def seq_len(self, seq, layer, head) -> int:
        r = lib().lc_seq_len(self._h, seq, layer, head)
        if r < 0:
            _check(int(r))
        return int(r)

    def attend_keys(self, seq, layer, head, query) -> np.ndarray:
        n = self.seq_len(seq, layer, head)
        out = np.empty(max(n, 1), np.float32)
        q = np.ascontiguousarray(query, np.float32)
        _check(lib().lc_attend_keys(self._h, seq, layer, head, _ptr(q), _ptr(out), len(out)))
        return out[:n]

    def attend_keys_qjl(self, seq, layer, head, query) -> np.ndarray:
        """Two-stage scores: estimate_inner_products (compressor.rs:122-159)."""
        n = self.seq_len(seq, layer, head)
        out = np.empty(max(n, 1), np.float32)
        q = np.ascontiguousarray(query, np.float32)
        _check(lib().lc_attend_keys_qjl(self._h, seq, layer, head, _ptr(q), _ptr(out), len(out)))
        return out[:n]

    def attend_values(self, seq, layer, head, weights) -> np.ndarray:
        w = np.ascontiguousarray(weights, np.float32)
        out = np.empty(self.head_dim, np.float32)
        _check(lib().lc_attend_values(self._h, seq, layer, head, _ptr(w) if len(w) else None, len(w), _ptr(out)))
        return out

    def clear(self):
        _check(lib().lc_clear(self._h))

    def truncate(self, seq, layer, n_keep):
        _check(lib().lc_truncate(self._h, seq, layer, n_keep))


class SplitGroup:
    """lc_group: the ranks (one process per GPU) that hold token shards of the
    same sequences. Collective: every rank creates it with the same id (from
    `SplitGroup.new_id()` on one rank, sent by any side channel)."""

    @staticmethod
    def new_id() -> bytes:
        buf = (C.c_uint8 * LC_GROUP_ID_BYTES)()
        _check(lib().lc_group_id(buf))
        return bytes(buf)

    def __init__(self, world: int, rank: int, group_id: bytes, max_rows: int, head_dim: int, device: int = 0,
                 nccl: bool = False):
        if len(group_id) != LC_GROUP_ID_BYTES:
            raise ValueError(f"group id must be {LC_GROUP_ID_BYTES} bytes")
        idb = (C.c_uint8 * LC_GROUP_ID_BYTES).from_buffer_copy(group_id)
        h = C.c_void_p()
        _check(lib().lc_group_create(world, rank, idb, device, max_rows, head_dim, LC_GROUP_NCCL if nccl else 0,
                                     C.byref(h)))
        self._h = h.value

    def info(self) -> dict:
        w, r, p = C.c_int32(), C.c_int32(), C.c_int32()
        _check(lib().lc_group_info(self._h, C.byref(w), C.byref(r), C.byref(p)))
        return {"world": w.value, "rank": r.value, "peer_stores": bool(p.value)}

    def status(self) -> int:
        return lib().lc_group_status(self._h)

    def close(self):
        if getattr(self, "_h", None):
            h, self._h = self._h, None
            _check(lib().lc_group_destroy(h))


class KVCache:
    """turboquant-cache's trait (traits.rs:9-37)."""

    def store(self, layer, head, keys, values, n_tokens): raise NotImplementedError
    def attend_keys(self, layer, head, query): raise NotImplementedError
    def attend_values(self, layer, head, weights): raise NotImplementedError
    def seq_len(self, layer, head): raise NotImplementedError
    def clear(self): raise NotImplementedError
    def truncate(self, layer, n_keep): raise NotImplementedError


class SimpleCache(KVCache):
    """Drop-in for turboquant-cache SimpleCache (simple.rs:13-185): one sequence,
    `n_layers` x `n_kv_heads`, compressed on the GPU."""

    def __init__(self, compressor: TurboQuantCompressor, n_layers: int, n_kv_heads: int, head_dim: int, *,
                 v_compressor: Optional[TurboQuantCompressor] = None, max_tokens: int = 1 << 16, device: int = 0):
        pages = (max_tokens + 255) // 256
        self._c = CudaKvCache(n_layers, n_kv_heads, head_dim, compressor, v_compressor, max_seqs=1,
                              max_pages=pages * n_layers + 8, max_pages_per_seq=pages + 1,
                              store_flags=LC_STORE_K_QJL | LC_STORE_V_QJL, device=device)
        self.compressor = compressor
        self.head_dim = head_dim

    def store(self, layer, head, keys, values, n_tokens):
        self._c.store(0, layer, head, keys, values, n_tokens)

    def attend_keys(self, layer, head, query):
        return self._c.attend_keys(0, layer, head, query)

    def estimate_inner_products(self, layer, head, query):
        """Two-stage scores of the cached keys (compressor.rs:122-159)."""
        return self._c.attend_keys_qjl(0, layer, head, query)

    def attend_values(self, layer, head, weights):
        return self._c.attend_values(0, layer, head, weights)

    def seq_len(self, layer, head):
        return self._c.seq_len(0, layer, head)

    def clear(self):
        self._c.clear()

    def truncate(self, layer, n_keep):
        self._c.truncate(0, layer, n_keep)

    def memory_bytes(self) -> int:
        """simple.rs:102-119 with config.rs:48-55 per vector."""
        total = 0
        for side, comp in ((0, self._c.k_codec), (1, self._c.v_codec)):
            per = packed_words(self.head_dim, comp.bits) * 8 + ((comp.qjl_m + 63) // 64) * 8 + 4 + 4 + 8 + 4
            for layer in range(self._c.n_layers):
                for head in range(self._c.n_kv_heads):
                    total += self.seq_len(layer, head) * per
        return total

    def fetch(self, layer):
        return self._c.fetch(0, layer)


# ---------------------------------------------------------------------------
# The raw ring: NativeRotatingKvCacheTurboQuant's buffers on the device
# ---------------------------------------------------------------------------
class RawRing:
    """lc_ring: n buffers of fixed row width moving in lockstep (native_cache.rs:65-335)."""

    def __init__(self, n_heads: int, max_size: int, keep: int, row_bytes: Sequence[int], device: int = 0):
        rb = (C.c_int64 * len(row_bytes))(*row_bytes)
        h = C.c_void_p()
        _check(lib().lc_ring_create(n_heads, max_size, keep, len(row_bytes), rb, device, C.byref(h)))
        self._h, self.n_heads, self.row_bytes = h, n_heads, list(row_bytes)
        self.max_size, self.keep = max_size, keep

    def update(self, news: Sequence[np.ndarray], prealloc: bool = True):
        n_tok = news[0].shape[-2] if news[0].ndim >= 2 else 1
        arrs = [np.ascontiguousarray(a) for a in news]
        ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        _check(lib().lc_ring_update(self._h, ptrs, n_tok, int(prealloc), None))

    def truncate_to(self, target: int) -> bool:
        r = lib().lc_ring_truncate_to(self._h, target)
        if r == LC_ERR_REFUSED:
            return False
        _check(r)
        return True

    def counters(self):
        o, i, b, v = C.c_int64(), C.c_int64(), C.c_int64(), C.c_int64()
        _check(lib().lc_ring_counters(self._h, C.byref(o), C.byref(i), C.byref(b), C.byref(v)))
        return dict(offset=o.value, idx=i.value, buf_len=b.value, view_len=v.value)

    def read(self, buf: int, which: int = LC_FETCH_VIEW) -> Optional[bytes]:
        c = self.counters()
        n = c["buf_len"] if which == LC_FETCH_BACKING else c["view_len"]
        out = np.empty(self.n_heads * n * self.row_bytes[buf], np.uint8)
        got = C.c_int64()
        r = lib().lc_ring_read(self._h, buf, which, _ptr(out) if out.size else None, out.size, C.byref(got))
        if r == LC_ERR_STATE:
            return None
        _check(r)
        return out.tobytes()

    def clear(self):
        _check(lib().lc_ring_clear(self._h))

    def deep_clone(self) -> "RawRing":
        h = C.c_void_p()
        _check(lib().lc_ring_deep_clone(self._h, C.byref(h)))
        r = object.__new__(RawRing)
        r._h, r.n_heads, r.row_bytes, r.max_size, r.keep = h, self.n_heads, self.row_bytes, self.max_size, self.keep
        return r

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib is not None:
            _lib.lc_ring_destroy(h)
            self._h = None


class NativeRotatingKvCacheTurboQuant:
    """native_cache.rs:1517-1862 on the device: update_and_fetch over pre-quantized
    (k_codes, k_sigma, v_codes, v_sigma) and, after with_qjl(m),
    update_and_fetch_qjl over the six slots. Inputs are [1, H, S, W] arrays."""

    def __init__(self, max_size: int = 1024, keep: int = 0, bits: int = 4, *, n_heads: int = 1,
                 widths=(1, 1), device: int = 0):
        if max_size <= 0:
            raise ValueError("TurboQuant cache: max_size must be > 0")
        if keep >= max_size:
            raise ValueError(f"TurboQuant cache: keep={keep} must be < max_size={max_size}")
        if not 2 <= bits <= 8:
            raise ValueError(f"TurboQuant cache: bits must be in [2, 8], got {bits}")
        self.max_size, self.keep, self.bits, self.n_heads, self.device = max_size, keep, bits, n_heads, device
        self.qjl_m = None
        self._widths = widths  # (k code bytes, v code bytes) per row
        self._ring = None
        self._dtypes = None

    def with_qjl(self, qjl_m: int, words: int = 2):
        if qjl_m <= 0:
            raise ValueError("TurboQuant cache: qjl_m must be > 0")
        self.qjl_m = qjl_m
        self._qjl_words = words
        return self

    def _ensure(self, arrays):
        if self._ring is None:
            self._dtypes = [a.dtype for a in arrays]
            self._shapes = [a.shape[3] for a in arrays]
            rows = [a.shape[3] * a.dtype.itemsize for a in arrays]
            self._ring = RawRing(arrays[0].shape[1], self.max_size, self.keep, rows, self.device)

    def _update(self, arrays, prealloc):
        for a in arrays:
            if a.ndim != 4:
                raise LumenError(LC_ERR_INVALID, "TurboQuant cache: expected 4D inputs [B, n_kv, S, D]")
        s = arrays[0].shape[2]
        if any(a.shape[2] != s for a in arrays):
            raise LumenError(LC_ERR_INVALID, "TurboQuant cache: seq-len mismatch")
        self._ensure(arrays)
        self._ring.update([a[0] for a in arrays], prealloc)
        return [self._view(i) for i in range(len(arrays))]

    def _view(self, i, which=LC_FETCH_VIEW):
        b = self._ring.read(i, which)
        if b is None:
            return None
        H = self._ring.n_heads
        a = np.frombuffer(b, self._dtypes[i])
        return a.reshape(1, H, -1, self._shapes[i])

    def update_and_fetch(self, k_codes, k_sigma, v_codes, v_sigma, prealloc: bool = True):
        kc, ks, vc, vs = self._update([k_codes, k_sigma, v_codes, v_sigma], prealloc)
        return (kc, ks), (vc, vs)

    def update_and_fetch_qjl(self, k_codes, k_sigma, k_signs, k_rnorm, v_codes, v_sigma, prealloc: bool = True):
        if self.qjl_m is None:
            raise LumenError(LC_ERR_STATE, "TurboQuant cache: update_and_fetch_qjl called but qjl_m is not "
                                           "configured. Construct with `.with_qjl(m)`.")
        kc, ks, ksg, krn, vc, vs = self._update([k_codes, k_sigma, k_signs, k_rnorm, v_codes, v_sigma], prealloc)
        return (kc, ks, ksg, krn), (vc, vs)

    def truncate_to(self, target: int) -> bool:
        if self._ring is None:
            return target == 0
        return self._ring.truncate_to(target)

    def counters(self):
        if self._ring is None:
            return dict(offset=0, idx=0, buf_len=0, view_len=0)
        return self._ring.counters()

    def offset(self):
        return self.counters()["offset"]

    def idx(self):
        return self.counters()["idx"]

    def cached_len(self):
        return self.counters()["buf_len"]

    def backing(self, i):
        return None if self._ring is None else self._view(i, LC_FETCH_BACKING)

    def clear(self):
        if self._ring is not None:
            self._ring.clear()
