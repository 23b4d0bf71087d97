"""TEST INFRASTRUCTURE ONLY: host model of the rotating KV ring and the
golden-digest harness that pins it.

Restates mlx-lm's RotatingKVCache as the reference implements it for every
ring-backed cache, TurboQuant included (rabbitson87/lumen-rs,
crates/lumen-mlx/src/native_cache.rs):
  rotating_concat        :86-125
  ring_update_in_place   :146-231   (S == 1 with step prealloc)
  ring_update_concat     :240-268   (anything else)
  ring_update            :277-290
  ring_truncate          :304-335
  KV_CACHE_STEP = 256    :37
and the digest harness of crates/lumen-mlx/src/native_cache/golden_tests.rs
(SplitMix64 inputs :25-66, FNV-1a over shapes/dtypes/bits :73-155, plans
:182-239, TurboQuant cases :360-411, recorded digests :465-497).

Arrays are numpy ``[1, H, S, W]`` like the reference's MLX arrays. Only the
index bookkeeping matters; the element type never changes.
"""
from __future__ import annotations

import numpy as np

from pyoracle import fnv1a

KV_CACHE_STEP = 256


class RingError(Exception):
    pass


def _cat(parts):
    return np.concatenate(parts, axis=2)


def _sl(a, start, end):
    # MLX/numpy slicing on axis 2: clamps, empty when start >= end.
    return a[:, :, start:end, :]


def rotating_concat(old, new, idx, offset, keep, max_size):
    """native_cache.rs:86-125"""
    buf = old.shape[2]
    if idx == buf:
        ordered = old
    elif idx < offset:
        ordered = _cat([_sl(old, 0, keep), _sl(old, idx, buf), _sl(old, keep, idx)])
    else:
        ordered = _sl(old, 0, idx)
    held = ordered.shape[2]
    trim = max(held + 1 - max_size, 0)
    if trim == 0:
        return _cat([ordered, new])
    return _cat([_sl(ordered, 0, keep), _sl(ordered, trim + keep, held), new])


class RingModel:
    """N parallel buffers moving in lockstep (native_cache.rs:146-335)."""

    def __init__(self, n_bufs: int, max_size: int, keep: int):
        if max_size <= 0 or keep >= max_size:
            raise RingError("invalid ring geometry")
        self.bufs = [None] * n_bufs
        self.offset = 0
        self.idx = 0
        self.max_size = max_size
        self.keep = keep

    def update(self, news, prealloc: bool):
        if news[0].shape[2] == 1 and prealloc:
            return self._in_place(news)
        return self._concat(news)

    def _in_place(self, news):
        prev = self.offset
        b0 = self.bufs[0]
        need_grow = b0 is None or (prev >= b0.shape[2] and b0.shape[2] < self.max_size)
        if need_grow:
            if prev > self.max_size:
                raise RingError("usize underflow in grow")  # Rust would panic
            new_size = min(KV_CACHE_STEP, self.max_size - prev)
            for i, new in enumerate(news):
                s = new.shape
                block = np.zeros((s[0], s[1], new_size, s[3]), new.dtype)
                self.bufs[i] = block if self.bufs[i] is None else _cat([self.bufs[i], block])
            self.idx = prev
        buf_size = self.bufs[0].shape[2]
        if buf_size > self.max_size:
            trim = buf_size - self.max_size
            for i in range(len(self.bufs)):
                b = self.bufs[i]
                self.bufs[i] = _cat([_sl(b, 0, self.keep), _sl(b, trim + self.keep, buf_size)])
            self.idx = self.max_size
        if self.idx == self.max_size:
            self.idx = self.keep
        w = self.idx
        for i, new in enumerate(news):
            self.bufs[i] = self.bufs[i].copy()
            self.bufs[i][:, :, w:w + 1, :] = new
        self.idx += 1
        self.offset = prev + 1
        out = []
        for b in self.bufs:
            out.append(b if self.offset >= self.max_size else _sl(b, 0, self.offset))
        return out

    def _concat(self, news):
        held = sum(b is not None for b in self.bufs)
        assert held in (0, len(self.bufs))
        fetched = []
        for b, new in zip(self.bufs, news):
            if b is None:
                fetched.append(new.copy())
            else:
                fetched.append(rotating_concat(b, new, self.idx, self.offset, self.keep, self.max_size))
        self.offset += news[0].shape[2]
        self.idx = fetched[0].shape[2]
        self.bufs = list(fetched)
        return fetched

    def truncate_to(self, target: int) -> bool:
        """native_cache.rs:304-335; False where the reference returns Err."""
        if target > self.offset:
            return False
        if target == self.offset:
            return True
        if self.offset > self.max_size:
            return False
        self.offset = target
        self.idx = target
        return True

    def cached_len(self) -> int:
        return 0 if self.bufs[0] is None else self.bufs[0].shape[2]


# ----------------------------------------------------------------------------
# Golden digest harness (golden_tests.rs)
# ----------------------------------------------------------------------------
class Rng:
    """SplitMix64 (golden_tests.rs:26-35)."""

    M = 0xFFFFFFFFFFFFFFFF

    def __init__(self, seed: int):
        self.s = seed

    def next(self) -> int:
        self.s = (self.s + 0x9E3779B97F4A7C15) & self.M
        z = self.s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & self.M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & self.M
        return z ^ (z >> 31)

    def _n(self, n):
        return [self.next() for _ in range(n)]

    def positive(self, h, s, d):
        """golden_tests.rs:48-53: f32 in [0.5, 1.5)."""
        v = np.array([x >> 40 for x in self._n(h * s * d)], np.float32)
        return (v / np.float32(1 << 24) + np.float32(0.5)).astype(np.float32).reshape(1, h, s, d)

    def codes(self, h, s, d):
        """golden_tests.rs:56-59: u8 codes below 16."""
        return np.array([x >> 60 for x in self._n(h * s * d)], np.uint8).reshape(1, h, s, d)

    def words(self, h, s, d):
        """golden_tests.rs:62-65: u32 words."""
        return np.array([x & 0xFFFFFFFF for x in self._n(h * s * d)], np.uint32).reshape(1, h, s, d)


class Digest:
    """FNV-1a over shapes, dtypes and element bits (golden_tests.rs:73-155)."""

    def __init__(self):
        self.h = 0xCBF29CE484222325

    def bytes(self, b: bytes):
        self.h = fnv1a(self.h, b)

    def num(self, n: int):
        self.bytes(int(n).to_bytes(8, "little"))

    def array(self, a: np.ndarray):
        self.num(a.ndim)
        for d in a.shape:
            self.num(d)
        if a.size == 0:
            return
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint8:
            self.num(1)
        elif a.dtype == np.uint32:
            self.num(2)
        elif a.dtype == np.float32:
            self.num(3)
        else:
            raise TypeError(f"golden digest: no reader for {a.dtype}")
        self.bytes(a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes())

    def opt(self, a):
        if a is None:
            self.num(0)
        else:
            self.num(1)
            self.array(a)


H = 2  # golden_tests.rs:285

# golden_tests.rs:182-226
FULL = [("D", 3), ("C", 250), ("D", 5), ("C", 300), ("R", 500), ("D", 3), ("R", 600), ("C", 7), ("R", 510), ("D", 2)]
SMALL_RING = [("C", 5), ("D", 3), ("R", 6), ("D", 4), ("C", 3), ("D", 10), ("C", 20), ("D", 5), ("R", 30), ("C", 4),
              ("D", 3)]
LARGE_RING = [("D", 3), ("R", 2), ("C", 260), ("D", 40), ("C", 30), ("D", 3), ("R", 50), ("C", 2)]

# golden_tests.rs:235-239
TQ_PLANS = [("small", 12, 2, SMALL_RING), ("large", 300, 4, LARGE_RING), ("full", 4096, 0, FULL)]

# golden_tests.rs:465-497, recorded from the reference.
RECORDED_TQ = {
    ("small", False): 0x317E3BFF116A9EE8,
    ("small", True): 0xECCE0A8165FC6B99,
    ("large", False): 0x9212159C7532A30B,
    ("large", True): 0x4F12B91EE3F90B33,
    ("full", False): 0xF9CAB87F57FB453B,
    ("full", True): 0xF2CF59207A0C8E31,
}
RECORDED_TQ_QJL = {
    ("small", False): 0x0F372B77B7090518,
    ("small", True): 0x602909E0D05E6F27,
    ("large", False): 0xE01557C21B1FD2CE,
    ("large", True): 0xB978336B3D4715D2,
    ("full", False): 0x2931526276ECF5F7,
    ("full", True): 0xC0A764840E88A73B,
}


def tq_inputs(rng: Rng, s: int, qjl: bool):
    """Draw one update's inputs in the reference's order (golden_tests.rs:373-375, 393-396).

    Returns the list in ring-buffer order: [kc, ks, vc, vs] or
    [kc, ks, ksg, krn, vc, vs] (native_cache.rs:1780-1788, 1837-1850).
    """
    kc, ks = rng.codes(H, s, 16), rng.positive(H, s, 1)
    if qjl:
        ksg, krn = rng.words(H, s, 2), rng.positive(H, s, 1)
    vc, vs = rng.codes(H, s, 24), rng.positive(H, s, 1)
    return [kc, ks, ksg, krn, vc, vs] if qjl else [kc, ks, vc, vs]


class ModelCase:
    """NativeRotatingKvCacheTurboQuant driven through the model ring."""

    def __init__(self, max_size, keep, qjl):
        self.qjl = qjl
        self.ring = RingModel(6 if qjl else 4, max_size, keep)

    def update(self, s, rng, d, prealloc):
        out = self.ring.update(tq_inputs(rng, s, self.qjl), prealloc)
        for a in out:
            d.array(a)

    def rewind(self, target):
        return self.ring.truncate_to(target)

    def buffers(self):
        """(keys_codes, keys_sigma, values_codes, values_sigma, keys_signs, keys_residual_norm)."""
        b = self.ring.bufs
        if self.qjl:
            return b[0], b[1], b[4], b[5], b[2], b[3]
        return b[0], b[1], b[2], b[3], None, None

    def counters(self):
        return self.ring.offset, self.ring.idx, self.ring.cached_len()


def turboquant_state(case, d: Digest):
    """golden_tests.rs:360-370"""
    for a in case.buffers():
        d.opt(a)
    off, idx, cl = case.counters()
    d.num(off)
    d.num(idx)
    d.num(cl)


def run_plan(case, steps, prealloc: bool) -> int:
    """golden_tests.rs:243-263"""
    rng = Rng(0x0022DEDC)
    d = Digest()
    for kind, n in steps:
        times, kind, n = (n, "C", 1) if kind == "D" else (1, kind, n)
        for _ in range(times):
            if kind == "C":
                case.update(n, rng, d, prealloc)
            else:
                d.num(1 if case.rewind(n) else 0)
            turboquant_state(case, d)
    return d.h


def digests(make_case, qjl: bool):
    out = {}
    for name, max_size, keep, steps in TQ_PLANS:
        for prealloc in (False, True):
            out[(name, prealloc)] = run_plan(make_case(max_size, keep, qjl), steps, prealloc)
    return out
