"""CPU: the page-sparse selection policy, and the selection algorithm the GPU
kernel runs, against a plain sort.

The policy is sdpa_page_sparse's (crates/lumen-mlx/src/native_attention.rs:
210-329): 64-token pages, the first page and the 4 most recent full pages
pinned, keep = max(pages / 8, 64), dense below 16384 keys or when pages <=
keep, the partial tail always attended, ties at the boundary to the lower
page.

k_page_select finds the keep-th largest bound by a radix select over the
order-preserving bit patterns of the bounds (4 passes of 8 bits, most
significant first), takes every key above it and the lowest-indexed keys
equal to it, and writes the chosen pages in ascending order. The model below
restates those steps in numpy so the tie handling is checked on CPU.
"""
import numpy as np
import pytest

PINNED = np.uint32(0xFFFFFFFF)


def order_key(f):
    """The kernel's order_key: f32 -> u32 with the same order (-0 as +0)."""
    f = np.where(f == 0, np.float32(0), np.asarray(f, np.float32)).astype(np.float32)
    u = f.view(np.uint32)
    return np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def radix_select(keys, keep):
    """(T, need): T the keep-th largest key, need how many keys equal to T are taken."""
    prefix, pmask, need = np.uint32(0), np.uint32(0), keep
    for shift in (24, 16, 8, 0):
        inside = (keys & pmask) == prefix
        hist = np.bincount(((keys[inside] >> np.uint32(shift)) & np.uint32(255)).astype(np.int64), minlength=256)
        cum = 0
        for b in range(255, -1, -1):  # bins from the top
            if cum + hist[b] >= need:
                prefix = prefix | np.uint32(b << shift)
                need -= cum
                break
            cum += hist[b]
        pmask = pmask | np.uint32(255 << shift)
    return prefix, need


def gpu_pages(bounds, P):
    """Chosen pages (ascending) the way k_page_select picks them."""
    keep = max(P // 8, 64)
    idx = np.arange(P)
    pinned = (idx < 1) | (idx >= P - 4)
    keys = np.where(pinned, PINNED, order_key(bounds))
    T, need = radix_select(keys, keep)
    eq = keys == T
    eq_rank = np.cumsum(eq) - eq  # ties before this page
    on = (keys > T) | (eq & (eq_rank < need))
    return np.flatnonzero(on)


def sorted_pages(bounds, P):
    """The policy by a plain sort: pinned first, then bound descending, then page."""
    keep = max(P // 8, 64)
    idx = np.arange(P)
    pinned = (idx < 1) | (idx >= P - 4)
    order = sorted(range(P), key=lambda p: (0 if pinned[p] else 1, -float(bounds[p]), p))
    return np.sort(np.array(order[:keep]))


@pytest.mark.parametrize("P,ties,seed", [(512, 0, 1), (512, 40, 2), (300, 200, 3), (4096, 500, 4), (257, 0, 5)])
def test_radix_select_matches_sort(P, ties, seed):
    rng = np.random.default_rng(seed)
    bounds = rng.standard_normal(P).astype(np.float32) * np.float32(3)
    if ties:  # many pages share the bound at the selection boundary
        keep = max(P // 8, 64)
        boundary = np.sort(bounds)[::-1][keep]
        bounds[rng.choice(P, size=ties, replace=False)] = boundary
    bounds[rng.choice(P, size=3, replace=False)] = -0.0  # -0 and +0 compare equal
    bounds[rng.choice(P, size=3, replace=False)] = 0.0
    got = gpu_pages(bounds, P)
    want = sorted_pages(bounds, P)
    np.testing.assert_array_equal(got, want)
    assert len(got) == max(P // 8, 64)


def test_order_key_preserves_order():
    rng = np.random.default_rng(9)
    f = np.concatenate([rng.standard_normal(1000).astype(np.float32) * np.float32(1e3),
                        np.array([0.0, -0.0, np.inf, -np.inf, 1e-38, -1e-38], np.float32)])
    k = order_key(f)
    for i in range(len(f)):
        assert ((k > k[i]) == (f > f[i])).all()
        assert ((k == k[i]) == (f == f[i])).all()


def test_quest_select_policy(orc):
    """pyoracle.quest_select: dense below the key threshold or when pages <=
    keep; otherwise pinned pages, exactly keep pages, the tail kept."""
    dim, bits = 128, 4
    t = orc.Tables.generate(dim, bits, 64, 42)
    comp = orc.Compressor(t)
    rng = np.random.default_rng(11)

    def stored(n):
        x = rng.standard_normal((n, dim)).astype(np.float32)
        words = np.stack([comp.compress(x[i])[0] for i in range(n)])
        sigma = np.array([comp.compress(x[i])[3] for i in range(n)], np.float32)
        return words, sigma

    q = rng.standard_normal((4, dim))
    words, sigma = stored(4096 + 30)  # below 16384 keys: dense
    mask, gap = orc.quest_select(words, sigma, t.cents, bits, dim, q)
    assert mask.all() and gap == float("inf")
    n = 16384 + 40
    words, sigma = stored(n)
    mask, _ = orc.quest_select(words, sigma, t.cents, bits, dim, q)
    P = n // 64
    keep = max(P // 8, 64)
    pages = mask[:P * 64].reshape(P, 64)
    assert (pages.all(1) | ~pages.any(1)).all()  # whole pages
    chosen = np.flatnonzero(pages.all(1))
    assert len(chosen) == keep
    assert 0 in chosen and all(p in chosen for p in range(P - 4, P))
    assert mask[P * 64:].all()  # the undigested tail
