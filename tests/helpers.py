"""Seeded synthetic inputs with the distributions BASELINE.json's configs name.

K, V ~ N(0, 1) with 4 seed-chosen channels per kv head scaled x8 (key
outliers); queries ~ N(0, 1) or N(0, 1/sqrt(head_dim)). The stream is the
oracle's SplitMix64 + Box-Muller, so tests, bench and fixtures agree.
"""
import numpy as np


def splitmix(seed: int):
    s = seed & 0xFFFFFFFFFFFFFFFF
    while True:
        s = (s + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        z = s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        yield z ^ (z >> 31)


def outlier_channels(seed: int, n_heads: int, dim: int, k: int = 4):
    g = splitmix(seed)
    out = []
    for _ in range(n_heads):
        ch = []
        while len(ch) < k:
            c = next(g) % dim
            if c not in ch:
                ch.append(int(c))
        out.append(sorted(ch))
    return out


def kv(orc, seed: int, n_seqs: int, n_heads: int, n_tok: int, dim: int, outliers: bool = True):
    """[n_seqs, n_heads, n_tok, dim] f32 with x8 outlier channels per head."""
    x = orc.gauss_f32(seed, n_seqs * n_heads * n_tok * dim).reshape(n_seqs, n_heads, n_tok, dim)
    if outliers:
        for h, ch in enumerate(outlier_channels(seed ^ 0x5EED, n_heads, dim)):
            x[:, h, :, ch] *= np.float32(8.0)
    return x


def queries(orc, seed: int, n_seqs: int, n_q: int, dim: int, std: float = 1.0):
    return (orc.gauss_f32(seed, n_seqs * n_q * dim).reshape(n_seqs, n_q, dim) * np.float32(std)).astype(np.float32)


def to_bf16(x: np.ndarray):
    """Round f32 to bf16 (nearest even); returns (torch bf16 tensor, exact f32 values)."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16)
    return t, t.float().numpy()


def rel_mse(ref, got):
    """turboquant.rs:993-1003: MSE / mean(ref^2)."""
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    return float(np.mean((ref - got) ** 2) / (np.mean(ref ** 2) + 1e-12))


ATTN_ATOL = 2e-3
ATTN_RTOL = 1e-3
ATTN_REL_MSE = 1e-3


def attn_close(got, ref):
    """Attention-output parity: for every output row (one query head's
    head_dim vector) max|got - ref| <= 2e-3 + 1e-3 * max|ref row|, and over all
    outputs the relative MSE of turboquant.rs:993-1003 <= 1e-3.

    The relative part is taken against the row's scale: the output is
    R^T o, and the rotation spreads a rounding of o evenly over every
    element of the row, small elements included. Returns (ok, message)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    scale = np.abs(ref).max(axis=-1, keepdims=True)
    excess = float((err - (ATTN_ATOL + ATTN_RTOL * scale)).max())
    rm = rel_mse(ref, got)
    ok = excess <= 0 and rm <= ATTN_REL_MSE
    return ok, f"max_abs={err.max():.3e} worst excess={excess:.3e} rel_mse={rm:.3e}"
