"""Write the golden fixtures of tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py

The reference repository commits no codebook, rotation, projection or
compressed-vector fixtures: its own tests pin the path by 12 ring digests
(native_cache/golden_tests.rs:465-497) and by statistical thresholds. The
oracle restates its algorithm and passes those tests (test_oracle_*.py).
Its outputs for the fixed seeds below are frozen here, so later changes to
the oracle, the product codec or the device kernels are caught bit for bit:

  tq_d128_s42.tqrm        rotation, TQRM format (rotation.rs:130-150), seed 42
  tq_d128_m64_s43.tqjl    QJL projection, TQJL format (qjl.rs:248-272), seed 43
  tq_b{2,3,4}.tqcb        Lloyd-Max codebooks, TQCB format (lloyd_max.rs:187-213)
  compress_d128.npz       24 seeded vectors with outlier channels and their
                          compressed form for bits 2, 3, 4: stage-1 words,
                          QJL words, residual norm, scale (compressor.rs:60-116)
  attend_d128_b4.npz      one sequence (8 kv heads, 300 tokens, 4-bit K/V)
                          and 32 queries: SimpleCache attend_keys + softmax +
                          attend_values outputs (simple.rs, scale 1/sqrt(128))
"""
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

DIM, M, SEED = 128, 64, 42


def write_tqrm(path, R):
    with open(path, "wb") as f:
        f.write(b"TQRM" + struct.pack("<I", R.shape[0]) + np.ascontiguousarray(R, "<f4").tobytes())


def write_tqjl(path, P):
    with open(path, "wb") as f:
        f.write(b"TQJL" + struct.pack("<II", P.shape[1], P.shape[0]) + np.ascontiguousarray(P, "<f4").tobytes())


def write_tqcb(path, bits, bounds, cents):
    with open(path, "wb") as f:
        f.write(b"TQCB" + struct.pack("<II", bits, 1 << bits))
        f.write(np.ascontiguousarray(bounds, "<f8").tobytes() + np.ascontiguousarray(cents, "<f8").tobytes())


def fixtures(orc):
    """Everything the files hold, recomputed: {name: value}."""
    import helpers

    out = {}
    tabs = {b: orc.Tables.generate(DIM, b, M, SEED) for b in (2, 3, 4)}
    out["R"] = tabs[4].R
    out["P"] = tabs[4].proj
    for b, t in tabs.items():
        out[f"bounds{b}"], out[f"cents{b}"] = t.bounds, t.cents
    X = helpers.kv(orc, 2024, 1, 3, 8, DIM)[0].reshape(24, DIM)
    comp = {"x": X}
    for b, t in tabs.items():
        s1, s2, rn, sc = orc.Compressor(t).compress(X)
        comp[f"stage1_b{b}"], comp[f"stage2_b{b}"], comp[f"rnorm_b{b}"], comp[f"scale_b{b}"] = s1, s2, rn, sc
    out["compress"] = comp
    t = tabs[4]
    c = orc.Compressor(t)
    sc = orc.SimpleCache(c, c, 1, 8, DIM)
    K = helpers.kv(orc, 77, 1, 8, 300, DIM)[0]
    V = helpers.kv(orc, 78, 1, 8, 300, DIM)[0]
    for h in range(8):
        sc.store(0, h, K[h], V[h], 300)
    q = helpers.queries(orc, 79, 1, 32, DIM)[0]
    scale = 1.0 / np.sqrt(DIM)
    att = np.stack([sc.attend(0, h // 4, q[h], scale) for h in range(32)])
    out["attend"] = {"kv_seeds": np.array([77, 78, 79]), "n_tokens": np.array(300), "q": q, "out": att}
    return out


def main():
    import pyoracle as orc

    orc.build()
    f = fixtures(orc)
    write_tqrm(os.path.join(HERE, "tq_d128_s42.tqrm"), f["R"])
    write_tqjl(os.path.join(HERE, "tq_d128_m64_s43.tqjl"), f["P"])
    for b in (2, 3, 4):
        write_tqcb(os.path.join(HERE, f"tq_b{b}.tqcb"), b, f[f"bounds{b}"], f[f"cents{b}"])
    np.savez(os.path.join(HERE, "compress_d128.npz"), **f["compress"])
    np.savez(os.path.join(HERE, "attend_d128_b4.npz"), **f["attend"])
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
