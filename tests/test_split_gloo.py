"""CPU, world size 2 over gloo: the sequence-split decode host path.

lumen-rs_b200/split.py shards one sequence's tokens over the ranks, gathers
each rank's softmax partials (m, l, o) and merges them. This test runs its
SplitSequenceDecoder in two gloo processes on CPU. Each rank stands in for
its GPU cache with an oracle SimpleCache of its token range: partials come
from the oracle's attend_keys / attend_values, and the merge restates the
combine of partial softmax states. The merged output must equal oracle
attention over the whole sequence. The CUDA partials and merge kernels
have their own GPU test (test_gpu_decode.py::test_partials_and_merge_split_sequence).
"""
import importlib
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LOG2E = 1.4426950408889634


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleShard:
    """decode_partials / merge_partials of one rank, on the CPU oracle."""

    def __init__(self, orc, tables, K, V, lo, hi):
        self.head_dim = K.shape[-1]
        comp = orc.Compressor(tables)
        self.hkv = K.shape[0]
        self.sc = orc.SimpleCache(comp, comp, 1, self.hkv, self.head_dim)
        for h in range(self.hkv):
            if hi > lo:
                self.sc.store(0, h, np.ascontiguousarray(K[h, lo:hi]), np.ascontiguousarray(V[h, lo:hi]), hi - lo)
        self.n = hi - lo

    def decode_partials(self, layer, seq_ids, q, n_q_heads, scale, flags, m, l, o):
        qn = q.numpy().reshape(n_q_heads, self.head_dim)
        G = n_q_heads // self.hkv
        for h in range(n_q_heads):
            if self.n == 0:
                m[h], l[h] = float("-inf"), 0.0
                o[h] = 0.0
                continue
            s = self.sc.attend_keys(0, h // G, qn[h]).astype(np.float64)
            z = s * scale * LOG2E
            mx = z.max()
            p = np.exp2(z - mx).astype(np.float32)
            m[h] = float(mx)
            l[h] = float(p.astype(np.float64).sum())
            o[h] = __import__("torch").from_numpy(self.sc.attend_values(0, h // G, p).astype(np.float32))

    def merge_partials(self, gm, gl, go, flags, out, out_dtype=0):
        gm, gl, go = gm.numpy().astype(np.float64), gl.numpy().astype(np.float64), go.numpy().astype(np.float64)
        M = gm.max(axis=0)
        w = np.where(np.isneginf(gm), 0.0, np.exp2(gm - M))
        L = (w * gl).sum(axis=0)
        res = (w[:, :, None] * go).sum(axis=0) / L[:, None]
        out[:] = __import__("torch").from_numpy(res.astype(np.float32))
        return out


def _worker(rank, world, port, n_tok, result_dir):
    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import helpers
    import pyoracle as orc

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        split = importlib.import_module("lumen-rs_b200.split")
        dim, hkv, hq = 64, 2, 8
        t = orc.Tables.generate(dim, 4, 0, 42)
        kv = helpers.kv(orc, 31, 2, hkv, n_tok, dim)
        K, V = kv[0], kv[1]
        lo, hi = split.shard_range(n_tok, rank, world)
        shard = OracleShard(orc, t, K, V, lo, hi)
        dec = split.SplitSequenceDecoder(shard)
        q = torch.from_numpy(helpers.queries(orc, 5, 1, hq, dim))
        out = dec.decode(0, q, hq, scale=1.0 / np.sqrt(dim))
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_tok", [301, 1])
def test_split_decode_gloo_world2(orc, tmp_path, n_tok):
    import torch.multiprocessing as mp

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import helpers

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), n_tok, str(tmp_path)), nprocs=world, join=True)
    dim, hkv, hq = 64, 2, 8
    t = orc.Tables.generate(dim, 4, 0, 42)
    comp = orc.Compressor(t)
    kv = helpers.kv(orc, 31, 2, hkv, n_tok, dim)
    K, V = kv[0], kv[1]
    full = orc.SimpleCache(comp, comp, 1, hkv, dim)
    for h in range(hkv):
        full.store(0, h, np.ascontiguousarray(K[h]), np.ascontiguousarray(V[h]), n_tok)
    q = helpers.queries(orc, 5, 1, hq, dim)[0]
    scale = 1.0 / np.sqrt(dim)
    ref = np.stack([full.attend(0, h // (hq // hkv), q[h], scale) for h in range(hq)])
    # f32 sums in a different order (per shard, then combined): 5e-5 of the
    # row scale
    tol = 5e-5 * np.abs(ref).max(axis=-1, keepdims=True)
    for r in range(world):
        got = np.load(tmp_path / f"out{r}.npy")
        assert (np.abs(got - ref) <= tol).all(), float(np.abs(got - ref).max())


def test_shard_range_partition():
    split = importlib.import_module("lumen-rs_b200.split")
    for n in [0, 1, 7, 8, 1048576, 1048577]:
        for world in [1, 2, 3, 8]:
            spans = [split.shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        split.shard_range(10, 2, 2)


def _worker_rank_fails(rank, world, port, result_dir):
    """Rank 1 leaves before the gather; rank 0's decode must fail, not hang."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import helpers
    import pyoracle as orc

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=3))
    if rank == 1:
        return  # leaves between steps, with nothing of its own in flight
    split = importlib.import_module("lumen-rs_b200.split")
    dim, hkv, hq, n_tok = 64, 2, 8, 64
    t = orc.Tables.generate(dim, 4, 0, 42)
    kv = helpers.kv(orc, 31, 2, hkv, n_tok, dim)
    lo, hi = split.shard_range(n_tok, rank, world)
    dec = split.SplitSequenceDecoder(OracleShard(orc, t, kv[0], kv[1], lo, hi))
    q = torch.from_numpy(helpers.queries(orc, 5, 1, hq, dim))
    try:
        dec.decode(0, q, hq, scale=1.0 / np.sqrt(dim))
        status = "completed"
    except Exception as e:  # the collective's timeout or closed-connection error
        status = "error: " + type(e).__name__
    with open(os.path.join(result_dir, "rank0.txt"), "w") as f:
        f.write(status)


def test_split_decode_peer_failure_is_an_error(tmp_path):
    """A rank that exits before the partials all-gather: the surviving rank's
    split decode raises within the process-group timeout instead of hanging."""
    import time

    import torch.multiprocessing as mp

    t0 = time.time()
    mp.spawn(_worker_rank_fails, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    status = (tmp_path / "rank0.txt").read_text()
    assert status.startswith("error"), status
    assert time.time() - t0 < 120
