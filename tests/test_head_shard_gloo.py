"""CPU, world size 2 over gloo: kv-head-group sharding.

split.head_shard gives each rank a contiguous range of kv heads, and the
rank holds those heads (with their query groups) of every sequence. The
reference's cache API is per kv head (tqc/traits.rs:1-37: store /
attend_keys / attend_values take a head), and a query head attends only to
its kv head, so the shards need no communication. Each rank here stands in
for its GPU cache with an oracle SimpleCache of its heads; the ranks'
outputs, gathered in rank order and concatenated over heads, must equal
the oracle's attention over all heads bit for bit.
"""
import importlib
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DIM, HKV, HQ, N = 64, 8, 16, 200


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
    import helpers
    import pyoracle as orc

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        split = importlib.import_module("lumen-rs_b200.split")
        lo, hi = split.head_shard(HKV, rank, world)
        G = HQ // HKV
        t = orc.Tables.generate(DIM, 4, 0, 42)
        comp = orc.Compressor(t)
        K = helpers.kv(orc, 51, 1, HKV, N, DIM)[0]
        V = helpers.kv(orc, 52, 1, HKV, N, DIM)[0]
        q = helpers.queries(orc, 53, 1, HQ, DIM)[0]
        sc = orc.SimpleCache(comp, comp, 1, hi - lo, DIM)
        for h in range(lo, hi):
            sc.store(0, h - lo, np.ascontiguousarray(K[h]), np.ascontiguousarray(V[h]), N)
        mine = np.stack([sc.attend(0, (qh - lo * G) // G, q[qh], 1.0 / np.sqrt(DIM)) for qh in range(lo * G, hi * G)])
        parts = [None] * world
        dist.all_gather_object(parts, mine)
        if rank == 0:
            np.save(os.path.join(result_dir, "gathered.npy"), np.concatenate(parts, axis=0))
    finally:
        dist.destroy_process_group()


def test_head_shards_concatenate_to_whole_attention(orc, tmp_path):
    import torch.multiprocessing as mp

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import helpers

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    t = orc.Tables.generate(DIM, 4, 0, 42)
    comp = orc.Compressor(t)
    K = helpers.kv(orc, 51, 1, HKV, N, DIM)[0]
    V = helpers.kv(orc, 52, 1, HKV, N, DIM)[0]
    q = helpers.queries(orc, 53, 1, HQ, DIM)[0]
    full = orc.SimpleCache(comp, comp, 1, HKV, DIM)
    for h in range(HKV):
        full.store(0, h, np.ascontiguousarray(K[h]), np.ascontiguousarray(V[h]), N)
    ref = np.stack([full.attend(0, qh // (HQ // HKV), q[qh], 1.0 / np.sqrt(DIM)) for qh in range(HQ)])
    got = np.load(tmp_path / "gathered.npy")
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_head_shard_partition(world):
    split = importlib.import_module("lumen-rs_b200.split")
    spans = [split.head_shard(8, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == 8
    assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
