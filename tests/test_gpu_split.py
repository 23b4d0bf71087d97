"""GPU: SplitSequenceDecoder on the CUDA partials and merge kernels.

Two shards of one sequence live in two sequence slots of one cache. The
decoder for shard 0 is given a gather that stacks its own partials with
shard 1's, as an all-gather over two ranks would. Its merged output must
match decode attention over the whole sequence, held in a third slot, to
the decode tolerance. A second test runs the real NCCL all-gather with one
rank.
"""
import importlib
import os
import socket

import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _cache(lc, orc, n, cut, dim=128, hkv=8):
    t = orc.Tables.generate(dim, 4, 64, 42)
    codec = lc.TurboQuantCompressor.from_tables(t.R, t.bounds, t.cents, t.proj)
    pages = (n + 255) // 256 + 2
    cache = lc.CudaKvCache(1, hkv, dim, codec, max_seqs=3, max_pages=3 * pages + 8, max_pages_per_seq=pages)
    K = helpers.kv(orc, 71, 1, hkv, n, dim)
    V = helpers.kv(orc, 72, 1, hkv, n, dim)
    cache.append(0, [0], np.ascontiguousarray(K[:, :, :cut]), np.ascontiguousarray(V[:, :, :cut]))
    cache.append(0, [1], np.ascontiguousarray(K[:, :, cut:]), np.ascontiguousarray(V[:, :, cut:]))
    cache.append(0, [2], K, V)
    return cache


def test_split_decoder_two_shards(lc, orc, gpu):
    import torch

    split = importlib.import_module("lumen-rs_b200.split")
    n, cut, hq, dim = 5000, 1800, 32, 128
    cache = _cache(lc, orc, n, cut)
    q = torch.from_numpy(helpers.queries(orc, 3, 1, hq, dim)).cuda()
    scale = 1.0 / np.sqrt(dim)

    def shard1_partials():
        buf = torch.empty(hq * (dim + 2), device="cuda")
        cache.decode_partials(0, [1], q, hq, scale, m=buf[:hq], l=buf[hq:2 * hq], o=buf[2 * hq:].view(hq, dim))
        return buf

    dec = split.SplitSequenceDecoder(cache, seq_id=0, gather=lambda b: torch.stack([b, shard1_partials()]))
    got = dec.decode(0, q, hq, scale)
    torch.cuda.synchronize()
    ref = cache.decode_attn(0, [2], q, hq, scale)
    ok, msg = helpers.attn_close(got.cpu().numpy(), ref[0])
    assert ok, msg
    cache.close()


def test_split_decoder_nccl_one_rank(lc, orc, gpu):
    import torch
    import torch.distributed as dist

    split = importlib.import_module("lumen-rs_b200.split")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            device_id=torch.device("cuda", 0))
    try:
        n, hq, dim = 3000, 32, 128
        cache = _cache(lc, orc, n, n // 2)
        q = torch.from_numpy(helpers.queries(orc, 4, 1, hq, dim)).cuda()
        scale = 1.0 / np.sqrt(dim)
        got = split.SplitSequenceDecoder(cache, seq_id=2).decode(0, q, hq, scale)
        torch.cuda.synchronize()
        ref = cache.decode_attn(0, [2], q, hq, scale)
        ok, msg = helpers.attn_close(got.cpu().numpy(), ref[0])
        assert ok, msg
        cache.close()
    finally:
        dist.destroy_process_group()
