"""GPU: one context split by tokens over a group of ranks (lc_group,
lc_decode_attn_split).

Each rank holds a contiguous token shard of the sequence in its own cache;
the library computes the rank's softmax partials, exchanges them (peer
stores over NVLink with release flags, or an in-place NCCL all-gather) and
merges them (native_quant_attention.rs:190-207), all on the stream. The
merged output must match the oracle's attention over the whole sequence
(helpers.attn_close), on every rank and on successive calls (the exchange
buffers alternate by call parity).

World 1 runs on one GPU. World 2 needs two GPUs (skipped otherwise): the
ranks are child processes, one per GPU, with a gloo process group for the
plumbing (the group id) and NCCL's NVLS off. The failure test keeps rank 1
alive but has it skip the call: rank 0's bounded wait for rank 1's flags
runs out, its output rows are NaN and lc_group_status reports
LC_ERR_TIMEOUT; no GPU hangs or faults.
"""
import importlib
import os
import socket
import sys

import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DIM, HKV, HQ = 128, 8, 32


def _two_gpus():
    try:
        import torch

        return torch.cuda.device_count() >= 2
    except Exception:
        return False


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _kv(orc, n):
    return helpers.kv(orc, 700, 1, HKV, n, DIM)[0], helpers.kv(orc, 701, 1, HKV, n, DIM)[0]


def _oracle(orc, n, q, scale):
    t = orc.Tables.generate(DIM, 4, 64, 42)
    comp = orc.Compressor(t)
    K, V = _kv(orc, n)
    ref = orc.SimpleCache(comp, comp, 1, HKV, DIM)
    for h in range(HKV):
        ref.store(0, h, np.ascontiguousarray(K[h]), np.ascontiguousarray(V[h]), n)
    return np.stack([ref.attend(0, h // (HQ // HKV), q[h], scale) for h in range(HQ)])


def _shard_cache(lc, orc, n, lo, hi, device):
    t = orc.Tables.generate(DIM, 4, 64, 42)
    ck = lc.TurboQuantCompressor.from_tables(t.R, t.bounds, t.cents, t.proj)
    pages = (hi - lo + 255) // 256 + 1
    cache = lc.CudaKvCache(1, HKV, DIM, ck, max_seqs=1, max_pages=pages + 4, max_pages_per_seq=pages, device=device)
    K, V = _kv(orc, n)
    if hi > lo:
        cache.append(0, [0], np.ascontiguousarray(K[None, :, lo:hi]), np.ascontiguousarray(V[None, :, lo:hi]))
    return cache


@pytest.mark.parametrize("nccl", [False, True])
def test_split_group_world1(lc, orc, gpu, nccl):
    """A one-rank group: the split call equals lc_decode_attn."""
    import torch

    n = 3000
    cache = _shard_cache(lc, orc, n, 0, n, 0)
    g = lc.SplitGroup(1, 0, lc.SplitGroup.new_id(), HQ, DIM, device=0, nccl=nccl)
    q = helpers.queries(orc, 5, 1, HQ, DIM, std=DIM ** -0.5)
    qd = torch.from_numpy(q).cuda()
    want = cache.decode_attn(0, [0], q, HQ, 1.0)
    for _ in range(3):
        out = torch.empty((1, HQ, DIM), device="cuda")
        cache.decode_attn_split(g, 0, [0], qd, HQ, 1.0, out=out)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), want, rtol=0, atol=2e-5)
    assert g.status() == lc.LC_OK
    ok, msg = helpers.attn_close(want[0], _oracle(orc, n, q[0], 1.0))
    assert ok, msg
    g.close()
    cache.close()


def _worker(rank, world, port, n, nccl, fail, result_dir):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
    import helpers as hp
    import pyoracle as orc

    lc = importlib.import_module("lumen-rs_b200")
    split = importlib.import_module("lumen-rs_b200.split")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        lo, hi = split.shard_range(n, rank, world)
        cache = _shard_cache(lc, orc, n, lo, hi, rank)
        g = split.make_group(HQ, DIM, rank, nccl=nccl)
        dec = split.SplitSequenceDecoder(cache, 0, lc_group=g)
        q = torch.from_numpy(hp.queries(orc, 5, 1, HQ, DIM, std=DIM ** -0.5)).cuda()
        outs = []
        if fail and rank == 1:
            pass  # stays alive with its buffers mapped, but skips the call
        else:
            for _ in range(1 if fail else 3):
                out = dec.decode(0, q, HQ, 1.0)
                torch.cuda.synchronize()
                outs.append(out.cpu().numpy())
            np.save(os.path.join(result_dir, f"out{rank}.npy"), np.stack(outs))
            with open(os.path.join(result_dir, f"status{rank}.txt"), "w") as f:
                f.write(str(g.status()) + " " + str(int(g.info()["peer_stores"])))
        dist.barrier()  # every rank past its last call before any buffer is freed
        g.close()
        cache.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
@pytest.mark.parametrize("nccl", [False, True])
def test_split_group_two_gpus(lc, orc, gpu, tmp_path, nccl):
    import torch.multiprocessing as mp

    n = 5001
    mp.spawn(_worker, args=(2, _free_port(), n, nccl, False, str(tmp_path)), nprocs=2, join=True)
    q = helpers.queries(orc, 5, 1, HQ, DIM, std=DIM ** -0.5)[0]
    ref = _oracle(orc, n, q, 1.0)
    for r in range(2):
        st, p2p = (tmp_path / f"status{r}.txt").read_text().split()
        assert int(st) == lc.LC_OK
        assert p2p == ("0" if nccl else "1")
        outs = np.load(tmp_path / f"out{r}.npy")
        for k in range(outs.shape[0]):
            ok, msg = helpers.attn_close(outs[k], ref)
            assert ok, f"rank {r} call {k}: {msg}"


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_split_group_peer_failure_times_out(lc, orc, gpu, tmp_path):
    import time

    import torch.multiprocessing as mp

    t0 = time.time()
    mp.spawn(_worker, args=(2, _free_port(), 2000, False, True, str(tmp_path)), nprocs=2, join=True)
    st, _ = (tmp_path / "status0.txt").read_text().split()
    assert int(st) == lc.LC_ERR_TIMEOUT
    assert np.isnan(np.load(tmp_path / "out0.npy")).all()
    assert time.time() - t0 < 120
