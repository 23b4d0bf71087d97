"""One long context split by sequence across the ranks of a process group.

Decode requests that fit on one GPU are sharded by request, with no
collective. A single context too long for that (the 1,048,576-token
sequence of the benchmark's scale-out config) is split by tokens:

- Each rank holds one contiguous token range of the sequence in its own
  cache (`shard_range`).
- Each rank computes, for every query head, the softmax partials of its
  range: m is the log2-domain max, l the sum of 2^(s - m), and o the
  unnormalised rotated output (`lc_decode_attn_partials`).
- The ranks exchange the partials once per layer, rows * (head_dim + 2)
  f32 per rank. On GPUs the library does it (`lc_decode_attn_split` over an
  `lc_group`): each rank stores its partials straight into every peer's
  buffer over NVLink and raises a flag there, and every rank merges once
  all flags are up, all on the stream. Without a group (CPU tests, gloo),
  a torch.distributed all-gather stands in.
- Every rank merges them (`lc_merge_partials` / the group's merge), the
  combine of partial softmax states in lumen-mlx
  native_quant_attention.rs:190-207.

New tokens go to the rank holding the sequence's end (`owner_of_next`).
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple


def shard_range(n_tokens: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous token range [lo, hi) of `rank`: near-equal shares in rank
    order, the first n_tokens % world ranks holding one token more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if n_tokens < 0:
        raise ValueError("n_tokens must be >= 0")
    base, extra = divmod(n_tokens, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def head_shard(n_kv_heads: int, rank: int, world: int) -> Tuple[int, int]:
    """Kv heads [lo, hi) of `rank` when a model's kv heads are split over the
    ranks (each rank also takes those heads' query groups): attention of a
    query head reads only its kv head, so the shards need no communication.
    Near-equal contiguous shares, as shard_range."""
    return shard_range(n_kv_heads, rank, world)


def owner_of_next(world: int) -> int:
    """Rank that appends the sequence's new tokens: the one holding its end."""
    return world - 1


def make_group(max_rows: int, head_dim: int, device: int, pg=None, nccl: bool = False):
    """The library's exchange group (lc_group) for the ranks of torch.distributed
    process group `pg`: rank 0 makes the id, a broadcast carries it (plumbing
    only; the per-layer exchange never goes through torch)."""
    import importlib

    import torch.distributed as dist

    lc = importlib.import_module("lumen-rs_b200")
    world, rank = dist.get_world_size(pg), dist.get_rank(pg)
    box = [lc.SplitGroup.new_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=dist.get_global_rank(pg, 0) if pg is not None else 0, group=pg)
    return lc.SplitGroup(world, rank, box[0], max_rows, head_dim, device=device, nccl=nccl)


class SplitSequenceDecoder:
    """Decode attention for one sequence whose tokens are sharded over ranks.

    `cache` is this rank's cache, holding its token range of the sequence in
    slot `seq_id` (a `CudaKvCache`, or any object with the same
    `decode_partials` / `merge_partials` methods). `gather(x)` returns the
    [world, *x.shape] stack of x over the ranks in rank order. The default is
    torch.distributed's all_gather_into_tensor on `group` (world size 1 when
    no process group is initialised).
    """

    def __init__(self, cache, seq_id: int = 0, group=None, gather: Optional[Callable] = None, lc_group=None):
        self.cache = cache
        self.seq_id = seq_id
        self.group = group
        self.lc_group = lc_group  # a SplitGroup: the library exchanges and merges
        self._gather = gather or self._dist_gather

    def _dist_gather(self, x):
        import torch
        import torch.distributed as dist

        x = x.contiguous()
        if not dist.is_available() or not dist.is_initialized():
            return x.unsqueeze(0)  # a single process: the whole sequence is here
        world = dist.get_world_size(self.group)
        out = torch.empty((world * x.numel(),), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.view(-1), group=self.group)
        return out.view((world,) + tuple(x.shape))

    def decode(self, layer: int, q, n_q_heads: int, scale: float = 1.0, flags: int = 0, out=None,
               out_dtype: Optional[int] = None):
        """softmax(scale q K^T) V over the whole split sequence; q [1, n_q_heads,
        head_dim] on this rank's device. Returns out [n_q_heads, head_dim]."""
        import torch

        rows, d = n_q_heads, self.cache.head_dim
        dev = q.device if hasattr(q, "device") else None
        if self.lc_group is not None:
            if out is None:
                out = torch.empty((rows, d), dtype=torch.float32, device=dev)
                out_dtype = 0
            self.cache.decode_attn_split(self.lc_group, layer, [self.seq_id], q, n_q_heads, scale, flags, out=out,
                                         out_dtype=0 if out_dtype is None else out_dtype)
            return out
        # one buffer [m | l | o] per rank, so one collective moves all three
        buf = torch.empty(rows * (d + 2), dtype=torch.float32, device=dev)
        m, l, o = buf[:rows], buf[rows:2 * rows], buf[2 * rows:].view(rows, d)
        self.cache.decode_partials(layer, [self.seq_id], q, n_q_heads, scale, flags, m=m, l=l, o=o)
        g = self._gather(buf)  # [world, rows * (d + 2)]
        gm = g[:, :rows].contiguous()
        gl = g[:, rows:2 * rows].contiguous()
        go = g[:, 2 * rows:].contiguous().view(g.shape[0], rows, d)
        kw = {} if out_dtype is None else {"out_dtype": out_dtype}
        if out is None:
            out = torch.empty((rows, d), dtype=torch.float32, device=dev)
            kw["out_dtype"] = 0
        return self.cache.merge_partials(gm, gl, go, flags, out=out, **kw)
