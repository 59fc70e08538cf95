"""Row sharding across ranks (one process per GPU) and the optional gather of
sampled ids.  Rows are independent, so the data path has no collective: each
rank samples rows [begin, begin+count) of the global batch with per-row seeds
rng_seed + global_row, and ids only move when a caller asks for them on one
rank.  On GPUs the gather is NCCL (torch.distributed "nccl" or the library's
own ncclAllGather); on CPU ranks it is gloo.
"""
import torch.distributed as dist

from . import lib, shard_rows  # noqa: F401  (shard_rows calls the C-ABI)


def local_rows(batch, world, rank):
    return shard_rows(batch, world, rank)


def gather_ids(ids_local, batch, world, rank, group=None):
    """All-gathers the int32 id shards (uneven shards padded to the largest)
    and returns the full [batch] tensor on every rank."""
    import torch
    counts = [shard_rows(batch, world, r)[1] for r in range(world)]
    width = max(counts) if counts else 0
    buf = torch.full((width,), -1, dtype=torch.int32, device=ids_local.device)
    buf[: ids_local.numel()] = ids_local
    out = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(out, buf, group=group)
    return torch.cat([o[:c] for o, c in zip(out, counts)])
