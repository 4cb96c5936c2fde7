"""Row sharding of independent decision requests across the GPUs of one box (one process per GPU).

The reference serves several GPUs as independent replicas behind its router (basal/router.py:901-912): requests
never exchange data, so the hot path shards by rows with no collective. This module holds the host side of that:

  varlen_lengths(n, lo, hi, seed)   the seeded request lengths of a workload (torch.randint, inclusive hi)
  cu_seqlens(lengths)               packed-row offsets of varlen requests (the compact rows of engine.py:1469-1475)
  shard_range(n, world, rank)       the contiguous block of request indices rank `rank` serves
  max_over_ranks(x, group)          the slowest rank's time (all-reduce MAX), the bench's clock for N > 1
  sum_over_ranks(x, group)          the units all ranks processed
  check_peers(group, timeout_s)     a bounded barrier: a rank that died or never joined surfaces as an error on the
                                    others within timeout_s (gloo's monitored barrier; NCCL groups use a store key)
Everything here is host logic; the GPUs run only libbasal200's kernels on their own rows.
"""
import datetime

import torch
import torch.distributed as dist


def varlen_lengths(n, lo, hi, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=g)


def cu_seqlens(lengths):
    lengths = torch.as_tensor(lengths, dtype=torch.int64)
    return torch.cat([torch.zeros(1, dtype=torch.int64), lengths.cumsum(0)])


def shard_range(n, world, rank):
    """Requests [start, stop) of `rank` among `world` ranks: contiguous, sizes differing by at most one."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _reduce(x, op, group):
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return float(x)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=op, group=group)
    return float(t.item())


def max_over_ranks(x, group=None):
    return _reduce(x, dist.ReduceOp.MAX, group)


def sum_over_ranks(x, group=None):
    return _reduce(x, dist.ReduceOp.SUM, group)


def check_peers(group=None, timeout_s=30.0, tag="peers"):
    """Returns once every rank reached this point; raises RuntimeError naming the failure when a peer does not
    arrive within timeout_s. On gloo it is a monitored barrier; on NCCL every rank sets a store key and waits for the
    others' keys (no device work, so a dead peer cannot wedge a GPU)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return
    timeout = datetime.timedelta(seconds=timeout_s)
    if dist.get_backend(group) == "gloo":
        try:
            dist.monitored_barrier(group=group, timeout=timeout, wait_all_ranks=True)
        except RuntimeError as e:
            raise RuntimeError(f"check_peers({tag}): {e}") from e
        return
    store = dist.distributed_c10d._get_default_store()
    rank, world = dist.get_rank(), dist.get_world_size()
    store.set(f"{tag}/{rank}", "1")
    try:
        store.wait([f"{tag}/{r}" for r in range(world)], timeout)
    except Exception as e:  # the store raises its own timeout type
        raise RuntimeError(f"check_peers({tag}): a peer did not arrive within {timeout_s} s: {e}") from e
