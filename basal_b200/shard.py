"""Row sharding of independent decision requests across the GPUs of one box (one process per GPU).

The reference serves several GPUs as independent replicas behind its router (basal/router.py:901-912): requests
never exchange data, so the hot path shards by rows with no collective. This module holds the host side of that:

  varlen_lengths(n, lo, hi, seed)   the seeded request lengths of a workload (torch.randint, inclusive hi)
  cu_seqlens(lengths)               packed-row offsets of varlen requests (the compact rows of engine.py:1470-1475)
  shard_range(n, world, rank)       the contiguous block of request indices rank `rank` serves
  max_over_ranks(x, group)          the slowest rank's time (all-reduce MAX), the bench's clock for N > 1
  sum_over_ranks(x, group)          the units all ranks processed
  check_peers(group, timeout_s)     a bounded barrier: a rank that died or never joined surfaces as an error on the
                                    others within timeout_s (gloo's monitored barrier; NCCL groups use a store key)
Everything above is host logic; the GPUs run only libbasal200's kernels on their own rows.

For a model too large for one GPU's share of rows, the weights can also be split by output rows (N) across the
ranks of a group that all serve the same rows (column parallelism, the tensor-parallel layout); every rank then needs
the whole output of each linear before the next operation:
  column_shard(n, world, rank)      the output rows a rank holds (whole 128-row scale blocks)
  ColumnShardedFP8Linear            an FP8-block linear split that way whose GEMM stores its columns straight into
                                    every rank's output (the all-gather done by the GEMM's epilogue over NVLink,
                                    peer-mapped symmetric memory), and the NCCL all-gather baseline beside it
"""
import ctypes
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


# ---------------------------------------------------------------------------------------------------------------
# column shards
# ---------------------------------------------------------------------------------------------------------------
MAX_PEERS = 8  # output buffers one gathered GEMM stores into (libbasal200's limit)
PAD_STATUS_WORD = 9  # BASAL200_PAD_STATUS_WORD: the sticky status word of a peer-barrier pad


def column_shard(n, world, rank, unit=128):
    """Output rows [start, stop) of `rank` when `n` rows are split across `world` ranks in whole `unit`-row blocks
    (a weight-scale block), contiguous, block counts differing by at most one."""
    if n % unit:
        raise ValueError(f"{n} output rows are not whole {unit}-row blocks")
    b0, b1 = shard_range(n // unit, world, rank)
    return b0 * unit, b1 * unit


class ColumnShardedFP8Linear(torch.nn.Module):
    """An FP8-block linear (basal_b200.fp8block.BlockFP8Linear) whose output rows are split across the ranks of
    `group`: each rank keeps its column shard (a part() view) and every rank's forward returns the whole output.

      forward(x)       act_quant, then one GEMM that stores this rank's columns into every rank's [M, N] output
                       buffer (peer-mapped symmetric memory: its stores cross NVLink tile by tile, no collective
                       kernel), between two barriers of the group (libbasal200's peer barrier on the buffers'
                       signal pads: before, every rank is done with the previous output; after, every rank's
                       columns have landed; a wait gives up after timeout_ms with a fault bit, never a trap). The
                       result is a view of the shared buffer, valid until the next forward of this module on any rank
                       (clone to keep it). It can be captured in a CUDA graph. Once a barrier has given up on any
                       rank, every rank's gathered GEMM stores nothing (a late rank must not overwrite a peer's
                       output), and check() raises.
      check()          synchronises the device and raises RuntimeError when a barrier of this module gave up on
                       this rank or a peer (the pad's sticky status word) or a bounded wait recorded a fault bit:
                       the outputs since the failure are not to be used.
      forward_nccl(x)  the baseline: the shard's own linear, an NCCL all-gather, the copy that interleaves the
                       ranks' columns.

    Each output element is computed exactly as the unsplit linear computes it (same kernel arithmetic, same K order),
    so both forwards equal BlockFP8Linear.forward bit for bit. Every rank runs the same forwards with the same rows
    (SPMD); bias is not supported (the gathered GEMM has none)."""

    def __init__(self, full, group=None, timeout_ms=10000):
        super().__init__()
        if full.bias is not None:
            raise ValueError("ColumnShardedFP8Linear: bias is not supported")
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > MAX_PEERS:
            raise ValueError(f"ColumnShardedFP8Linear: at most {MAX_PEERS} ranks, not {self.world}")
        self.out_features, self.in_features = full.out_features, full.in_features
        start, stop = column_shard(self.out_features, self.world, self.rank)
        if stop == start:
            raise ValueError(f"ColumnShardedFP8Linear: {self.out_features} rows leave rank {self.rank} none")
        self.col_off = start
        self.shard = full.part(start, stop - start)
        self.timeout_ms = int(timeout_ms)
        self._buf = None
        self._hdl = None
        self._outs = None  # the C array of every rank's buffer pointer
        self._pads = None  # the C array of every rank's signal pad pointer

    def _buffer(self, rows, dtype, device):
        """The [rows, N] symmetric output buffer of every rank (made, collectively, when it must grow)."""
        if self._buf is None or self._buf.shape[0] < rows or self._buf.dtype != dtype:
            import torch.distributed._symmetric_memory as symm_mem
            size = max(rows, 2 * self._buf.shape[0]) if self._buf is not None and self._buf.dtype == dtype else rows
            self._buf, self._hdl, self._outs, self._pads = None, None, None, None
            buf = symm_mem.empty((size, self.out_features), dtype=dtype, device=device)
            hdl = symm_mem.rendezvous(buf, self.group)
            off = buf.data_ptr() - hdl.buffer_ptrs[hdl.rank]  # the tensor's place in its allocation, alike everywhere
            self._outs = (ctypes.c_void_p * self.world)(*[p + off for p in hdl.buffer_ptrs])
            hdl.get_signal_pad(hdl.rank, (16,), dtype=torch.int32).zero_()  # the barrier's words, before any use
            torch.cuda.synchronize(device)
            check_peers(self.group, timeout_s=max(1.0, self.timeout_ms / 1000), tag="column-shard pads")
            self._pads = (ctypes.c_void_p * self.world)(*hdl.signal_pad_ptrs)
            self._buf, self._hdl = buf, hdl
        return self._buf, self._hdl

    def forward(self, x):
        from . import _lib, ops
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        M = x2.shape[0]
        if x.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("ColumnShardedFP8Linear: bf16 or fp16 activations")
        buf, hdl = self._buffer(M, x.dtype, x.device)
        q, s = ops.fp8_act_quant(x2)
        outs = self._outs
        w = self.shard
        tmo = self.timeout_ms * 1000000
        _lib.call("basal200_peer_barrier", x.device, self._pads, self.world, self.rank, tmo)
        _lib.call("basal200_fp8_block_gemm_gather", x.device, _lib.ptr(q), _lib.ptr(s), _lib.ptr(w.weight),
                  _lib.ptr(w.weight_scale), outs, self.world, self.col_off, self.out_features, _lib.code(x.dtype),
                  M, w.out_features, self.in_features, self._pads[self.rank])
        _lib.call("basal200_peer_barrier", x.device, self._pads, self.world, self.rank, tmo)
        return buf[:M].view(*shape[:-1], self.out_features)

    def check(self):
        """Raises RuntimeError when a peer barrier of this module gave up (on this rank or on a peer) or a bounded
        wait of a kernel on this device recorded a fault bit; synchronises the device (not for the hot path)."""
        from . import _lib
        if self._hdl is None:
            return
        dev = self._buf.device
        torch.cuda.synchronize(dev)
        status = int(self._hdl.get_signal_pad(self._hdl.rank, (16,), dtype=torch.int32)[PAD_STATUS_WORD].item())
        faults = _lib.device_faults(dev.index if dev.index is not None else 0, clear=False)
        if status or faults:
            raise RuntimeError(f"ColumnShardedFP8Linear (rank {self.rank}): a peer barrier gave up (status {status}, "
                               f"fault bits {faults}); the gathered outputs since then are incomplete")

    def forward_nccl(self, x):
        shape = x.shape
        y = self.shard(x.reshape(-1, shape[-1]))
        M, n = y.shape
        if all(column_shard(self.out_features, self.world, r)[1] - column_shard(self.out_features, self.world, r)[0]
               == n for r in range(self.world)):
            parts = torch.empty((self.world, M, n), dtype=y.dtype, device=y.device)
            dist.all_gather_into_tensor(parts, y, group=self.group)
            out = parts.permute(1, 0, 2).reshape(M, self.out_features)
        else:
            parts = [torch.empty((M, column_shard(self.out_features, self.world, r)[1]
                                  - column_shard(self.out_features, self.world, r)[0]), dtype=y.dtype, device=y.device)
                     for r in range(self.world)]
            dist.all_gather(parts, y, group=self.group)
            out = torch.cat(parts, 1)
        return out.view(*shape[:-1], self.out_features)
