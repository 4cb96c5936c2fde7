"""The multi-GPU host logic on CPU ranks (gloo, world size 2): row shards of independent requests cover every
request once, the bench's clock is the slowest rank's, units add up over ranks, and a rank that fails or never
arrives surfaces on its peer as an error within a short timeout (failure made on the host, no GPU involved)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from basal_b200 import shard


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))


def _worker_shards(rank, world, port, out):
    _init(rank, world, port)
    try:
        lengths = shard.varlen_lengths(64, 128, 2048, seed=0)
        start, stop = shard.shard_range(len(lengths), world, rank)
        rows = int(lengths[start:stop].sum())
        total = shard.sum_over_ranks(rows)
        slowest = shard.max_over_ranks(1.0 + rank)
        shard.check_peers(timeout_s=10, tag="t")
        out.put((rank, start, stop, rows, total, slowest))
    finally:
        dist.destroy_process_group()


def test_shards_cover_every_request_once_and_reduce():
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_shards, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lengths = shard.varlen_lengths(64, 128, 2048, seed=0)
    assert [(r[1], r[2]) for r in res] == [(0, 32), (32, 64)]
    assert sum(r[3] for r in res) == int(lengths.sum()) == res[0][4] == res[1][4]
    assert res[0][5] == res[1][5] == 2.0


def _worker_dies(rank, world, port, out):
    _init(rank, world, port)
    if rank == 1:
        os._exit(3)  # leaves between steps, without a word to its peer
    try:
        shard.check_peers(timeout_s=3, tag="dead")
        out.put("no error")
    except RuntimeError as e:
        out.put("error: " + str(e)[:200])


def test_a_dead_rank_surfaces_as_an_error_on_its_peer():
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_dies, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error"), msg


def test_shard_range_edges():
    assert shard.shard_range(5, 2, 0) == (0, 3) and shard.shard_range(5, 2, 1) == (3, 5)
    assert shard.shard_range(3, 8, 7) == (3, 3)
    with pytest.raises(ValueError):
        shard.shard_range(4, 2, 2)
    assert shard.cu_seqlens(torch.tensor([3, 2])).tolist() == [0, 3, 5]


def test_column_shards_are_whole_scale_blocks():
    assert [shard.column_shard(5120, 8, r) for r in (0, 7)] == [(0, 640), (4480, 5120)]
    assert shard.column_shard(19456, 8, 7) == (17024, 19456)                 # 152 blocks: 19 a rank
    assert [shard.column_shard(640, 4, r) for r in range(4)] == [(0, 256), (256, 384), (384, 512), (512, 640)]
    with pytest.raises(ValueError):
        shard.column_shard(200, 2, 0)


def _worker_column_module(rank, world, port, out):
    _init(rank, world, port)
    try:
        from basal_b200.fp8block import BlockFP8Linear
        N, K = 640, 256
        w = torch.arange(N * K, dtype=torch.float32).reshape(N, K).to(torch.float8_e4m3fn)
        s = torch.arange(N // 128 * K // 128, dtype=torch.float32).reshape(N // 128, K // 128)
        m = shard.ColumnShardedFP8Linear(BlockFP8Linear(w, s), timeout_ms=5000)
        start, stop = shard.column_shard(N, world, rank)
        ok = (m.col_off == start and m.shard.out_features == stop - start
              and torch.equal(m.shard.weight.view(torch.uint8), w[start:stop].view(torch.uint8))
              and torch.equal(m.shard.weight_scale, s[start // 128: stop // 128]))
        out.put((rank, ok, m.col_off, m.shard.out_features))
    finally:
        dist.destroy_process_group()


def test_column_sharded_linear_holds_its_rows_and_scale_blocks():
    """Host side of the column-parallel linear on gloo ranks: each rank keeps the views of its whole scale blocks."""
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_column_module, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == [(0, True, 0, 384), (1, True, 384, 256)]
