"""The column-parallel FP8 linear on 2 GPUs (child processes, one GPU each, NCCL): the gathered output of the GEMM
whose epilogue stores each rank's columns into every rank's buffer equals the unsplit linear bit for bit, and so does
the NCCL all-gather baseline; rows on the few-rows and the many-rows kernel. Skipped with fewer than 2 GPUs."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import basal_b200 as b2
        from basal_b200 import shard
        dev = torch.device("cuda", rank)
        g = torch.Generator().manual_seed(3)
        N, K = 1280, 1024
        lin = torch.nn.Linear(K, N, bias=False)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
        full = b2.fp8block.BlockFP8Linear.of(lin.to(dev))
        m = shard.ColumnShardedFP8Linear(full, timeout_ms=20000)
        res = []
        for M in (16, 300, 37):
            x = torch.randn(M, K, generator=g).bfloat16().to(dev)
            want = full(x)
            got = m(x).clone()
            base = m.forward_nccl(x)
            res.append((M, torch.equal(got, want), torch.equal(base, want)))
        torch.cuda.synchronize()
        res.append(("faults", b2._lib.device_faults(rank)))
        out.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gathered_column_parallel_linear_equals_the_whole_linear():
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in procs), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, rows in res:
        assert rows[-1] == ("faults", 0)
        for M, fused_ok, nccl_ok in rows[:-1]:
            assert fused_ok, (rank, M)
            assert nccl_ok, (rank, M)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA")
def test_peer_barrier_gives_up_on_an_absent_rank():
    """The barrier's wait for a rank that never arrives (a second pad that nothing writes, local memory, one GPU) ends
    after its limit with the peer-timeout fault bit, and the context stays usable; a one-rank barrier passes. The
    timeout sets the pad's sticky status word, on this rank's pad and on the absent rank's."""
    import ctypes

    import basal_b200 as b2
    from basal_b200 import _lib
    b2._lib.device_faults(0)  # clear
    pads = [torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2)]
    arr = (ctypes.c_void_p * 2)(*[p.data_ptr() for p in pads])
    _lib.call("basal200_peer_barrier", torch.device("cuda", 0), arr, 1, 0, 50_000_000)
    assert b2._lib.device_faults(0) == 0
    assert int(pads[0][0]) == 1 and int(pads[0][8]) == 1  # its own arrival and call count
    assert int(pads[0][9]) == 0                           # status: fine
    _lib.call("basal200_peer_barrier", torch.device("cuda", 0), arr, 2, 0, 50_000_000)  # rank 1 never comes
    assert b2._lib.device_faults(0) == 32                                                  # BASAL200_FAULT_TIMEOUT_PEER
    assert int(pads[1][0]) == 2                         # it told the absent rank it arrived (call 2)
    assert int(pads[0][9]) == 1 and int(pads[1][9]) == 1  # the status, here and written to the peer
    y = torch.ones(4, device="cuda") * 2
    assert float(y.sum()) == 8.0


@pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA")
@pytest.mark.parametrize("M", [16, 300])
def test_gathered_gemm_stores_nothing_after_a_barrier_gave_up(M):
    """One GPU, two local output buffers standing for two ranks' outputs: with a clean barrier pad the gathered GEMM
    writes the linear's output into both (few-rows kernel at M = 16, the large-M kernel at M = 300); with the pad's
    status word set (a barrier that gave up), it stores nothing into either, on both kernels."""
    import ctypes

    import basal_b200 as b2
    from basal_b200 import _lib
    N, K = 384, 512
    g = torch.Generator().manual_seed(M)
    lin = torch.nn.Linear(K, N, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
    full = b2.fp8block.BlockFP8Linear.of(lin.cuda())
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    q, s = b2.ops.fp8_act_quant(x)
    want = full(x)
    sentinel = torch.full((M, N), 7.0, dtype=torch.bfloat16, device="cuda")
    for status in (0, 1):
        pad = torch.zeros(16, dtype=torch.int32, device="cuda")
        pad[9] = status
        outs = [sentinel.clone(), sentinel.clone()]
        arr = (ctypes.c_void_p * 2)(*[o.data_ptr() for o in outs])
        _lib.call("basal200_fp8_block_gemm_gather", x.device, q.data_ptr(), s.data_ptr(), full.weight.data_ptr(),
                  full.weight_scale.data_ptr(), arr, 2, 0, N, _lib.BF16, M, N, K, pad.data_ptr())
        torch.cuda.synchronize()
        for o in outs:
            assert torch.equal(o, sentinel if status else want), status
    assert b2._lib.device_faults(0) == 0
