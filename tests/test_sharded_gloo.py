"""Host logic of the row-sharded multi-GPU GEMM on CPU ranks (gloo, world size 2
and 3): row plans, the B broadcast (blocking, or pipelined one step ahead on its
own communicator) and the chunked all-gather / gather-to-root exchange, with an
FP32 torch product standing in for the GPU kernel."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sharded import BroadcastPipeline, ShardPlan, chunk_rows, pipelined_step, shard_rows, sharded_step


def test_shard_rows_partition_every_row_once():
    for m in (1, 7, 8, 37, 32768):
        for world in (1, 2, 3, 8):
            ranges = [shard_rows(m, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == m
            for (s0, e0), (s1, e1) in zip(ranges, ranges[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_rows(8, 2, 2)


def test_chunk_rows():
    assert chunk_rows(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert chunk_rows(2, 4) == [(0, 1), (1, 2)]
    assert chunk_rows(0, 4) == []


@pytest.mark.parametrize("m,chunks,tail", [(8192, 8, 2), (8192, 8, 4), (1000, 3, 4), (5, 8, 3), (3, 1, 5),
                                            (1000, 4, 1)])
def test_end_to_end_row_blocks(m, chunks, tail):
    """end_to_end.HostMatmul's row blocks: contiguous, non-empty, covering [0, m), the
    last of the ``chunks`` blocks split again (the 8192-row, 8-block, 2-way split
    that the end-to-end benchmark uses gives two 512-row tail blocks)."""
    from end_to_end import row_blocks

    blocks = row_blocks(m, chunks, tail)
    assert blocks[0][0] == 0 and blocks[-1][1] == m
    assert all(lo < hi for lo, hi in blocks)
    assert all(blocks[i][1] == blocks[i + 1][0] for i in range(len(blocks) - 1))
    base = min(chunks, m)
    last = m - chunk_rows(m, chunks)[-1][0]
    assert len(blocks) == base - 1 + min(tail, last)
    if (m, chunks, tail) == (8192, 8, 2):
        assert blocks[-2:] == [(7168, 7680), (7680, 8192)]


def test_plan_peers():
    plan = ShardPlan(64, 8, 8, 4, 2, chunks=2, gather="all")
    assert plan.receivers() == [0, 1, 3] and plan.senders() == [0, 1, 3]
    root = ShardPlan(64, 8, 8, 4, 0, chunks=2, gather="root")
    assert root.receivers() == [] and root.senders() == [1, 2, 3]
    leaf = ShardPlan(64, 8, 8, 4, 3, chunks=2, gather="root")
    assert leaf.receivers() == [0] and leaf.senders() == []
    assert plan.global_chunk(1, 1) == (24, 32)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_gemm(a_rows, b, c_rows):
    torch.matmul(a_rows, b, out=c_rows)


def _worker(rank, world, port, m, k, n, chunks, gather, results, pipelined=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if pipelined:
            _pipelined(rank, world, m, k, n, chunks, gather, results)
            return
        torch.manual_seed(0)
        a_full = torch.randn(m, k)
        b_full = torch.randn(k, n)
        plan = ShardPlan(m, k, n, world, rank, chunks=chunks, gather=gather)
        start, stop = plan.local_rows
        a_local = a_full[start:stop].clone()
        b = b_full.clone() if rank == 0 else torch.zeros(k, n)
        c = torch.full((m, n), float("nan"))
        for _ in range(2):
            sharded_step(plan, a_local, b, c, _cpu_gemm)
        expected = a_full @ b_full
        if gather == "all" or rank == 0:
            ok = torch.allclose(c, expected, rtol=1e-5, atol=1e-4)
        else:
            ok = torch.allclose(c[start:stop], expected[start:stop], rtol=1e-5, atol=1e-4)
        ok = ok and torch.equal(b, b_full)
        results[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def _pipelined(rank, world, m, k, n, chunks, gather, results):
    """Three steps whose B changes every step: step s must compute with B_s."""
    b_group = dist.new_group(list(range(world)))
    torch.manual_seed(0)
    a_full = torch.randn(m, k)
    bs = [torch.randn(k, n) for _ in range(4)]
    plan = ShardPlan(m, k, n, world, rank, chunks=chunks, gather=gather)
    start, stop = plan.local_rows
    a_local = a_full[start:stop].clone()
    b0 = bs[0].clone() if rank == 0 else torch.zeros(k, n)
    dist.broadcast(b0, src=0)                        # B of the first step, before the loop
    pipe = BroadcastPipeline(b0, b_group)
    ok = True
    for step in range(3):
        if rank == 0:
            pipe.pending.copy_(bs[step + 1])         # rank 0 supplies the next step's B
        c = torch.full((m, n), float("nan"))
        pipelined_step(plan, a_local, pipe, c, _cpu_gemm)
        expected = a_full @ bs[step]
        rows = slice(None) if gather == "all" or rank == 0 else slice(start, stop)
        ok = ok and torch.allclose(c[rows], expected[rows], rtol=1e-5, atol=1e-4)
        ok = ok and torch.equal(pipe.current, bs[step + 1])
    results[rank] = bool(ok)


@pytest.mark.parametrize("world,m,chunks,gather,pipelined", [
    (2, 64, 4, "all", False), (2, 37, 3, "all", False), (3, 50, 2, "root", False), (2, 5, 8, "root", False),
    (2, 64, 4, "all", True), (3, 50, 2, "root", True)])
def test_row_sharded_gemm_on_gloo_ranks(world, m, chunks, gather, pipelined):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, 24, 40, chunks, gather, results, pipelined))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert dict(results) == {r: True for r in range(world)}


class _FakeStream:
    def wait_event(self, event):
        pass


class _FakeHandle:
    """Stands in for a symmetric-memory handle: rank p's buffer is ``buffers[p]``."""

    def __init__(self, buffers):
        self.buffers = buffers

    def get_buffer(self, peer, shape, dtype):
        buffer = self.buffers[peer]
        assert tuple(buffer.shape) == tuple(shape) and buffer.dtype == dtype
        return buffer


def _memmove_copy(dst, src, nbytes, stream):
    import ctypes

    ctypes.memmove(dst, src, nbytes)


@pytest.mark.parametrize("streams", (1, 3))
@pytest.mark.parametrize("world,m,chunks,gather", [(2, 37, 3, "all"), (3, 64, 4, "all"), (4, 9, 8, "all"),
                                                   (3, 50, 2, "root"), (8, 100, 3, "all")])
def test_copy_engine_gather_places_every_chunk(world, m, chunks, gather, streams):
    """CopyEngineGather's row arithmetic: after every rank has posted every chunk,
    each receiver's C holds every sender's rows at the right place (all ranks in one
    process, host buffers standing in for the peers' mapped C, memmove for the copy)."""
    from sharded import CopyEngineGather

    n = 5
    expected = torch.arange(m * n, dtype=torch.float32).reshape(m, n)
    buffers = []
    plans = [ShardPlan(m, 3, n, world, r, chunks=chunks, gather=gather) for r in range(world)]
    for r, plan in enumerate(plans):
        c = torch.full((m, n), -1.0)
        lo, hi = plan.local_rows
        c[lo:hi] = expected[lo:hi]
        buffers.append(c)
    handle = _FakeHandle(buffers)
    gathers = [CopyEngineGather(plan, buffers[r], group=object(), handle=handle, copy=_memmove_copy,
                                new_stream=_FakeStream, streams=streams) for r, plan in enumerate(plans)]
    for r, g in enumerate(gathers):
        # Peers in the order rank+1, rank+2, ... so that every rank sends to a different peer at a time.
        assert g.order == [p for p in ((r + d) % world for d in range(1, world)) if p in plans[r].receivers()]
        assert len(g.streams) == (min(streams, len(g.order)) if g.order else 0)
    for index in range(plans[0].chunk_count):
        for g in gathers:
            g.post(index, event=None)
    for r in range(world):
        if gather == "all" or r == 0:
            assert torch.equal(buffers[r], expected), r
        else:
            lo, hi = plans[r].local_rows
            assert torch.equal(buffers[r][lo:hi], expected[lo:hi])
            outside = torch.ones(m, dtype=torch.bool)
            outside[lo:hi] = False
            assert torch.all(buffers[r][outside] == -1.0)


@pytest.mark.parametrize("world,m,chunks,gather", [(2, 37, 3, "all"), (4, 9, 8, "all"), (3, 50, 2, "root"),
                                                   (8, 100, 3, "all")])
def test_kernel_push_gather_places_every_chunk(world, m, chunks, gather):
    """KernelPushGather's addresses: each post hands the push function this rank's
    chunk and the matching rows of every receiver's C (memmove standing in for the
    push kernel, all ranks in one process)."""
    import ctypes

    from sharded import KernelPushGather

    n = 6
    expected = torch.arange(m * n, dtype=torch.float32).reshape(m, n)
    plans = [ShardPlan(m, 3, n, world, r, chunks=chunks, gather=gather) for r in range(world)]
    buffers = []
    for plan in plans:
        c = torch.full((m, n), -1.0)
        lo, hi = plan.local_rows
        c[lo:hi] = expected[lo:hi]
        buffers.append(c)
    handle = _FakeHandle(buffers)
    calls = []

    def push(src, dsts, nbytes, stream, ctas):
        calls.append(len(dsts))
        for dst in dsts:
            ctypes.memmove(dst, src, nbytes)

    gathers = [KernelPushGather(plan, buffers[r], push, group=object(), handle=handle, new_stream=_FakeStream)
               for r, plan in enumerate(plans)]
    for index in range(plans[0].chunk_count):
        for g in gathers:
            g.post(index, event=None)
    for r in range(world):
        if gather == "all" or r == 0:
            assert torch.equal(buffers[r], expected), r
    assert max(calls) == (world - 1 if gather == "all" else 1)


@pytest.mark.parametrize("world,k", [(2, 7), (3, 10), (4, 9), (8, 100), (8, 5)])
def test_copy_engine_broadcast_delivers_b_to_every_rank(world, k):
    """CopyEngineBroadcast's two phases: after rank 0's scatter and every owner's
    forward, each rank's pending buffer holds rank 0's B, rank 0 sent each row of B
    exactly once, and the current buffers are untouched (all ranks in one process,
    host buffers standing in for the peers' mapped buffers, memmove for the copy)."""
    import ctypes

    from sharded import CopyEngineBroadcast, broadcast_parts

    n = 3
    b_next = torch.arange(k * n, dtype=torch.float32).reshape(k, n)
    currents = [torch.full((k, n), 7.0) for _ in range(world)]
    pendings = [b_next.clone() if r == 0 else torch.full((k, n), -1.0) for r in range(world)]
    sent = [0] * world

    def copier(rank):
        def copy(dst, src, nbytes, stream):
            sent[rank] += nbytes
            ctypes.memmove(dst, src, nbytes)
        return copy

    handles = [_FakeHandle(currents), _FakeHandle(pendings)]
    pipes = [CopyEngineBroadcast(currents[r], pendings[r], object(), handles, copy=copier(r),
                                 new_stream=_FakeStream, world=world, rank=r) for r in range(world)]
    parts = broadcast_parts(k, world)
    assert parts[0][0] == 0 and parts[-1][1] == k and len(parts) == min(world - 1, k)
    for pipe in pipes:
        pipe.scatter()
    for pipe in pipes:
        pipe.forward()
    for r in range(world):
        assert torch.equal(pendings[r], b_next), r
        assert torch.all(currents[r] == 7.0)
    assert sent[0] == k * n * 4


@pytest.mark.parametrize("world", [2, 3, 8])
def test_copy_engine_broadcast_alternates_buffers_over_steps(world):
    """Three steps, each with a different B on rank 0: after every step's pushes and
    swap, every rank computes with that step's B, and the buffer the pushes wrote
    was never the one a rank was computing with during the step."""
    import ctypes

    from sharded import CopyEngineBroadcast

    k, n = 11, 3
    first = [torch.full((k, n), 1.0) for _ in range(world)]
    second = [torch.full((k, n), -1.0) for _ in range(world)]
    handles = [_FakeHandle(first), _FakeHandle(second)]
    pipes = [CopyEngineBroadcast(first[r], second[r], object(), handles, copy=_memmove_copy,
                                 new_stream=_FakeStream, world=world, rank=r) for r in range(world)]
    for step in range(3):
        b_next = torch.arange(k * n, dtype=torch.float32).reshape(k, n) + 100.0 * (step + 1)
        pipes[0].pending.copy_(b_next)                 # rank 0: the next step's B
        in_use = [pipe.current.clone() for pipe in pipes]
        for pipe in pipes:
            pipe.scatter()
        for pipe in pipes:
            pipe.forward()
        for r, pipe in enumerate(pipes):
            assert torch.equal(pipe.current, in_use[r]), (step, r)   # not written while computed with
            pipe.swap()
            assert torch.equal(pipe.current, b_next), (step, r)
            assert pipe.pending.data_ptr() != pipe.current.data_ptr()
