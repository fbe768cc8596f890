"""Row-sharded multi-GPU GEMM: C = A * B over P ranks of one node.

The reference is single-device (src/benchmark_backends.py selects one
``--device``); this module is the multi-GPU layer of the B200 backend:

* rank r owns rows ``shard_rows(M, P, r)`` of A and C (contiguous row blocks);
* B (K x N) lives on rank 0 and is broadcast to every rank over NVLink;
* each rank computes its C rows with the library's tcgen05 GEMM, one row
  chunk at a time, and every finished chunk is exchanged with grouped
  point-to-point transfers straight into each peer's full C (all-gather) or
  into rank 0's C only (gather to root), so the exchange of chunk i overlaps
  the GEMM of chunk i+1.  No kernel reads peer memory;
* the B broadcast runs one step ahead (double-buffered B), so it too overlaps
  the GEMMs.  ``CopyEngineBroadcast`` does it with copy-engine pushes over
  symmetric memory (rank 0 scatters B's parts, their owners forward them), so
  only two one-element all-reduces per step need an SM; ``BroadcastPipeline``
  does it with NCCL on its own communicator, whose kernels need SMs for the
  whole transfer.  Either way the GEMMs are launched on fewer SMs than the
  device has (``matmul_set_sm_limit``) so that the communication kernels find
  free SMs while they run;
* with ``CopyEngineGather`` the C exchange takes no SM at all: C lives in
  symmetric memory (every rank maps every peer's C), and each finished chunk
  is pushed into the peers' C by copy-engine transfers (one cudaMemcpyAsync per
  peer, peers visited in the order rank + 1, rank + 2, ... on one copy stream by
  default); a one-element NCCL all-reduce at the end of the step completes only
  when every rank's pushes are done, which makes the gathered C safe to read.

Collectives are issued through ``torch.distributed`` (one process per GPU);
the host-side plan (row ranges, chunking, peer lists) is independent of the
backend and is tested with ``gloo`` ranks on CPU.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


def shard_rows(m: int, world: int, rank: int) -> tuple[int, int]:
    """Row range [start, stop) of rank ``rank``: contiguous, sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(m, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def chunk_rows(rows: int, chunks: int) -> list[tuple[int, int]]:
    """Split ``rows`` local rows into at most ``chunks`` non-empty contiguous ranges."""
    chunks = max(1, min(chunks, rows)) if rows > 0 else 0
    return [shard_rows(rows, chunks, i) for i in range(chunks)]


@dataclass
class ShardPlan:
    m: int
    k: int
    n: int
    world: int
    rank: int
    chunks: int
    gather: str = "all"           # "all": every rank gets C; "root": rank 0 gets C

    def __post_init__(self):
        if self.gather not in ("all", "root"):
            raise ValueError("gather must be 'all' or 'root'")
        self.rows = [shard_rows(self.m, self.world, r) for r in range(self.world)]
        # Every rank splits its rows into the same number of chunks so that chunk i
        # is exchanged in the same grouped call on every rank.
        min_rows = min(stop - start for start, stop in self.rows)
        self.chunk_count = max(1, min(self.chunks, min_rows)) if min_rows > 0 else 1
        self.chunk_ranges = [chunk_rows(stop - start, self.chunk_count) for start, stop in self.rows]

    @property
    def local_rows(self) -> tuple[int, int]:
        return self.rows[self.rank]

    def global_chunk(self, owner: int, index: int) -> tuple[int, int]:
        """Global row range of chunk ``index`` of rank ``owner``."""
        start = self.rows[owner][0]
        lo, hi = self.chunk_ranges[owner][index]
        return start + lo, start + hi

    def receivers(self) -> list[int]:
        if self.gather == "all":
            return [r for r in range(self.world) if r != self.rank]
        return [0] if self.rank != 0 else []

    def senders(self) -> list[int]:
        if self.gather == "all":
            return [r for r in range(self.world) if r != self.rank]
        return [r for r in range(1, self.world)] if self.rank == 0 else []


def exchange_chunk(plan: ShardPlan, index: int, c_full: torch.Tensor, group=None):
    """Post the grouped sends/receives of chunk ``index``; returns the works (or [])."""
    ops = []
    lo, hi = plan.global_chunk(plan.rank, index)
    mine = c_full[lo:hi]
    for peer in plan.receivers():
        ops.append(dist.P2POp(dist.isend, mine, peer, group=group))
    for peer in plan.senders():
        plo, phi = plan.global_chunk(peer, index)
        ops.append(dist.P2POp(dist.irecv, c_full[plo:phi], peer, group=group))
    if not ops:
        return []
    return dist.batch_isend_irecv(ops)


def sharded_step(plan: ShardPlan, a_local: torch.Tensor, b: torch.Tensor, c_full: torch.Tensor,
                 gemm: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], None], group=None,
                 broadcast_b: bool = True) -> None:
    """One row-sharded GEMM: broadcast B, then per chunk GEMM + exchange.

    ``gemm(a_rows, b, c_rows)`` writes ``c_rows = a_rows @ b`` on the current
    stream.  ``c_full`` is the full M x N output (on rank 0 only needed for
    gather="root"; other ranks may pass their full buffer or just their rows
    as long as ``c_full[global rows]`` addresses them).
    """
    if broadcast_b and plan.world > 1:
        dist.broadcast(b, src=0, group=group)
    start, _ = plan.local_rows
    works = []
    for index, (lo, hi) in enumerate(plan.chunk_ranges[plan.rank]):
        gemm(a_local[lo:hi], b, c_full[start + lo:start + hi])
        if plan.world > 1:
            works.extend(exchange_chunk(plan, index, c_full, group))
    for work in works:
        work.wait()



class BroadcastPipeline:
    """Double-buffered B whose broadcast for the next step overlaps this step's work.

    ``current`` holds the B every rank computes with now; ``start()`` broadcasts
    rank 0's ``pending`` buffer (the next step's B) into every rank's ``pending``
    on the communicator ``group`` without blocking the compute stream, and
    ``finish()`` makes the current stream wait for it and swaps the buffers.
    Every step still moves one full B from rank 0 to all ranks.
    """

    def __init__(self, b: torch.Tensor, group=None):
        self.current = b
        self.pending = b.clone()          # rank 0: the next step's B (the same matrix here)
        self.group = group
        self.work = None

    def start(self) -> None:
        if self.work is not None:
            raise RuntimeError("broadcast already in flight")
        self.work = dist.broadcast(self.pending, src=0, group=self.group, async_op=True)

    def join(self, stream=None) -> None:
        """Make ``stream`` (default: the current one) wait for the broadcast in flight."""
        if self.work is None:
            raise RuntimeError("no broadcast in flight")
        with torch.cuda.stream(stream or torch.cuda.current_stream(self.current.device)):
            self.work.wait()

    def finish(self) -> None:
        if self.work is None:
            raise RuntimeError("no broadcast in flight")
        self.work.wait()
        self.work = None
        self.current, self.pending = self.pending, self.current


def broadcast_parts(k: int, world: int) -> list[tuple[int, int]]:
    """Row ranges of B's parts for ``CopyEngineBroadcast``: part j (rows of B, in
    order) belongs to rank j + 1; rank 0 holds B and owns none."""
    return chunk_rows(k, world - 1) if world > 1 else []


class CopyEngineBroadcast:
    """``BroadcastPipeline`` with the transfers done by copy engines instead of NCCL kernels.

    ``current`` and ``pending`` must come from
    ``torch.distributed._symmetric_memory.empty`` on every rank (same shape), with
    their rendezvous handles.  ``start()`` sends rank 0's ``pending`` (the next
    step's B) to every rank in two phases on a side stream, taking no SM:

    1. rank 0 pushes part j of B (``broadcast_parts``) into rank j + 1's
       ``pending`` only, so each row of B leaves rank 0 once;
    2. after a one-element all-reduce on ``group`` (every part has landed), each
       rank j + 1 pushes its part into every other rank's ``pending``.

    ``finish()`` makes the current stream wait for this rank's pushes, runs a
    second one-element all-reduce (every rank's pushes are done, so every
    ``pending`` is whole) and swaps the buffers.  Rank 0 egresses one B, every
    other rank receives one B, and no kernel runs on the SMs the GEMM uses apart
    from the two small all-reduces.
    """

    def __init__(self, current: torch.Tensor, pending: torch.Tensor, group, handles, *, copy=None,
                 new_stream=None, world: int | None = None, rank: int | None = None):
        self.current, self.pending = current, pending
        self.group = group
        self.world = dist.get_world_size(group) if world is None else world
        self.rank = dist.get_rank(group) if rank is None else rank
        self.copy = copy if copy is not None else _memcpy_d2d
        shape, dtype = tuple(current.shape), current.dtype
        # handles[i] is the rendezvous handle of buffer i (0: the initial current, 1: the initial pending).
        self.peer_views = [{peer: handle.get_buffer(peer, shape, dtype) for peer in range(self.world)
                            if peer != self.rank} for handle in handles]
        self.local = [current, pending]
        self.which = 1                    # index of the buffer that is pending now
        self.row_bytes = current.shape[1] * current.element_size()
        self.parts = broadcast_parts(current.shape[0], self.world)
        self.stream = (new_stream or (lambda: torch.cuda.Stream(device=current.device)))()
        self.token = torch.zeros(1, dtype=torch.float32, device=current.device)
        self.in_flight = False

    def _push(self, part: int, peers) -> None:
        lo, hi = self.parts[part]
        if hi <= lo:
            return
        src = self.local[self.which].data_ptr() + lo * self.row_bytes
        for peer in peers:
            dst = self.peer_views[self.which][peer].data_ptr() + lo * self.row_bytes
            self.copy(dst, src, (hi - lo) * self.row_bytes, self.stream)

    def scatter(self) -> None:
        """Phase 1 (rank 0): part j of the pending B into rank j + 1's pending buffer."""
        if self.rank == 0:
            for part in range(len(self.parts)):
                self._push(part, [part + 1])

    def forward(self) -> None:
        """Phase 2 (rank j + 1): part j into every other rank's pending buffer but rank 0's,
        peers in the order rank + 1, rank + 2, ..."""
        if 0 < self.rank <= len(self.parts):       # B with fewer rows than ranks leaves some without a part
            order = [(self.rank + d) % self.world for d in range(1, self.world)]
            self._push(self.rank - 1, [peer for peer in order if peer != 0])

    def start(self) -> None:
        if self.in_flight:
            raise RuntimeError("broadcast already in flight")
        self.in_flight = True
        if self.world < 2:
            return
        # The pending buffer is free on every rank: the previous step ended with an
        # all-reduce that followed every rank's GEMMs.
        self.stream.wait_stream(torch.cuda.current_stream(self.current.device))
        with torch.cuda.stream(self.stream):
            self.scatter()
            dist.all_reduce(self.token, group=self.group)
            self.forward()

    def join(self, stream=None) -> None:
        """Make ``stream`` (default: the current one) wait for this rank's pushes."""
        (stream or torch.cuda.current_stream(self.current.device)).wait_stream(self.stream)

    def finish(self) -> None:
        if not self.in_flight:
            raise RuntimeError("no broadcast in flight")
        self.in_flight = False
        if self.world > 1:
            self.join()
            dist.all_reduce(self.token, group=self.group)
        self.swap()

    def swap(self) -> None:
        """The buffer just filled becomes ``current``; the one computed with until
        now becomes ``pending`` (and its peers' mappings the target of the next
        pushes).  ``finish`` calls it once every rank's pushes are done."""
        self.which ^= 1
        self.current, self.pending = self.local[self.which ^ 1], self.local[self.which]


def pipelined_step(plan: ShardPlan, a_local: torch.Tensor, pipe: BroadcastPipeline, c_full: torch.Tensor,
                   gemm: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], None], group=None) -> None:
    """``sharded_step`` with the B broadcast for the next step overlapping this one.

    Every rank posts the broadcast of the next B, runs its chunked GEMMs on the
    current B with the C exchange of each chunk, and ends the step when both the
    exchanges and the broadcast are complete.
    """
    if plan.world > 1:
        pipe.start()
    start, _ = plan.local_rows
    works = []
    for index, (lo, hi) in enumerate(plan.chunk_ranges[plan.rank]):
        gemm(a_local[lo:hi], pipe.current, c_full[start + lo:start + hi])
        if plan.world > 1:
            works.extend(exchange_chunk(plan, index, c_full, group))
    for work in works:
        work.wait()
    if plan.world > 1:
        pipe.finish()


def _memcpy_d2d(dst: int, src: int, nbytes: int, stream) -> None:
    """One device-to-device cudaMemcpyAsync (a copy-engine transfer; across GPUs
    over NVLink when ``dst`` maps a peer's memory).  Raw pointers, no kernel."""
    from cuda.bindings import runtime as cudart

    (err,) = cudart.cudaMemcpyAsync(dst, src, nbytes, cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice,
                                    stream.cuda_stream)
    if err != cudart.cudaError_t.cudaSuccess:
        raise RuntimeError(f"cudaMemcpyAsync failed: {err}")


class CopyEngineGather:
    """C exchange of a row-sharded GEMM by copy-engine pushes into the peers' C.

    ``c_full`` must come from ``torch.distributed._symmetric_memory.empty`` on
    every rank (same shape).  ``post(index, event)`` pushes this rank's chunk
    ``index`` to every receiver of the plan once ``event`` (recorded after that
    chunk's GEMM) has completed; ``finish()`` makes the current stream wait for
    this rank's pushes and runs a one-element all-reduce that completes only when
    every rank's pushes are done.  Every rank calls ``finish()`` once per step.

    The receivers are visited in the order rank + 1, rank + 2, ... (mod world)
    and spread round-robin over ``streams`` copy streams: with one stream each
    rank sends to one peer at a time and, since every rank walks the same
    offsets, each rank also receives from about one peer at a time.  Copies to
    all peers at once (one stream per peer) measured about 400 GB/s of ingress
    per GPU at 8 GPUs, against 733 GB/s for a single peer-to-peer flow.
    """

    def __init__(self, plan: ShardPlan, c_full: torch.Tensor, group=None, handle=None, *, copy=None,
                 new_stream=None, streams: int = 1):
        self.plan = plan
        self.c_full = c_full
        self.group = group if group is not None else dist.group.WORLD
        if handle is None:
            import torch.distributed._symmetric_memory as symm_mem

            handle = symm_mem.rendezvous(c_full, self.group)
        self.handle = handle
        self.copy = copy if copy is not None else _memcpy_d2d
        if new_stream is None:
            new_stream = lambda: torch.cuda.Stream(device=c_full.device)  # noqa: E731
        shape, dtype = tuple(c_full.shape), c_full.dtype
        world, rank = plan.world, plan.rank
        receivers = set(plan.receivers())
        self.order = [(rank + d) % world for d in range(1, world) if (rank + d) % world in receivers]
        self.peer_c = {peer: self.handle.get_buffer(peer, shape, dtype) for peer in self.order}
        count = max(1, min(streams, len(self.order))) if self.order else 0
        self.streams = [new_stream() for _ in range(count)]
        self.token = torch.zeros(1, dtype=torch.float32, device=c_full.device)
        self.row_bytes = c_full.shape[1] * c_full.element_size()

    def post(self, index: int, event) -> None:
        lo, hi = self.plan.global_chunk(self.plan.rank, index)
        if hi <= lo:
            return
        src = self.c_full.data_ptr() + lo * self.row_bytes
        for stream in self.streams:
            stream.wait_event(event)
        for i, peer in enumerate(self.order):
            self.copy(self.peer_c[peer].data_ptr() + lo * self.row_bytes, src, (hi - lo) * self.row_bytes,
                      self.streams[i % len(self.streams)])

    def finish(self) -> None:
        current = torch.cuda.current_stream(self.c_full.device)
        for stream in self.streams:
            current.wait_stream(stream)
        dist.all_reduce(self.token, group=self.group)


def _timing_event(stream=None):
    event = torch.cuda.Event(enable_timing=True)
    event.record(stream)
    return event


def pipelined_step_ce(plan: ShardPlan, a_local: torch.Tensor, pipe: BroadcastPipeline, gather,
                      gemm: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], None],
                      marks: list | None = None) -> None:
    """``pipelined_step`` with the C exchange of ``gather`` (``CopyEngineGather`` or
    ``KernelPushGather``): each chunk is posted as soon as its GEMM is enqueued.

    With ``marks`` (a list), timing events are appended as (name, event) pairs:
    "start", "gemm<i>" after chunk i's GEMM, "exchange" when this rank's pushes
    are done, "broadcast" when ``pipe.join`` returns (NCCL: the next B has
    arrived here; ``CopyEngineBroadcast``: this rank's pushes of it are done, so
    the B is whole everywhere at the latest of these over the ranks), "end"
    after the step.
    """
    if marks is not None:
        marks.append(("start", _timing_event()))
    if plan.world > 1:
        pipe.start()
        if marks is not None:
            side = torch.cuda.Stream(device=a_local.device)
            pipe.join(side)
            marks.append(("broadcast", _timing_event(side)))
    start, _ = plan.local_rows
    c_full = gather.c_full
    for index, (lo, hi) in enumerate(plan.chunk_ranges[plan.rank]):
        gemm(a_local[lo:hi], pipe.current, c_full[start + lo:start + hi])
        if plan.world > 1:
            event = torch.cuda.Event(enable_timing=marks is not None)
            event.record()
            gather.post(index, event)
            if marks is not None:
                marks.append((f"gemm{index}", event))
    if plan.world > 1:
        if marks is not None:
            side = torch.cuda.Stream(device=a_local.device)
            for stream in getattr(gather, "streams", []) + ([gather.stream] if hasattr(gather, "stream") else []):
                side.wait_stream(stream)
            marks.append(("exchange", _timing_event(side)))
        gather.finish()
        pipe.finish()
    if marks is not None:
        marks.append(("end", _timing_event()))


class KernelPushGather:
    """C exchange of a row-sharded GEMM by this library's push kernel (``matmul_peer_push``).

    The same contract as ``CopyEngineGather``: ``c_full`` comes from
    ``torch.distributed._symmetric_memory.empty`` on every rank; ``post(index,
    event)`` sends chunk ``index`` to every receiver once ``event`` has completed,
    here as one kernel launch on a side stream that stores the rows into all the
    receivers' C over NVLink; ``finish()`` joins the side stream and runs the
    one-element all-reduce that completes when every rank's pushes are done.  The
    kernel runs on SMs the GEMM leaves free (``matmul_set_sm_limit``).
    """

    def __init__(self, plan: ShardPlan, c_full: torch.Tensor, push, group=None, handle=None, *, ctas: int = 0,
                 new_stream=None):
        self.plan = plan
        self.c_full = c_full
        self.push = push            # push(src_ptr, [dst_ptr, ...], nbytes, stream, ctas)
        self.ctas = ctas
        self.group = group if group is not None else dist.group.WORLD
        if handle is None:
            import torch.distributed._symmetric_memory as symm_mem

            handle = symm_mem.rendezvous(c_full, self.group)
        self.handle = handle
        world, rank = plan.world, plan.rank
        receivers = set(plan.receivers())
        self.order = [(rank + d) % world for d in range(1, world) if (rank + d) % world in receivers]
        # Each peer's C as this process sees it (the same view CopyEngineGather copies into).
        shape, dtype = tuple(c_full.shape), c_full.dtype
        self.peer_base = {peer: self.handle.get_buffer(peer, shape, dtype).data_ptr() for peer in self.order}
        self.stream = (new_stream or (lambda: torch.cuda.Stream(device=c_full.device)))()
        self.token = torch.zeros(1, dtype=torch.float32, device=c_full.device)
        self.row_bytes = c_full.shape[1] * c_full.element_size()

    def post(self, index: int, event) -> None:
        lo, hi = self.plan.global_chunk(self.plan.rank, index)
        if hi <= lo or not self.order:
            return
        self.stream.wait_event(event)
        byte_offset = lo * self.row_bytes
        self.push(self.c_full.data_ptr() + byte_offset, [self.peer_base[p] + byte_offset for p in self.order],
                  (hi - lo) * self.row_bytes, self.stream, self.ctas)

    def finish(self) -> None:
        torch.cuda.current_stream(self.c_full.device).wait_stream(self.stream)
        dist.all_reduce(self.token, group=self.group)
