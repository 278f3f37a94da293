"""Head-parallel (Ulysses) Veda attention across the GPUs of one node.

The reference runs one clip per GPU and has no sequence parallelism
(miowtion/train/parallel.py:3-5): a tile permutation needs every row of a
sequence on one device. Heads, however, are independent through the whole
Veda path (veda/attention.py:735-738), so a sequence-sharded [S/P, H, D]
activation is exchanged with NCCL all-to-alls into [S, H/P, D], the local
heads run the complete sparse layer, and all-to-alls return [S/P, H, D].
The predictor stays replicated (predictor.py:344-348); each rank scores its
own heads with their global indices.

The local heads can be processed in `pieces` contiguous chunks so that
the exchanges overlap the attention: the inputs of piece j + 1 and the
output of piece j - 1 cross NVLink (asynchronous collectives on NCCL's
stream) while piece j computes. Measured at config 3 on 2 B200 this does
not pay: the persistent attention kernel holds every SM, so NCCL's kernels
either delay some of its CTAs (pieces 2: 20.1 ms/layer) or get SMs it gives
up (pieces 2, 16 SMs reserved: 20.5 ms), against 19.5 ms with one piece.
The default is therefore one piece. Every rank issues the same collectives
in the same order. Exchange layout of a piece of c heads: the send buffer is
[P, S/P, c, D] (chunk p = this rank's rows of rank p's piece heads); the
receive buffer [P, S/P, c, D] is then [S, c, D] in sequence order.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from miowtion_b200 import _lib
from miowtion_b200 import attention as veda_attention
from miowtion_b200 import kernels
from miowtion_b200 import plan as veda_plan


def local_plan(plan: veda_plan.TilePlan, rank: int,
               world: int) -> veda_plan.TilePlan:
    """The plan restricted to this rank's contiguous block of heads."""
    heads = len(plan.head_shape[0])
    if heads % world:
        raise ValueError(f'{heads} heads do not split over {world} ranks')
    per = heads // world
    rows = [row[rank * per:(rank + 1) * per] for row in plan.head_shape]
    return veda_plan.TilePlan(plan.geometry, plan.grid, plan.shapes, rows,
                              dict(plan.provenance, rank=rank, world=world))


def piece_bounds(local_heads: int, pieces: int) -> list[tuple[int, int]]:
    """[start, stop) of each piece of the local heads (at most `pieces`,
    none empty)."""
    pieces = max(1, min(pieces, local_heads))
    size = -(-local_heads // pieces)
    return [(a, min(a + size, local_heads))
            for a in range(0, local_heads, size)]


def _head_blocks(src: torch.Tensor, dst: torch.Tensor, world: int,
                 start: int, stop: int, pack: bool) -> None:
    """veda_head_blocks between a [S/P, H, D] tensor (strided side) and a
    [P, S/P, c, D] one (packed side), for heads p * H/P + [start, stop)."""
    strided = src if pack else dst
    rows, heads, dim = strided.shape
    per = heads // world
    size = strided.element_size()
    if not (strided.is_cuda and strided.is_contiguous()
            and (dst if pack else src).is_contiguous()):
        raise ValueError('the exchange buffers must be contiguous CUDA '
                         'tensors')
    _lib.call('veda_head_blocks', src.data_ptr(), dst.data_ptr(), rows,
              world, (stop - start) * dim * size, heads * dim * size,
              per * dim * size, start * dim * size, 1 if pack else 0,
              _lib.stream_ptr(strided.device))


def _pack(x: torch.Tensor, world: int, start: int, stop: int) -> torch.Tensor:
    """[S/P, H, D] -> [P, S/P, c, D]: chunk p holds heads
    p * H/P + [start, stop)."""
    rows, heads, dim = x.shape
    if not x.is_cuda:
        per = heads // world
        return x.view(rows, world, per, dim)[:, :, start:stop].transpose(
            0, 1).contiguous()
    out = torch.empty(world, rows, stop - start, dim, dtype=x.dtype,
                      device=x.device)
    _head_blocks(x.contiguous(), out, world, start, stop, pack=True)
    return out


def seq_to_heads(x: torch.Tensor, group=None) -> torch.Tensor:
    """[S/P, H, D] on every rank -> [S, H/P, D] (rank r gets heads block r)."""
    world = dist.get_world_size(group)
    rows, heads, dim = x.shape
    if heads % world:
        raise ValueError('heads must divide by the world size')
    send = _pack(x, world, 0, heads // world)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(world * rows, heads // world, dim)


def heads_to_seq(y: torch.Tensor, group=None) -> torch.Tensor:
    """[S, H/P, D] -> [S/P, H, D] (the inverse of seq_to_heads)."""
    world = dist.get_world_size(group)
    seq, local_heads, dim = y.shape
    if seq % world:
        raise ValueError('the sequence must divide by the world size')
    send = y.view(world, seq // world, local_heads, dim)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send.contiguous(), group=group)
    if not recv.is_cuda:
        return recv.transpose(0, 1).reshape(seq // world,
                                            world * local_heads, dim)
    out = torch.empty(seq // world, world * local_heads, dim, dtype=y.dtype,
                      device=y.device)
    _head_blocks(recv, out, world, 0, local_heads, pack=False)
    return out


class _ToHeads(torch.autograd.Function):
    """seq_to_heads as a differentiable op. The exchange is a permutation of
    rows and heads across the ranks, so its adjoint is the inverse exchange:
    the incoming gradient [S, H/P, D] goes back through heads_to_seq."""

    @staticmethod
    def forward(ctx, x, group):  # pylint: disable=arguments-differ
        ctx.group = group
        return seq_to_heads(x.contiguous(), group)

    @staticmethod
    def backward(ctx, grad):  # pylint: disable=arguments-differ
        return heads_to_seq(grad.contiguous(), ctx.group), None


class _ToSeq(torch.autograd.Function):
    """heads_to_seq as a differentiable op; its adjoint is seq_to_heads."""

    @staticmethod
    def forward(ctx, y, group):  # pylint: disable=arguments-differ
        ctx.group = group
        return heads_to_seq(y.contiguous(), group)

    @staticmethod
    def backward(ctx, grad):  # pylint: disable=arguments-differ
        return seq_to_heads(grad.contiguous(), ctx.group), None


class CopyEngineExchange:
    """The head-parallel exchange of one shard shape on the copy engines.

    Every rank owns receive buffers for q, k and v ([S, H/P, D] each, the
    rank's heads of every row) and a result buffer of the same shape, and
    maps its peers' buffers through CUDA IPC. Inputs are pushed: rank r
    copies rows [r S/P, (r + 1) S/P) of peer p's heads straight from its
    [S/P, H, D] shard into p's receive buffer, one strided 2-D copy per
    peer and tensor (no packing pass). Outputs are pulled: rank r copies its
    rows of every peer's result buffer into the heads of its output shard.
    The copies run on the copy engines, one stream per peer, and take no SM
    from the attention.

    Ordering between the ranks uses interprocess CUDA events (one per rank
    and purpose: inputs pushed, q/k pushed, v pushed, receive buffers free,
    result written, results pulled), waited on by the GPU streams; a host
    barrier on a gloo group between each record and the peers' waits makes
    the waits refer to this step's records. Every rank calls the same
    barriers in the same order.
    """

    EVENTS = ('qk', 'v', 'free', 'result', 'pulled')

    def __init__(self, rows: int, heads: int, dim: int, dtype: torch.dtype,
                 device: torch.device, group=None, host_group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if heads % self.world:
            raise ValueError('heads must divide by the world size')
        self.rows, self.heads, self.dim = rows, heads, dim
        self.per = heads // self.world
        self.elem = torch.empty((), dtype=dtype).element_size()
        self.device = device
        self.host_group = host_group or dist.new_group(backend='gloo')
        seq = rows * self.world
        self.recv = torch.empty(3, seq, self.per, dim, dtype=dtype,
                                device=device)
        self.result = torch.empty(seq, self.per, dim, dtype=dtype,
                                  device=device)
        # One copy stream per peer (own rows included), so the copies to
        # different GPUs run on different copy engines at once; `stream`
        # joins them for the events.
        self.stream = torch.cuda.Stream(device)
        self.streams = [torch.cuda.Stream(device) for _ in range(self.world)]
        lib = _lib.load()
        mine = []
        for buf in (self.recv, self.result):
            handle = (ctypes.c_uint8 * 64)()
            offset = ctypes.c_int64()
            _lib.check(lib.veda_ipc_handle(ctypes.c_void_p(buf.data_ptr()),
                                           handle, ctypes.byref(offset)),
                       'veda_ipc_handle')
            mine.append((bytes(handle), offset.value))
        self.events = {name: torch.cuda.Event(interprocess=True)
                       for name in self.EVENTS}
        ev_handles = {name: e.ipc_handle() for name, e in self.events.items()}
        gathered = [None] * self.world
        dist.all_gather_object(gathered, (mine, ev_handles),
                               group=self.host_group)
        self._opened = []
        self.peer_recv, self.peer_result, self.peer_events = [], [], []
        for p, (bufs, evs) in enumerate(gathered):
            if p == self.rank:
                self.peer_recv.append(self.recv.data_ptr())
                self.peer_result.append(self.result.data_ptr())
                self.peer_events.append(self.events)
                continue
            addrs = []
            for handle, offset in bufs:
                base = ctypes.c_void_p()
                raw = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
                _lib.check(lib.veda_ipc_open(raw, ctypes.byref(base)),
                           'veda_ipc_open')
                self._opened.append(base.value)
                addrs.append(base.value + offset)
            self.peer_recv.append(addrs[0])
            self.peer_result.append(addrs[1])
            self.peer_events.append({
                name: torch.cuda.Event.from_ipc_handle(device, h)
                for name, h in evs.items()})

    def close(self) -> None:
        """Unmaps the peers' buffers (after every rank's last use)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.host_group)
        for base in self._opened:
            _lib.call('veda_ipc_close', base)
        self._opened = []

    def _barrier(self) -> None:
        dist.barrier(group=self.host_group)

    @staticmethod
    def _copy(stream, dst: int, dst_pitch: int, src: int, src_pitch: int,
              width: int, height: int) -> None:
        _lib.call('veda_copy_2d', dst, dst_pitch, src, src_pitch, width,
                  height, stream.cuda_stream)

    def _join(self) -> None:
        for st in self.streams:
            self.stream.wait_stream(st)

    def run(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
            attend, v_wait=None, timers=None) -> torch.Tensor:
        """One exchanged layer: `attend(q_h, k_h, v_h, out)` runs this
        rank's heads on [S, H/P, D] views of the receive buffers and writes
        `out` (the result buffer). With `v_wait`, `attend` receives a
        callable that makes the current stream wait for v, to call at its
        first read of v; otherwise all inputs are waited for first. Returns the [S/P, H, D] output
        shard. `timers` (StageEvents) records 'exchange' on the current
        stream: until q and k have arrived, and from the result until the
        output shard is assembled."""
        timers = timers or veda_attention._NO_EVENTS  # pylint: disable=protected-access
        for t in (q, k, v):
            if (t.shape != (self.rows, self.heads, self.dim) or
                    not t.is_contiguous() or t.device != self.device):
                raise ValueError('the exchange was set up for contiguous '
                                 f'[{self.rows}, {self.heads}, {self.dim}] '
                                 'shards on this device')
        world, rank, per = self.world, self.rank, self.per
        row_b = per * self.dim * self.elem        # one row of a head block
        shard_b = self.heads * self.dim * self.elem  # one row of a shard
        block_b = self.rows * row_b               # a rank's rows of a block
        plane_b = world * block_b                 # one receive buffer
        cur = torch.cuda.current_stream(self.device)
        ev = self.events
        tok = timers.start('exchange')
        # Every rank has enqueued the previous layer (its buffer-free and
        # pulled records) before anyone waits on them.
        self._barrier()
        for p, st in enumerate(self.streams):
            st.wait_stream(cur)  # q, k, v are ready
            st.wait_event(self.peer_events[p]['free'])
        for t, x in enumerate((q, k, v)):
            for p, st in enumerate(self.streams):
                self._copy(st, self.peer_recv[p] + t * plane_b +
                           rank * block_b, row_b, x.data_ptr() + p * row_b,
                           shard_b, row_b, self.rows)
            if t == 1:
                self._join()
                ev['qk'].record(self.stream)
        self._join()
        ev['v'].record(self.stream)
        self._barrier()
        for p in range(world):
            cur.wait_event(self.peer_events[p]['qk'])
            # The result buffer is free once every peer pulled the last one.
            cur.wait_event(self.peer_events[p]['pulled'])
        timers.stop(tok)

        def wait_v():
            for p in range(world):
                cur.wait_event(self.peer_events[p]['v'])

        if not v_wait:
            wait_v()
        q_h, k_h, v_h = self.recv.unbind(0)
        attend(q_h, k_h, v_h, self.result, wait_v if v_wait else None)
        wait_v()  # v arrived before the buffers count as free again
        ev['result'].record(cur)
        ev['free'].record(cur)
        tok = timers.start('exchange')
        self._barrier()
        out = torch.empty_like(q)
        for p, st in enumerate(self.streams):
            st.wait_stream(cur)  # `out` is allocated on `cur`
            st.wait_event(self.peer_events[p]['result'])
            self._copy(st, out.data_ptr() + p * row_b, shard_b,
                       self.peer_result[p] + rank * block_b, row_b, row_b,
                       self.rows)
        self._join()
        ev['pulled'].record(self.stream)
        cur.wait_stream(self.stream)
        timers.stop(tok)
        return out


class UlyssesSparseStudent:
    """`AttentionFn` over sequence-sharded q, k, v [S/P, H, D] per rank.

    `student` is the rank's SparseStudent over its local plan (heads
    [rank * H/P, (rank + 1) * H/P)); its clip and predictor are shared by
    the per-piece students built here. `piece_factory(layer, start, stop,
    first_head)` may replace that construction: it returns the attention
    function of local heads [start, stop), whose first global head is
    `first_head` (the CPU tests pass stand-ins this way).
    """

    def __init__(self, student: veda_attention.SparseStudent | None,
                 group=None, pieces: int = 1, piece_factory=None,
                 reserve_sms: int = 16, transport: str = 'nccl'):
        """`transport`: 'nccl' (all-to-alls, with packing kernels) or 'copy'
        (`CopyEngineExchange`: copy-engine copies between IPC-mapped
        buffers; the inference path of CUDA tensors, one piece)."""
        if transport not in ('nccl', 'copy'):
            raise ValueError(f"transport must be 'nccl' or 'copy': "
                             f'{transport!r}')
        self.transport = transport
        self._exchanges: dict = {}
        self.student = student
        self.group = group
        self.pieces = pieces
        self.piece_factory = piece_factory
        # While pieces overlap exchanges, the attention leaves this many
        # SMs to NCCL's kernels (its persistent CTAs would otherwise hold
        # every SM until it ends).
        self.reserve_sms = reserve_sms
        self._students: dict = {}

    def _piece_student(self, layer_index: int, start: int, stop: int,
                       head0: int) -> veda_attention.SparseStudent:
        key = (layer_index, start, stop)
        if key not in self._students and self.piece_factory is not None:
            self._students[key] = self.piece_factory(layer_index, start, stop,
                                                     head0 + start)
        if key not in self._students:
            base = self.student
            plan = base.plan
            sub = veda_plan.TilePlan(
                plan.geometry, plan.grid, plan.shapes,
                [list(r)[start:stop] for r in plan.head_shape],
                dict(plan.provenance, piece=[start, stop]))
            self._students[key] = veda_attention.SparseStudent(
                base.clip, sub, base.predictor, head_offset=head0 + start)
        return self._students[key]

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 layer_index: int) -> torch.Tensor:
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        rows, heads, dim = q.shape
        if heads % world:
            raise ValueError('heads must divide by the world size')
        per = heads // world
        if self.piece_factory is None and len(
                self.student.plan.head_shape[layer_index]) != per:
            raise ValueError('the student plan does not hold this rank\'s '
                             f'{per} heads')
        if torch.is_grad_enabled() and any(t.requires_grad
                                           for t in (q, k, v)):
            return self._run_grad(q, k, v, layer_index, rank, per)
        if self.transport == 'copy' and q.is_cuda:
            return self._run_copy(q, k, v, layer_index, rank, per)
        bounds = piece_bounds(per, self.pieces)
        reserve = self.reserve_sms if (world > 1 and len(bounds) > 1
                                       and self.piece_factory is None) else 0
        if reserve:
            kernels.set_sm_reserve(reserve)
        try:
            return self._run(q, k, v, layer_index, world, rank, per, bounds)
        finally:
            if reserve:
                kernels.set_sm_reserve(0)

    def _run_copy(self, q, k, v, layer_index, rank, per):
        """The inference layer over `CopyEngineExchange` (one piece): the
        rank's student reads q, k, v from the receive buffers, waits for v
        only after scoring, and writes the shared result buffer."""
        key = (tuple(q.shape), q.dtype, q.device)
        ex = self._exchanges.get(key)
        if ex is None:
            ex = CopyEngineExchange(q.shape[0], q.shape[1], q.shape[2],
                                    q.dtype, q.device, self.group)
            self._exchanges[key] = ex
        student = self._piece_student(layer_index, 0, per, rank * per)
        timers = veda_attention._NO_EVENTS  # pylint: disable=protected-access
        if self.student is not None:
            student.events = self.student.events
            timers = self.student.events
        sparse = isinstance(student, veda_attention.SparseStudent)

        def attend(q_h, k_h, v_h, out, wait_v):
            if sparse:
                student.v_ready = wait_v
                try:
                    student(q_h, k_h, v_h, layer_index, out=out)
                finally:
                    student.v_ready = None
            else:
                out.copy_(student(q_h, k_h, v_h, layer_index))

        return ex.run(q, k, v, attend, v_wait=sparse, timers=timers)

    def close(self) -> None:
        """Releases the copy-engine exchanges (collective: every rank)."""
        for ex in self._exchanges.values():
            ex.close()
        self._exchanges.clear()

    def to_heads(self, x: torch.Tensor) -> torch.Tensor:
        """[S/P, H, D] shard -> [S, H/P, D] (differentiable)."""
        return _ToHeads.apply(x, self.group)

    def to_seq(self, y: torch.Tensor) -> torch.Tensor:
        """[S, H/P, D] -> [S/P, H, D] shard (differentiable)."""
        return _ToSeq.apply(y, self.group)

    def local(self, layer_index: int):
        """The attention function of this rank's heads, in the head
        layout (global predictor indices)."""
        if self.student is None:
            raise ValueError("local() needs the rank's SparseStudent")
        per = len(self.student.plan.head_shape[layer_index])
        rank = dist.get_rank(self.group)
        return self._piece_student(layer_index, 0, per, rank * per)

    def _run_grad(self, q, k, v, layer_index, rank, per):
        """The differentiable layer (the stage-2 student step across
        ranks): q, k, v go to the head layout through `_ToHeads`, the rank's
        heads run the sparse layer with its autograd backward, and the
        output returns through `_ToSeq`. The backward therefore exchanges
        dO into the head layout, runs the sparse backward, and exchanges
        dQ, dK, dV back to the sequence shards. Every rank builds the same
        graph, so the backward's collectives come in the same order on
        every rank. One piece: the backward has no overlap to gain."""
        ev = (self.student.events if self.student is not None
              else veda_attention._NO_EVENTS)  # pylint: disable=protected-access
        t = ev.start('exchange')
        qh, kh, vh = (self.to_heads(x) for x in (q, k, v))
        ev.stop(t)
        student = self._piece_student(layer_index, 0, per, rank * per)
        if self.student is not None:
            student.events = self.student.events
        out = student(qh, kh, vh, layer_index)
        t = ev.start('exchange')
        out = self.to_seq(out)
        ev.stop(t)
        return out

    def _run(self, q, k, v, layer_index, world, rank, per, bounds):
        rows, _, dim = q.shape
        inputs: dict = {}

        def post_inputs(j: int) -> None:
            start, stop = bounds[j]
            bufs, works = [], []
            for x in (q, k, v):
                send = _pack(x, world, start, stop)
                recv = torch.empty_like(send)
                works.append(dist.all_to_all_single(recv, send,
                                                    group=self.group,
                                                    async_op=True))
                bufs.append((send, recv))
            inputs[j] = (bufs, works)

        def v_waiter(work):
            # The student reads v only after scoring its heads from q and k:
            # until then v's exchange runs beside the pooling, predictor and
            # selection kernels.
            done = []

            def wait():
                if not done:
                    work.wait()
                    done.append(True)
            return wait

        # Stage timers (bench): the exchanges, packing included, on the
        # launching stream. With several pieces they overlap the attention.
        ev = (self.student.events if self.student is not None
              else veda_attention._NO_EVENTS)  # pylint: disable=protected-access
        out = torch.empty_like(q)
        outputs = []
        t = ev.start('exchange')
        post_inputs(0)
        for j, (start, stop) in enumerate(bounds):
            if j + 1 < len(bounds):
                post_inputs(j + 1)
            bufs, works = inputs.pop(j)
            student = self._piece_student(layer_index, start, stop,
                                          rank * per)
            # A SparseStudent waits for v itself, after scoring from q and
            # k; any other attention function gets all three first.
            defer_v = isinstance(student, veda_attention.SparseStudent)
            for w in (works[:2] if defer_v else works):
                w.wait()
            if j == 0:
                ev.stop(t)
            c = stop - start
            qj, kj, vj = (recv.view(world * rows, c, dim)
                          for _, recv in bufs)
            if self.student is not None:
                # Stage timers set on the rank's student cover its pieces.
                student.events = self.student.events
            if defer_v:
                wait_v = v_waiter(works[2])
                student.v_ready = wait_v
                try:
                    result = student(qj, kj, vj, layer_index)
                finally:
                    student.v_ready = None
                wait_v()  # a path that did not read v
            else:
                result = student(qj, kj, vj, layer_index)
            back = torch.empty_like(result).view(world, rows, c, dim)
            if j + 1 == len(bounds):
                t = ev.start('exchange')
            work = dist.all_to_all_single(
                back, result.view(world, rows, c, dim), group=self.group,
                async_op=True)
            outputs.append((start, stop, back, result, work))
        for start, stop, back, _result, work in outputs:
            work.wait()
            if out.is_cuda:
                _head_blocks(back, out, world, start, stop, pack=False)
            else:
                out.view(rows, world, per, dim)[:, :, start:stop] = (
                    back.transpose(0, 1))
        ev.stop(t)
        return out
