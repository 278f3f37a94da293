"""The multi-GPU (Ulysses head-parallel) host logic on CPU: world size 2 and
4 over the gloo backend, spawned processes, rendezvous on 127.0.0.1.

The exchange must hand rank r exactly heads block r of the whole sequence,
the inverse must restore the shards, and the wrapper must give every rank
the rows its attention function produced for its heads.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from miowtion_b200 import plan as veda_plan
from miowtion_b200 import tiling
from miowtion_b200 import ulysses

SEQ, HEADS, DIM = 48, 8, 16


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _global(seed: int) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(SEQ, HEADS, DIM, generator=gen)


class _PerHeadScale:
    """Stand-in attention function: scales local head j by its global head
    id + 1 and checks the shapes it is given."""

    def __init__(self, first: int, local: int):
        self.first = first
        self.local = local

    def __call__(self, q, k, v, layer_index):
        assert q.shape == (SEQ, self.local, DIM)
        assert k.shape == v.shape == q.shape
        ids = torch.arange(self.first, self.first + self.local,
                           dtype=q.dtype) + 1
        return (q + k + v) * ids[None, :, None] + layer_index


class _PerHeadSoftmax:
    """Differentiable stand-in attention: softmax(q k^T / 4) v per local
    head, one head at a time (the same arithmetic whichever heads a rank
    holds), scaled by the global head id + 1."""

    def __init__(self, first: int, local: int):
        self.first = first
        self.local = local

    def __call__(self, q, k, v, layer_index):
        assert q.shape == (SEQ, self.local, DIM)
        outs = []
        for j in range(self.local):
            p = torch.softmax(q[:, j] @ k[:, j].T / 4.0, -1)
            outs.append((p @ v[:, j]) * (self.first + j + 1))
        return torch.stack(outs, 1)


def _grad_worker(rank: int, world: int, port: int, errors) -> None:
    """The exchanged layer's gradients on every rank equal the rows of the
    one-process gradients of the same function over all heads."""
    try:
        os.environ['MASTER_ADDR'] = '127.0.0.1'
        os.environ['MASTER_PORT'] = str(port)
        dist.init_process_group('gloo', rank=rank, world_size=world)
        shard = SEQ // world
        rows = slice(rank * shard, (rank + 1) * shard)
        q, k, v, dout = (_global(s) for s in (11, 12, 13, 14))
        leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
        whole = _PerHeadSoftmax(0, HEADS)(*leaves, 0)
        (whole * dout).sum().backward()
        shards = [t[rows].clone().requires_grad_(True) for t in (q, k, v)]
        fn = ulysses.UlyssesSparseStudent(
            None, piece_factory=lambda layer, a, b, first: _PerHeadSoftmax(
                first, b - a))
        out = fn(*shards, 0)
        assert torch.equal(out, whole.detach()[rows]), 'forward'
        (out * dout[rows]).sum().backward()
        for name, mine, full in zip('qkv', shards, leaves):
            assert torch.equal(mine.grad, full.grad[rows]), f'd{name}'
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # surfaced by the parent
        errors.put(f'rank {rank}: {e!r}')
        raise


def _worker(rank: int, world: int, port: int, errors) -> None:
    try:
        os.environ['MASTER_ADDR'] = '127.0.0.1'
        os.environ['MASTER_PORT'] = str(port)
        dist.init_process_group('gloo', rank=rank, world_size=world)
        shard = SEQ // world
        rows = slice(rank * shard, (rank + 1) * shard)
        heads = slice(rank * HEADS // world, (rank + 1) * HEADS // world)
        q, k, v = (_global(s) for s in (1, 2, 3))
        # seq_to_heads: rank r receives every row of its head block.
        got = ulysses.seq_to_heads(q[rows].contiguous())
        assert torch.equal(got, q[:, heads]), 'seq_to_heads'
        # heads_to_seq inverts it.
        back = ulysses.heads_to_seq(got)
        assert torch.equal(back, q[rows]), 'heads_to_seq'
        # The wrapper: every rank ends with its rows of every head, for any
        # number of overlapped pieces of its heads.
        ids = torch.arange(HEADS, dtype=q.dtype) + 1
        want = (q + k + v)[rows] * ids[None, :, None] + 3
        for pieces in (1, 2, 3):
            fn = ulysses.UlyssesSparseStudent(
                None, pieces=pieces,
                piece_factory=lambda layer, a, b, first: _PerHeadScale(
                    first, b - a))
            out = fn(q[rows].contiguous(), k[rows].contiguous(),
                     v[rows].contiguous(), 3)
            assert torch.equal(out, want), f'UlyssesSparseStudent {pieces}'
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # surfaced by the parent
        errors.put(f'rank {rank}: {e!r}')
        raise


def _spawn(target, world):
    ctx = mp.get_context('spawn')
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, errors))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not alive, 'a rank did not finish'
    assert not msgs, '\n'.join(msgs)
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.parametrize('world', [2, 4])
def test_exchange_and_wrapper_gloo(world):
    _spawn(_worker, world)


@pytest.mark.parametrize('world', [2, 4])
def test_exchange_backward_gloo(world):
    """The stage-2 student across ranks: gradients flow back through the
    inverse exchanges (dO to the head layout, dQ / dK / dV to the shards)."""
    _spawn(_grad_worker, world)


def test_local_plan_splits_heads_in_contiguous_blocks():
    plan = veda_plan.TilePlan(
        'g', (26, 45, 80), [tiling.TileShape(2, 8, 8),
                            tiling.TileShape(1, 8, 16)],
        [[0] * 24 + [1] * 24])
    for world in (1, 2, 4, 8):
        parts = [ulysses.local_plan(plan, r, world) for r in range(world)]
        joined = sum((p.head_shape[0] for p in parts), [])
        assert joined == plan.head_shape[0]
        assert all(len(p.head_shape[0]) == 48 // world for p in parts)
    with pytest.raises(ValueError):
        ulysses.local_plan(plan, 0, 5)


def test_piece_bounds_cover_the_local_heads():
    assert ulysses.piece_bounds(6, 2) == [(0, 3), (3, 6)]
    assert ulysses.piece_bounds(5, 2) == [(0, 3), (3, 5)]
    assert ulysses.piece_bounds(2, 3) == [(0, 1), (1, 2)]
    assert ulysses.piece_bounds(24, 1) == [(0, 24)]
