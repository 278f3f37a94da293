"""Head-parallel (Ulysses) Veda attention across the GPUs of one node.

The reference runs one clip per GPU and has no sequence parallelism
(miowtion/train/parallel.py:3-5): a tile permutation needs every row of a
sequence on one device. Heads, however, are independent through the whole
Veda path (veda/attention.py:735-738), so a sequence-sharded [S/P, H, D]
activation is exchanged with one NCCL all-to-all into [S, H/P, D], the local
heads run the complete sparse layer, and a second all-to-all returns
[S/P, H, D]. The predictor stays replicated (predictor.py:344-348).

Exchange layout: the send buffer is [P, S/P, H/P, D] (chunk p = this
rank's rows of rank p's heads); the receive buffer [P, S/P, H/P, D] is then
exactly [S, H/P, D] in sequence order, so no unpack copy is needed.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from miowtion_b200 import attention as veda_attention
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


def seq_to_heads(x: torch.Tensor, group=None) -> torch.Tensor:
    """[S/P, H, D] on every rank -> [S, H/P, D] (rank r gets heads block r)."""
    world = dist.get_world_size(group)
    rows, heads, dim = x.shape
    if heads % world:
        raise ValueError('heads must divide by the world size')
    send = x.view(rows, world, heads // world, dim).transpose(0, 1)
    send = send.contiguous()
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
    return recv.transpose(0, 1).reshape(seq // world, world * local_heads,
                                        dim)


class UlyssesSparseStudent:
    """`AttentionFn` over sequence-sharded q, k, v [S/P, H, D] per rank."""

    def __init__(self, student: veda_attention.SparseStudent, group=None):
        self.student = student
        self.group = group

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 layer_index: int) -> torch.Tensor:
        qh = seq_to_heads(q, self.group)
        kh = seq_to_heads(k, self.group)
        vh = seq_to_heads(v, self.group)
        out = self.student(qh, kh, vh, layer_index)
        return heads_to_seq(out, self.group)
