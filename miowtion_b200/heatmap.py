"""Teacher block heat: drop-in for the reference's `miowtion/veda/heatmap.py`
heat entry points (`teacher_heat`, `teacher_heat_reference`), backed by the
tcgen05 kernel `veda_teacher_heat`. The reference's supervision losses in the
same module (seer_kl, transport_loss, ...) are small fp32 torch on the tile
grid and stay outside this package.
"""

from __future__ import annotations

import math

import torch

from miowtion_b200 import _lib
from miowtion_b200 import kernels
from miowtion_b200 import tiling


@torch.no_grad()
def teacher_heat(q: torch.Tensor, k: torch.Tensor, lse: torch.Tensor,
                 layout: tiling.TileLayout, q_tiles: torch.Tensor,
                 reduce: str = 'max') -> torch.Tensor:
    """Per-block teacher heat (heatmap.py:36-110).

    Args:
        q: [N, H', D] bf16 tile-ordered queries.
        k: [N, H', D] bf16 tile-ordered keys.
        lse: [N, H'] fp32 tile-ordered teacher LSE (0 on padding slots).
        layout: Tile layout.
        q_tiles: [R] int64 query tiles to supervise.
        reduce: 'max' for the block's peak probability, 'sum' for its mass.

    Returns:
        [H', R, n_tiles] fp32 heat, 0 on padding query rows / empty keys.

    Raises:
        ValueError: On an unknown reduction or mismatched shapes.
        NotImplementedError: Off B200 (no fallback).
    """
    if reduce not in ('max', 'sum'):
        raise ValueError(f"reduce must be 'max' or 'sum': {reduce!r}")
    kernels._require(q, 'teacher_heat')  # pylint: disable=protected-access
    heads = q.shape[1]
    if k.shape != q.shape or q.shape[0] != layout.num_slots:
        raise ValueError('q and k must be [num_slots, H\', D]')
    if lse.shape != (layout.num_slots, heads):
        raise ValueError('lse must be [num_slots, H\']')
    for name, t in (('q', q), ('k', k)):
        tiling._check_rows(t, name)  # pylint: disable=protected-access
    lse = lse.float()
    q_tiles = q_tiles.to(device=q.device, dtype=torch.int64).contiguous()
    heat = torch.empty(heads, q_tiles.numel(), layout.n_tiles,
                       dtype=torch.float32, device=q.device)
    _lib.call('veda_teacher_heat', q.data_ptr(), q.stride(0), q.stride(1),
              k.data_ptr(), k.stride(0), k.stride(1), lse.data_ptr(),
              lse.stride(0), lse.stride(1), heads, layout.n_tiles,
              layout.valid_count.data_ptr(), q_tiles.data_ptr(),
              q_tiles.numel(), 1 if reduce == 'sum' else 0, heat.data_ptr(),
              1.0 / math.sqrt(q.shape[-1]), _lib.stream_ptr(q.device))
    return heat


def teacher_heat_reference(q: torch.Tensor, k: torch.Tensor,
                           lse: torch.Tensor, layout: tiling.TileLayout,
                           q_tiles: torch.Tensor, q_chunk: int = 2048,
                           k_chunk: int = 8192,
                           reduce: str = 'max') -> torch.Tensor:
    """The reference's name for the same computation (heatmap.py:36-99);
    the chunk sizes of its torch loop do not apply to the kernel."""
    del q_chunk, k_chunk
    return teacher_heat(q, k, lse, layout, q_tiles, reduce)


@torch.no_grad()
def fused_dense_heat(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     layout: tiling.TileLayout, reduce: str = 'max'
                     ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The teacher's dense attention of one head group and its block heat
    for every query tile in one pass (the fused kernel the reference plans,
    docs/features/veda_kernel.md:285-288).

    Args:
        q, k, v: [N, H', D] bf16 tile-ordered rows of the group.
        layout: Tile layout of the group.
        reduce: 'max' (the block's peak probability, the reference's bf16
            score rounding included) or 'sum' (its mass, from the fp32
            scores of the softmax).

    Returns:
        (out [N, H', D] bf16 in tile order, lse [H', N] fp32 natural log,
        heat [H', n_tiles, n_tiles] fp32). Padding slots' out and lse are
        unspecified; `tiling.scatter_tiles_` drops them.

    Raises:
        ValueError: On an unknown reduction or mismatched shapes.
        NotImplementedError: Off B200 (no fallback).
    """
    if reduce not in ('max', 'sum'):
        raise ValueError(f"reduce must be 'max' or 'sum': {reduce!r}")
    kernels._require(q, 'fused_dense_heat')  # pylint: disable=protected-access
    heads = q.shape[1]
    n = layout.n_tiles
    if k.shape != q.shape or v.shape != q.shape or (
            q.shape[0] != layout.num_slots):
        raise ValueError('q, k and v must be [num_slots, H\', D]')
    for name, t in (('q', q), ('k', k), ('v', v)):
        tiling._check_rows(t, name)  # pylint: disable=protected-access
    keep = layout.kv_ok.view(1, 1, n).expand(heads, n, n)
    lists = kernels._lists(keep, layout,  # pylint: disable=protected-access
                           transpose=False, tails=False)
    out = torch.empty_like(q)
    lse = torch.empty(heads, layout.num_slots, dtype=torch.float32,
                      device=q.device)
    heat = torch.zeros(heads, n, n, dtype=torch.float32, device=q.device)
    ws_bytes = _lib.load().veda_bsa_fwd_heat_workspace(n)
    ws = torch.empty(max(1, ws_bytes // 4), dtype=torch.float32,
                     device=q.device)
    _lib.call('veda_bsa_fwd_heat', q.data_ptr(), q.stride(0), q.stride(1),
              k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(),
              v.stride(0), v.stride(1), heads, n,
              layout.valid_count.data_ptr(), lists.part_cnt.data_ptr(),
              lists.part_idx.data_ptr(), lists.full_cnt.data_ptr(),
              lists.full_idx.data_ptr(), lists.part_idx.shape[-1],
              out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
              1 if reduce == 'sum' else 0, heat.data_ptr(),
              1.0 / math.sqrt(q.shape[-1]), ws.data_ptr(), ws.numel() * 4,
              _lib.stream_ptr(q.device))
    return out, lse, heat
