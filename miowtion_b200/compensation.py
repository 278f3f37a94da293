"""Zero-order compensation next to the block-sparse kernel: drop-in for the
reference's `miowtion/kernels/compensation_triton.py` (`compensate`,
`attention`) and the torch form `veda.attention.zero_order_compensation`
(attention.py:591-689), backed by `veda_compensate` (csrc/compensate.cu).

Each dropped key tile is replaced by one virtual key at its centroid
(mean k) carrying its value sum (sum v) and weighted by its real row count,
folded into the sparse output with the sparse kernel's own LSE as the
exponent reference:

    out = (o_kept + sum_dropped p_t vsum_t) / (1 + sum_dropped p_t B_t),
    p_t = exp(q . kmean_t * scale - lse_kept).
"""

from __future__ import annotations

import math

import torch

from miowtion_b200 import _lib
from miowtion_b200 import kernels
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import tiling

TILE = tiling.TILE_SIZE


def _check_rows(t: torch.Tensor, name: str) -> None:
    tiling._check_rows(t, name)  # pylint: disable=protected-access


def compensate_lists(o_kept: torch.Tensor, lse_kept: torch.Tensor,
                     q_tiles: torch.Tensor, k_tiles: torch.Tensor,
                     v_tiles: torch.Tensor, lists: veda_mask.BlockLists,
                     tile_layout: tiling.TileLayout,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """The compensated output of query tiles whose kept key tiles are the
    forward's index lists (rows of `lists` = query tiles of q_tiles).
    `out` may be `o_kept` itself (in place)."""
    kernels._require(q_tiles, 'zero-order compensation')  # noqa: SLF001
    rows, heads, dim = o_kept.shape
    if dim != 128:
        raise ValueError('the compensation kernel takes head_dim 128')
    if q_tiles.shape != o_kept.shape:
        raise ValueError(f'q_tiles is {tuple(q_tiles.shape)}, expected '
                         f'{tuple(o_kept.shape)}')
    if lse_kept.shape != (heads, rows):
        raise ValueError(f'lse_kept is {tuple(lse_kept.shape)}, expected '
                         f'{(heads, rows)}')
    if k_tiles.shape[0] != tile_layout.num_slots or v_tiles.shape != (
            k_tiles.shape) or k_tiles.shape[1:] != (heads, dim):
        raise ValueError('k_tiles and v_tiles must be [num_slots, H, D]')
    if lists.part_cnt.shape != (heads, rows // TILE):
        raise ValueError('lists must cover (heads, query tiles)')
    for name, t in (('o_kept', o_kept), ('q_tiles', q_tiles),
                    ('k_tiles', k_tiles), ('v_tiles', v_tiles)):
        _check_rows(t, name)
    lse_kept = lse_kept.float().contiguous()
    out = torch.empty_like(o_kept) if out is None else out
    _check_rows(out, 'out')
    lib = _lib.load()
    ws_bytes = lib.veda_compensate_workspace(heads, tile_layout.n_tiles)
    ws = torch.empty(ws_bytes // 2, dtype=torch.bfloat16,
                     device=o_kept.device)
    _lib.call('veda_compensate', o_kept.data_ptr(), o_kept.stride(0),
              o_kept.stride(1), lse_kept.data_ptr(), q_tiles.data_ptr(),
              q_tiles.stride(0), q_tiles.stride(1), k_tiles.data_ptr(),
              k_tiles.stride(0), k_tiles.stride(1), v_tiles.data_ptr(),
              v_tiles.stride(0), v_tiles.stride(1), heads, rows // TILE,
              tile_layout.n_tiles, tile_layout.valid_count.data_ptr(),
              lists.part_cnt.data_ptr(), lists.part_idx.data_ptr(),
              lists.full_cnt.data_ptr(), lists.full_idx.data_ptr(),
              lists.part_idx.shape[-1], out.data_ptr(), out.stride(0),
              out.stride(1), 1.0 / math.sqrt(dim), ws.data_ptr(), ws_bytes,
              _lib.stream_ptr(o_kept.device))
    return out


def zero_order_compensation(o_kept: torch.Tensor, lse_kept: torch.Tensor,
                            q_tiles: torch.Tensor, k_tiles: torch.Tensor,
                            v_tiles: torch.Tensor, block_mask: torch.Tensor,
                            tile_layout: tiling.TileLayout,
                            chunk_rows: int = 4096) -> torch.Tensor:
    """The torch form's contract (veda/attention.py:591-689): query tiles
    may be any subset whose rows `block_mask` [H', R, n] describes.
    `chunk_rows` bounds the torch form's score matrix; the kernel keeps its
    scores on chip, so it has no effect here.

    Raises:
        ValueError: On a shape mismatch.
    """
    del chunk_rows
    rows, heads = o_kept.shape[0], o_kept.shape[1]
    if block_mask.shape != (heads, rows // TILE, tile_layout.n_tiles):
        raise ValueError(
            f'block_mask is {tuple(block_mask.shape)}, expected '
            f'{(heads, rows // TILE, tile_layout.n_tiles)}')
    lists = kernels._lists(block_mask, tile_layout,  # noqa: SLF001
                           transpose=False, tails=False)
    return compensate_lists(o_kept, lse_kept, q_tiles, k_tiles, v_tiles,
                            lists, tile_layout)


def compensate(o_kept: torch.Tensor, lse_kept: torch.Tensor,
               q_tiles: torch.Tensor, k_tiles: torch.Tensor,
               v_tiles: torch.Tensor, block_mask: torch.Tensor,
               tile_layout: tiling.TileLayout) -> torch.Tensor:
    """compensation_triton.compensate (:176-226): the same term for every
    query tile (R == n_tiles), with the same argument checks.

    Raises:
        ValueError: On a shape mismatch, or a query-tile subset (the
            reference's kernel pairs mask row r with query tile r).
    """
    rows, heads, _ = o_kept.shape
    tiles = tile_layout.n_tiles
    if q_tiles.shape != o_kept.shape:
        raise ValueError(f'q_tiles is {tuple(q_tiles.shape)}, expected '
                         f'{tuple(o_kept.shape)}')
    if lse_kept.shape != (heads, rows):
        raise ValueError(f'lse_kept is {tuple(lse_kept.shape)}, expected '
                         f'{(heads, rows)}')
    if block_mask.shape != (heads, rows // TILE, tiles):
        raise ValueError(f'block_mask is {tuple(block_mask.shape)}, '
                         f'expected {(heads, rows // TILE, tiles)}')
    if rows // TILE != tiles:
        raise ValueError(
            f'{rows // TILE} query tiles but {tiles} key tiles; this '
            f'kernel indexes both with the same id')
    return zero_order_compensation(o_kept, lse_kept, q_tiles, k_tiles,
                                   v_tiles, block_mask, tile_layout)


def attention(q_tiles: torch.Tensor, k_tiles: torch.Tensor,
              v_tiles: torch.Tensor, block_mask: torch.Tensor,
              tile_layout: tiling.TileLayout) -> torch.Tensor:
    """Block-sparse attention plus the compensation, end to end
    (compensation_triton.attention, :229-245): the forward writes o_kept and
    its LSE, the compensation rewrites o_kept in place."""
    kept = block_mask & tile_layout.kv_ok[None, None, :]
    lists = kernels._lists(kept, tile_layout,  # noqa: SLF001
                           transpose=False, tails=False)
    o_kept, lse = kernels.block_sparse_attention_lists(
        q_tiles, k_tiles, v_tiles, lists, tile_layout, return_lse=True)
    return compensate_lists(o_kept, lse, q_tiles, k_tiles, v_tiles, lists,
                            tile_layout, out=o_kept)
