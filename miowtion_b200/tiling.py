"""Tile permutations: reorder packed rows so every 128 rows form a 3D tile.

Host-side mirror of the reference's `miowtion/veda/tiling.py` (same names,
argument meaning and errors). The permutation itself is computed on the
device by `veda_build_layout` (closed form, see csrc/layout.cu); the
derived constants are built once per (spans, shape, device) and cached by
the caller, as in the reference (tiling.py:159-166).

A tile shape (tt, th, tw) with tt*th*tw = 128 cuts a (T, H, W) token grid
into boxes. Each tiled span is cut with its own shape; all other real rows
are "global" and are chunked into 128-row tiles in sequence order, after
all video tiles. Inside a tile, real rows form a prefix of length
valid_count[tile].
"""

from __future__ import annotations

import dataclasses
import itertools
from collections.abc import Sequence

import torch

from miowtion_b200 import _lib

TILE_SIZE = 128


@dataclasses.dataclass(frozen=True, order=True)
class TileShape:
    """A (t, h, w) box of TILE_SIZE tokens (tiling.py:43-82)."""

    t: int
    h: int
    w: int

    def __post_init__(self):
        if self.t * self.h * self.w != TILE_SIZE:
            raise ValueError(f'tile {self} does not hold {TILE_SIZE} tokens')

    def __str__(self) -> str:
        return f'{self.t}x{self.h}x{self.w}'

    @classmethod
    def parse(cls, text: str) -> TileShape:
        t, h, w = (int(v) for v in text.split('x'))
        return cls(t, h, w)

    def transposed(self) -> TileShape:
        return TileShape(self.t, self.w, self.h)

    def padded_grid(self, grid: Sequence[int]) -> tuple[int, int, int]:
        return tuple(-(-g // s) * s for g, s in zip(grid, (self.t, self.h,
                                                          self.w)))

    def num_tiles(self, grid: Sequence[int]) -> int:
        tp, hp, wp = self.padded_grid(grid)
        return tp * hp * wp // TILE_SIZE

    def padding_ratio(self, grid: Sequence[int]) -> float:
        t, h, w = grid
        return self.num_tiles(grid) * TILE_SIZE / (t * h * w) - 1.0

    def aspect_spread(self) -> float:
        return max(self.t, self.h, self.w) / min(self.t, self.h, self.w)


def all_shapes() -> list[TileShape]:
    """All 36 power-of-two triples with product TILE_SIZE (tiling.py:85-92)."""
    exponent = TILE_SIZE.bit_length() - 1
    shapes = []
    for i, j in itertools.product(range(exponent + 1), repeat=2):
        if i + j <= exponent:
            shapes.append(TileShape(2**i, 2**j, 2**(exponent - i - j)))
    return sorted(shapes)


def candidate_shapes(grid: Sequence[int]) -> list[TileShape]:
    return [s for s in all_shapes()
            if s.t <= grid[0] and s.h <= grid[1] and s.w <= grid[2]]


def least_padding_shape(grid: Sequence[int]) -> TileShape:
    """Least padding; ties by the most cubic, then lexicographic
    (tiling.py:101-105)."""
    shapes = candidate_shapes(grid) or all_shapes()
    return min(shapes, key=lambda s: (s.num_tiles(grid), s.aspect_spread(),
                                      (s.t, s.h, s.w)))


@dataclasses.dataclass(frozen=True)
class TiledSpan:
    """A span of packed rows [start, start + T*H*W) tiled with `shape`."""

    start: int
    grid: tuple[int, int, int]
    shape: TileShape

    @property
    def num_rows(self) -> int:
        t, h, w = self.grid
        return t * h * w


@dataclasses.dataclass
class TileLayout:
    """One permutation of the packed sequence and its derived constants
    (same fields as tiling.py:159-211)."""

    perm: torch.Tensor
    valid_count: torch.Tensor
    n_video_tiles: int
    n_ref_tiles: int
    n_global_tiles: int
    ref_tokens: int
    target_tokens: int
    used: int
    seq_len: int
    gather_index: torch.Tensor
    scatter_index: torch.Tensor
    pad_slots: torch.Tensor
    partial_tiles: torch.Tensor
    kv_ok: torch.Tensor
    full_tile: torch.Tensor
    slot_valid: torch.Tensor
    # The spans this layout tiles, and the same tiles in box order for the
    # attention that reads the packed tensors in place: box_perm
    # [n_tiles * 128] int64 (packed row of every box slot, -1 outside the
    # grid; global tiles as in perm) and key_mask [n_tiles * 4] int32 (bit
    # slot % 32 of word slot // 32 set for real rows).
    spans: tuple = ()
    box_perm: torch.Tensor | None = None
    key_mask: torch.Tensor | None = None
    # Balanced forward work orders, built once per (heads, SMs, budgets).
    work_orders: dict = dataclasses.field(default_factory=dict)

    @property
    def n_tiles(self) -> int:
        return self.n_video_tiles + self.n_global_tiles

    @property
    def num_slots(self) -> int:
        return self.n_tiles * TILE_SIZE


def _check_spans(spans: Sequence[TiledSpan], used: int) -> None:
    if not spans:
        raise ValueError('at least the target span must be tiled')
    prev_stop = 0
    for span in spans:
        if span.start < prev_stop or span.start + span.num_rows > used:
            raise ValueError(f'span {span} overlaps or exceeds used={used}')
        prev_stop = span.start + span.num_rows


def layout_counts(spans: Sequence[TiledSpan], used: int) -> tuple[int, ...]:
    """(n_video_tiles, n_ref_tiles, n_global_tiles) without building it."""
    _check_spans(spans, used)
    counts = [s.shape.num_tiles(s.grid) for s in spans]
    covered = sum(s.num_rows for s in spans)
    n_global = -(-(used - covered) // TILE_SIZE)
    return sum(counts), sum(counts[:-1]), n_global


def span_array(spans: Sequence[TiledSpan]):
    """The spans as a ctypes veda_span_t array."""
    arr = (_lib.Span * len(spans))()
    for i, s in enumerate(spans):
        arr[i].start = s.start
        arr[i].grid[:] = list(s.grid)
        arr[i].shape[:] = [s.shape.t, s.shape.h, s.shape.w]
    return arr


def build_tile_layout(spans: Sequence[TiledSpan], used: int, seq_len: int,
                      device: torch.device | str = 'cuda') -> TileLayout:
    """Builds the permutation for tiled spans on a CUDA device
    (tiling.py:214-275).

    Raises:
        ValueError: If spans overlap, are out of order or exceed `used`.
        RuntimeError: Without a CUDA device (the permutation is a kernel).
    """
    n_video, n_ref, n_global = layout_counts(spans, used)
    device = torch.device(device)
    if device.type != 'cuda':
        raise RuntimeError('build_tile_layout runs on a CUDA device; '
                           f'{device} has no kernel (no CPU fallback)')
    n_tiles = n_video + n_global
    arr = span_array(spans)
    perm = torch.empty(n_tiles * TILE_SIZE, dtype=torch.int64, device=device)
    valid_count = torch.empty(n_tiles, dtype=torch.int32, device=device)
    box_perm = torch.empty_like(perm)
    key_mask = torch.empty(n_tiles * 4, dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        _lib.call('veda_build_layout', arr, len(spans), used, seq_len,
                  n_tiles, perm.data_ptr(), valid_count.data_ptr(),
                  _lib.stream_ptr(device))
        _lib.call('veda_build_box_layout', arr, len(spans), used, seq_len,
                  n_tiles, box_perm.data_ptr(), key_mask.data_ptr(),
                  _lib.stream_ptr(device))
    return TileLayout(
        perm=perm, valid_count=valid_count, n_video_tiles=n_video,
        n_ref_tiles=n_ref, n_global_tiles=n_global,
        ref_tokens=sum(s.num_rows for s in spans[:-1]),
        target_tokens=spans[-1].num_rows, used=used, seq_len=seq_len,
        gather_index=perm.clamp(min=0),
        scatter_index=torch.where(perm < 0, seq_len, perm),
        pad_slots=torch.nonzero(perm < 0).view(-1),
        partial_tiles=torch.nonzero(
            (valid_count > 0) & (valid_count < TILE_SIZE)).view(-1),
        kv_ok=valid_count > 0,
        full_tile=valid_count == TILE_SIZE,
        slot_valid=(perm >= 0).to(torch.int32),
        spans=tuple(spans), box_perm=box_perm, key_mask=key_mask)


def _heads_arg(x: torch.Tensor, heads: torch.Tensor | None):
    if heads is None:
        heads = torch.arange(x.shape[1], device=x.device)
    return heads.to(device=x.device, dtype=torch.int64).contiguous()


def _check_rows(x: torch.Tensor, name: str) -> None:
    if x.dim() != 3 or x.shape[-1] != 128 or x.stride(-1) != 1:
        raise ValueError(f'{name} must be [rows, heads, 128] with a '
                         'contiguous head dim')
    if x.dtype != torch.bfloat16:
        raise NotImplementedError(f'{name}: the kernels take bf16, got '
                                  f'{x.dtype}')
    if not x.is_cuda:
        raise RuntimeError(f'{name} is on {x.device}; the permutation '
                           'kernels run on CUDA only')


def gather_and_pool(x: torch.Tensor, layout: TileLayout,
                    heads: torch.Tensor | None, pool: bool = True,
                    second: bool = False):
    """tiling.gather_tiles and predictor.pool_tiles in one kernel pass
    (kernels/tile_gather_triton.py:162-209).

    Returns rows [N, H', D] and, with `pool`, features [H', n, 3D] fp32
    (plus E[x^2] and Var(x) [H', n, D] with `second`).
    """
    _check_rows(x, 'x')
    heads = _heads_arg(x, heads)
    n_heads = heads.numel()
    out = torch.empty(layout.num_slots, n_heads, x.shape[-1], dtype=x.dtype,
                      device=x.device)
    feats = sq = var = None
    if pool:
        feats = torch.empty(n_heads, layout.n_tiles, 3 * x.shape[-1],
                            dtype=torch.float32, device=x.device)
    if second:
        sq = torch.empty(n_heads, layout.n_tiles, x.shape[-1],
                         dtype=torch.float32, device=x.device)
        var = torch.empty_like(sq)
    _lib.call('veda_gather_pool', x.data_ptr(), x.stride(0), x.stride(1),
              layout.perm.data_ptr(), layout.valid_count.data_ptr(),
              layout.n_tiles, heads.data_ptr(), n_heads, out.data_ptr(),
              out.stride(0), out.stride(1), _lib.ptr(feats), _lib.ptr(sq),
              _lib.ptr(var), _lib.stream_ptr(x.device))
    if not pool:
        return out
    return (out, feats, sq, var) if second else (out, feats)


def gather_images(x: torch.Tensor, layout: TileLayout,
                  heads: torch.Tensor | None, pool: bool = False):
    """`gather_and_pool` with the tiles written as shared-memory images
    [H', n_tiles, 2, 128, 64] bf16 (one contiguous 32 KB block per tile
    and head, its 128-byte rows swizzled as a TMA load lays them out): the
    key / value input of `kernels.block_sparse_attention_packed`. With
    `pool`, also returns the features [H', n, 3D]."""
    _check_rows(x, 'x')
    heads = _heads_arg(x, heads)
    n_heads = heads.numel()
    image = torch.empty(n_heads, layout.n_tiles, 2, TILE_SIZE, 64,
                        dtype=x.dtype, device=x.device)
    feats = (torch.empty(n_heads, layout.n_tiles, 3 * x.shape[-1],
                         dtype=torch.float32, device=x.device)
             if pool else None)
    _lib.call('veda_gather_pool_images', x.data_ptr(), x.stride(0),
              x.stride(1), layout.perm.data_ptr(),
              layout.valid_count.data_ptr(), layout.n_tiles, heads.data_ptr(),
              n_heads, image.data_ptr(), _lib.ptr(feats),
              _lib.stream_ptr(x.device))
    return (image, feats) if pool else image


def pool_features(x: torch.Tensor, layout: TileLayout,
                  heads: torch.Tensor | None) -> torch.Tensor:
    """predictor.pool_tiles of x [S, H, D] read in place: features
    [H', n, 3D] fp32 (masked mean | max | min per tile), without writing a
    tile-ordered copy (the input of the packed attention path)."""
    _check_rows(x, 'x')
    heads = _heads_arg(x, heads)
    n_heads = heads.numel()
    feats = torch.empty(n_heads, layout.n_tiles, 3 * x.shape[-1],
                        dtype=torch.float32, device=x.device)
    _lib.call('veda_gather_pool', x.data_ptr(), x.stride(0), x.stride(1),
              layout.perm.data_ptr(), layout.valid_count.data_ptr(),
              layout.n_tiles, heads.data_ptr(), n_heads, None, 0, 0,
              feats.data_ptr(), None, None, _lib.stream_ptr(x.device))
    return feats


def gather_tiles(x: torch.Tensor, layout: TileLayout,
                 heads: torch.Tensor | None) -> torch.Tensor:
    """Permutes rows of x [S, H, D] into tile order [N, H', D], zeroing
    padding slots (tiling.py:278-297)."""
    return gather_and_pool(x, layout, heads, pool=False)


def tile_rows_perm(layout: TileLayout, rows: torch.Tensor
                   ) -> tuple[torch.Tensor, torch.Tensor]:
    """(perm [R * 128], valid_count [R]) of the tiles `rows` alone: the
    packed row of every slot of those tiles (-1 on padding)."""
    rows = rows.to(device=layout.perm.device, dtype=torch.int64)
    perm = layout.perm.view(-1, TILE_SIZE).index_select(0, rows)
    return (perm.reshape(-1).contiguous(),
            layout.valid_count.index_select(0, rows).contiguous())


def gather_tile_rows(x: torch.Tensor, layout: TileLayout, rows: torch.Tensor,
                     heads: torch.Tensor | None) -> torch.Tensor:
    """The tiles `rows` of the tile order only: x [S, H, D] ->
    [R * 128, H', D], padding slots zero. Equals
    `gather_tiles(x, layout, heads)` indexed by those tiles' slots, without
    permuting the rest (the row-subset input of the search's forward)."""
    _check_rows(x, 'x')
    heads = _heads_arg(x, heads)
    perm, valid = tile_rows_perm(layout, rows)
    n_rows = valid.numel()
    out = torch.empty(n_rows * TILE_SIZE, heads.numel(), x.shape[-1],
                      dtype=x.dtype, device=x.device)
    if n_rows == 0:
        return out
    _lib.call('veda_gather_pool', x.data_ptr(), x.stride(0), x.stride(1),
              perm.data_ptr(), valid.data_ptr(), n_rows, heads.data_ptr(),
              heads.numel(), out.data_ptr(), out.stride(0), out.stride(1),
              None, None, None, _lib.stream_ptr(x.device))
    return out


def scatter_tiles_(out: torch.Tensor, tiled: torch.Tensor,
                   layout: TileLayout, heads: torch.Tensor | None) -> None:
    """Writes tile-ordered rows back into out[S + 1, H, D] in place
    (tiling.py:300-312). Real rows are written; padding slots belong to the
    discarded row out[S], which this kernel leaves untouched."""
    if out.shape[0] != layout.seq_len + 1:
        raise ValueError(f'scatter buffer needs {layout.seq_len + 1} rows')
    scatter_rows_(out, tiled, layout, heads)


def scatter_rows_(out: torch.Tensor, tiled: torch.Tensor, layout: TileLayout,
                  heads: torch.Tensor | None) -> None:
    """The inverse permutation into out[>= S, H, D] (real rows only)."""
    _check_rows(out, 'out')
    _check_rows(tiled, 'tiled')
    heads = _heads_arg(out, heads)
    if tiled.shape[0] != layout.num_slots or tiled.shape[1] != heads.numel():
        raise ValueError('tiled must be [num_slots, len(heads), D]')
    _lib.call('veda_scatter', tiled.data_ptr(), tiled.stride(0),
              tiled.stride(1), layout.perm.data_ptr(), layout.n_tiles,
              heads.data_ptr(), heads.numel(), out.data_ptr(), out.stride(0),
              out.stride(1), _lib.stream_ptr(out.device))


def gather_lse(lse: torch.Tensor, layout: TileLayout,
               heads: torch.Tensor) -> torch.Tensor:
    """[S, H] LSE -> [N, H'] tile order, 0 on padding slots
    (veda/attention.py:299-305)."""
    if lse.dtype != torch.float32 or lse.dim() != 2:
        raise ValueError('lse must be [S, H] float32')
    heads = _heads_arg(lse[:, :, None], heads)
    out = torch.empty(layout.num_slots, heads.numel(), dtype=torch.float32,
                      device=lse.device)
    _lib.call('veda_gather_lse', lse.data_ptr(), lse.stride(0), lse.stride(1),
              layout.perm.data_ptr(), layout.n_tiles, heads.data_ptr(),
              heads.numel(), out.data_ptr(), _lib.stream_ptr(lse.device))
    return out

