"""Block masks from tile scores: budgets, top-k selection, block lists.

Mirror of the reference's `miowtion/veda/mask.py` (rules 1-7 of its module
docstring, same names and errors). Budgets are resolved on the host in fp64
exactly as the reference does; selection runs in one CUDA kernel
(csrc/select.cu), which can also emit the block mask and the full/partial
index lists directly, so the sparse path never materialises a Selection.

The reference's default rule 'topk' runs entirely in that kernel; its
'threshold' rule (an ablation arm) ranks candidates in it and sets each
row's count with a per-head threshold in torch.
"""

from __future__ import annotations

import dataclasses
import functools
import math

import torch

from miowtion_b200 import _lib
from miowtion_b200 import tiling


@dataclasses.dataclass(frozen=True)
class Budget:
    """Keep budget of one column block: a ratio or an absolute tile count
    (mask.py:38-65)."""

    ratio: float | None = None
    tiles: float | None = None

    def __post_init__(self):
        if (self.ratio is None) == (self.tiles is None):
            raise ValueError('set exactly one of ratio / tiles')
        value = self.ratio if self.tiles is None else self.tiles
        if value <= 0:
            raise ValueError(f'budget must be positive: {self}')

    @property
    def keeps_all(self) -> bool:
        return self.ratio is not None and self.ratio >= 1.0

    def per_row(self, real_tokens: int, n_tiles: int) -> float:
        if self.tiles is not None:
            return float(self.tiles)
        n_ideal = math.ceil(real_tokens / tiling.TILE_SIZE)
        return self.ratio * n_ideal * n_ideal / n_tiles


def split_budget(budget: float, n_cols: int) -> tuple[int, int, float]:
    """(k_lo, k_hi, frac) with 1 <= k_lo <= k_hi <= n_cols (mask.py:68-76)."""
    if budget >= n_cols:
        return n_cols, n_cols, 0.0
    k_lo = min(max(1, math.floor(budget)), n_cols)
    frac = round(min(max(budget - k_lo, 0.0), 1.0), 12)
    return k_lo, min(k_lo + 1, n_cols), frac


@functools.lru_cache(maxsize=256)
def _bresenham(n_rows: int, frac: float, device: str) -> torch.Tensor:
    ramp = torch.floor(torch.arange(n_rows + 1, dtype=torch.float64) * frac)
    return (ramp[1:] > ramp[:-1]).to(device)


def bresenham_extra(n_rows: int, frac: float,
                    device: torch.device | str) -> torch.Tensor:
    """[n_rows] bool: row r keeps k_hi iff floor((r+1)f) > floor(r f)
    (mask.py:79-93). The selection kernel evaluates the same fp64 expression
    per row; this host copy serves callers of the reference API."""
    return _bresenham(n_rows, float(frac), str(torch.device(device)))


@dataclasses.dataclass(frozen=True)
class ColumnBlock:
    """A sparse column block of the video quadrant (mask.py:96-103)."""

    start: int
    stop: int
    budget: Budget
    real_tokens: int


def column_blocks(layout: tiling.TileLayout, target_budget: Budget,
                  ref_budget: Budget | None = None) -> list[ColumnBlock]:
    """Target block, preceded by a reference block when references are
    tiled (mask.py:106-120)."""
    target = ColumnBlock(layout.n_ref_tiles, layout.n_video_tiles,
                         target_budget, layout.target_tokens)
    if layout.n_ref_tiles == 0:
        return [target]
    if ref_budget is None:
        raise ValueError('tiled references need their own budget')
    return [ColumnBlock(0, layout.n_ref_tiles, ref_budget, layout.ref_tokens),
            target]


@dataclasses.dataclass
class Selection:
    """Selected video key tiles per video query tile (mask.py:123-134)."""

    index: torch.Tensor
    keep: torch.Tensor


def resolve_blocks(blocks: list[ColumnBlock]):
    """ctypes array of the blocks with their budgets split (host fp64)."""
    arr = (_lib.ColumnBlockC * len(blocks))()
    for i, b in enumerate(blocks):
        n_cols = b.stop - b.start
        arr[i].start, arr[i].stop = b.start, b.stop
        if b.budget.keeps_all:
            arr[i].k_lo = arr[i].k_hi = n_cols
            arr[i].frac = 0.0
            arr[i].keeps_all = 1
            continue
        k_lo, k_hi, frac = split_budget(
            b.budget.per_row(b.real_tokens, n_cols), n_cols)
        arr[i].k_lo, arr[i].k_hi, arr[i].frac = k_lo, k_hi, frac
        arr[i].keeps_all = 0
    return arr


def _selection_width(blocks: list[ColumnBlock]) -> int:
    width = 0
    for b in blocks:
        n_cols = b.stop - b.start
        if b.budget.keeps_all:
            width += n_cols
        else:
            width += split_budget(b.budget.per_row(b.real_tokens, n_cols),
                                  n_cols)[1]
    return width


def _check_scores(scores: torch.Tensor, layout: tiling.TileLayout,
                  num_rows: int) -> torch.Tensor:
    if scores.dim() != 3:
        raise ValueError('scores must be [H\', R, >= n_video]')
    if scores.shape[1] != num_rows:
        raise ValueError(
            f'scores has {scores.shape[1]} query rows but rows has '
            f'{num_rows}; index the query axis by `rows` before calling')
    if scores.shape[2] < layout.n_video_tiles:
        raise ValueError('scores must cover the video columns')
    if not scores.is_cuda:
        raise RuntimeError('selection runs on CUDA only (no CPU fallback)')
    scores = scores.float()
    if scores.stride(2) != 1 or scores.stride(1) != scores.shape[2] or (
            scores.stride(0) != scores.shape[1] * scores.shape[2]):
        scores = scores.contiguous()
    return scores


def _rows_arg(rows, layout, device):
    if rows is None:
        return None, layout.n_video_tiles
    rows = rows.to(device=device, dtype=torch.int64).contiguous()
    return rows, rows.numel()


# [rows whose threshold count reached the widened cap, rows seen] of the
# 'threshold' rule (mask.py:136-140); reading it synchronises the host.
SATURATED = [0, 0]


def threshold_allowed(sorted_scores: torch.Tensor, valid: torch.Tensor,
                      mean_k: float, cap: int) -> torch.Tensor:
    """Kept count per row [H', R] of the 'threshold' rule (mask.py:143-197).

    Each row's candidates (descending, forced columns +inf) are
    standardised over its valid, non-forced entries (sample variance, at
    least 2 counted); the head's threshold is its round(mean_k * R)-th
    largest standardised score over all rows, so the head spends the top-k
    total unevenly across rows. A row keeps its candidates at or above the
    threshold, at least 1.
    """
    counts = valid.sum(-1, keepdim=True).clamp(min=2).float()
    x = torch.where(valid, sorted_scores.float(), 0.0)
    forced = torch.isposinf(x)
    x = torch.where(forced, 0.0, x)
    n_stat = (counts - forced.sum(-1, keepdim=True)).clamp(min=2)
    mean = x.sum(-1, keepdim=True) / n_stat
    var = torch.where(valid & ~forced, (x - mean).square(), 0.0).sum(
        -1, keepdim=True) / (n_stat - 1)
    z = (sorted_scores.float() - mean) / var.sqrt().clamp(min=1e-12)
    z = torch.where(valid, z, float('-inf'))
    z = torch.where(forced, float('inf'), z)
    heads, rows, width = z.shape
    total = max(1, min(int(round(float(mean_k) * rows)), width * rows))
    cut = z.reshape(heads, -1).topk(total, dim=-1).values[:, -1:]
    allowed = (z >= cut[:, :, None]).sum(-1)
    SATURATED[0] += int((allowed >= cap).sum())
    SATURATED[1] += heads * rows
    return allowed.clamp(min=1)


def _select_threshold(scores, layout, blocks, rows, cap_mult):
    """The 'threshold' rule: the selection kernel ranks each block's top
    ceil(cap_mult * budget) candidates (at least the top-k width) in the
    reference's order, and `threshold_allowed` sets each row's count."""
    wide, widths = [], []
    for b in blocks:
        n_cols = b.stop - b.start
        if b.budget.keeps_all:
            wide.append(b)
            widths.append(None)
            continue
        budget = b.budget.per_row(b.real_tokens, n_cols)
        k_hi = split_budget(budget, n_cols)[1]
        k_wide = min(n_cols, max(k_hi, math.ceil(cap_mult * budget)))
        wide.append(ColumnBlock(b.start, b.stop, Budget(tiles=k_wide),
                                b.real_tokens))
        widths.append((k_wide, budget))
    ranked = select_video_blocks(scores, layout, wide, rows)
    rows_t = (torch.arange(layout.n_video_tiles, device=scores.device)
              if rows is None else rows.to(device=scores.device,
                                           dtype=torch.int64))
    indices, keeps, off = [], [], 0
    for b, w, b_wide in zip(blocks, widths, wide):
        span = _selection_width([b_wide])
        if w is None:
            indices.append(ranked.index[..., off:off + span])
            keeps.append(ranked.keep[..., off:off + span])
            off += span
            continue
        k_wide, budget = w
        idx = ranked.index[..., off:off + k_wide]
        off += span
        s = scores[:, :, b.start:b.stop].float().masked_fill(
            ~layout.kv_ok[None, None, b.start:b.stop], float('-inf'))
        own = (rows_t >= b.start) & (rows_t < b.stop)
        # Each row's own column to +inf when the row lies in this block,
        # without a boolean index (which would wait on the host for its
        # count): gather the diagonal entry, replace it, scatter it back.
        col = (rows_t - b.start).clamp(0, b.stop - b.start - 1)
        col = col[None, :, None].expand(s.shape[0], -1, 1)
        s.scatter_(-1, col, torch.where(own[None, :, None], float('inf'),
                                        s.gather(-1, col)))
        vals = s.gather(-1, idx - b.start)
        live = vals > float('-inf')
        allowed = threshold_allowed(vals, live, budget, k_wide)
        keeps.append((torch.arange(k_wide, device=scores.device)
                      < allowed[:, :, None]) & live)
        indices.append(idx)
    return Selection(torch.cat(indices, -1), torch.cat(keeps, -1))


@torch.no_grad()
def select_video_blocks(scores: torch.Tensor, layout: tiling.TileLayout,
                        blocks: list[ColumnBlock],
                        rows: torch.Tensor | None = None,
                        rule: str = 'topk',
                        cap_mult: float = 4.0) -> Selection:
    """Top-k over the video quadrant of `scores` (mask.py:200-285); with
    rule 'threshold' each row's count follows `threshold_allowed`, capped
    at cap_mult times the block's mean budget."""
    if rule not in ('topk', 'threshold'):
        raise ValueError(f"rule must be 'topk' or 'threshold': {rule!r}")
    if rule == 'threshold':
        _check_scores(scores, layout, layout.n_video_tiles if rows is None
                      else rows.numel())
        return _select_threshold(scores, layout, blocks, rows, cap_mult)
    rows_t, num_rows = _rows_arg(rows, layout, scores.device)
    scores = _check_scores(scores, layout, num_rows)
    heads = scores.shape[0]
    width = _selection_width(blocks)
    index = torch.empty(heads, num_rows, width, dtype=torch.int64,
                        device=scores.device)
    keep = torch.empty(heads, num_rows, width, dtype=torch.uint8,
                       device=scores.device)
    arr = resolve_blocks(blocks)
    _lib.call('veda_block_select', scores.data_ptr(), scores.shape[2], heads,
              num_rows, _lib.ptr(rows_t), layout.valid_count.data_ptr(),
              layout.n_tiles, layout.n_video_tiles, arr, len(blocks), 0,
              None, None, None, None, None, 0, index.data_ptr(),
              keep.data_ptr(), _lib.stream_ptr(scores.device))
    return Selection(index, keep.bool())


@torch.no_grad()
def dense_block_mask(selection: Selection, layout: tiling.TileLayout,
                     global_rows: bool = True) -> torch.Tensor:
    """Block mask of a selection (mask.py:288-317): [H', n, n] bool, or
    [H', R, n] without global rows."""
    heads, num_rows, _ = selection.index.shape
    n, n_video = layout.n_tiles, layout.n_video_tiles
    if global_rows and num_rows != n_video:
        raise ValueError('global_rows needs a selection of all video rows')
    mask = torch.zeros(heads, n if global_rows else num_rows, n,
                       dtype=torch.bool, device=selection.index.device)
    mask[:, :num_rows].scatter_(2, selection.index, selection.keep)
    mask[:, :, n_video:] = layout.kv_ok[n_video:]
    if global_rows:
        mask[:, n_video:, :] = layout.kv_ok
    return mask


@dataclasses.dataclass
class BlockLists:
    """Full / partial index lists in BlockSparseTensors order
    (kernels/fa4.py:286-288), each [H', R(, n)] int32, plus the row stride of
    the idx tensors. `mask` is set when it was requested."""

    part_cnt: torch.Tensor
    part_idx: torch.Tensor
    full_cnt: torch.Tensor
    full_idx: torch.Tensor
    mask: torch.Tensor | None = None

    def as_fa4(self) -> tuple[torch.Tensor, ...]:
        """(partial_cnt, partial_idx, full_cnt, full_idx) with the leading
        batch axis of the reference ([1, H', R] / [1, H', R, n])."""
        return (self.part_cnt[None], self.part_idx[None],
                self.full_cnt[None], self.full_idx[None])


@torch.no_grad()
def select_block_lists(scores: torch.Tensor, layout: tiling.TileLayout,
                       blocks: list[ColumnBlock],
                       rows: torch.Tensor | None = None,
                       global_rows: bool = True, want_mask: bool = False,
                       fill_tails: bool = False) -> BlockLists:
    """select_video_blocks -> dense_block_mask -> fa4.index_lists fused.

    Returns the lists the sparse kernel walks (rows = all video query tiles
    plus, with `global_rows`, the dense global ones). `fill_tails` writes the
    non-member columns after the members like the reference's argsort; the
    attention kernel reads only the first cnt entries.
    """
    rows_t, num_rows = _rows_arg(rows, layout, scores.device)
    scores = _check_scores(scores, layout, num_rows)
    heads = scores.shape[0]
    if global_rows and num_rows != layout.n_video_tiles:
        raise ValueError('global_rows needs a selection of all video rows')
    rows_out = num_rows + (layout.n_global_tiles if global_rows else 0)
    n = layout.n_tiles
    dev = scores.device
    lists = BlockLists(
        part_cnt=torch.empty(heads, rows_out, dtype=torch.int32, device=dev),
        part_idx=torch.empty(heads, rows_out, n, dtype=torch.int32,
                             device=dev),
        full_cnt=torch.empty(heads, rows_out, dtype=torch.int32, device=dev),
        full_idx=torch.empty(heads, rows_out, n, dtype=torch.int32,
                             device=dev))
    if want_mask:
        lists.mask = torch.empty(heads, rows_out, n, dtype=torch.uint8,
                                 device=dev)
    arr = resolve_blocks(blocks)
    _lib.call('veda_block_select', scores.data_ptr(), scores.shape[2], heads,
              num_rows, _lib.ptr(rows_t), layout.valid_count.data_ptr(),
              n, layout.n_video_tiles, arr, len(blocks),
              1 if global_rows else 0, _lib.ptr(lists.mask),
              lists.part_cnt.data_ptr(), lists.part_idx.data_ptr(),
              lists.full_cnt.data_ptr(), lists.full_idx.data_ptr(),
              1 if fill_tails else 0, None, None, _lib.stream_ptr(dev))
    return lists


def kept_tiles_per_row(selection: Selection) -> torch.Tensor:
    """[H', n_video] number of selected video tiles (mask.py:320-322)."""
    return selection.keep.sum(-1)
