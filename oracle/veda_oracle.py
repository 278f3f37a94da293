"""CPU oracle for the Veda sparse-attention hot path (TEST INFRASTRUCTURE ONLY).

This module is a numpy restatement of the reference algorithm
(veda-sparse/Miowtion, `miowtion/veda/*` and `miowtion/kernels/reference.py`).
It exists to check the CUDA product path; it is never the thing measured or
shipped. Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU
baseline leg may import it.

Parity of this restatement is pinned against golden vectors produced by the
reference itself (`tests/golden/make_golden.py` imports the reference's own
Python and writes `tests/golden/*.npz`; `tests/test_oracle_golden.py` checks
this module against them).

Conventions:
  * Arrays are numpy. Token tensors are [rows, heads, head_dim].
  * Integer/index outputs follow the reference's dtypes (int64 for perm and
    selection indices, int32 for counts and index lists).
  * bf16 inputs are represented as float32 arrays holding bf16-representable
    values (see `round_bf16`).
  * Ties in top-k are broken lowest-index-first (`torch.topk` leaves the order
    of equal values unspecified; the reference's parity inputs have no ties).
"""

from __future__ import annotations

import dataclasses
import math

import numpy as np

TILE = 128  # miowtion/veda/tiling.py:34-40 (MIOWTION_TILE_SIZE default)


# ---------------------------------------------------------------------------
# numeric helpers
# ---------------------------------------------------------------------------

def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), as float32.

    This is what `tensor.to(torch.bfloat16)` does; used to emulate the
    reference's bf16 inputs and its bf16 `bmm` outputs.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) >> 16) << 16
    nan = np.isnan(x)
    out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


# ---------------------------------------------------------------------------
# a1: tiling (miowtion/veda/tiling.py)
# ---------------------------------------------------------------------------

@dataclasses.dataclass(frozen=True)
class Span:
    """A tiled span of packed rows (tiling.py:108-119, `TiledSpan`)."""

    start: int
    grid: tuple
    shape: tuple

    @property
    def num_rows(self) -> int:
        t, h, w = self.grid
        return t * h * w


def padded_grid(grid, shape):
    """tiling.py:67-69."""
    return tuple(-(-g // s) * s for g, s in zip(grid, shape))


def num_tiles(grid, shape) -> int:
    """tiling.py:71-73."""
    tp, hp, wp = padded_grid(grid, shape)
    return tp * hp * wp // TILE


def span_tiles(span: Span) -> np.ndarray:
    """[n_tiles, 128] packed rows of one span, -1 on padding (tiling.py:122-136).

    Tile order is (h-block, w-block, t-block); rows inside a tile are
    t, h, w row-major, then stably compacted so real rows form a prefix.
    """
    t, h, w = span.grid
    st, sh, sw = span.shape
    tp, hp, wp = padded_grid(span.grid, span.shape)
    grid = np.full((tp, hp, wp), -1, dtype=np.int64)
    grid[:t, :h, :w] = span.start + np.arange(t * h * w).reshape(t, h, w)
    tiles = grid.reshape(tp // st, st, hp // sh, sh, wp // sw, sw)
    tiles = tiles.transpose(2, 4, 0, 1, 3, 5).reshape(-1, TILE)
    order = np.argsort((tiles < 0).astype(np.int8), axis=1, kind='stable')
    return np.take_along_axis(tiles, order, axis=1)


@dataclasses.dataclass
class Layout:
    """Mirror of `TileLayout` (tiling.py:159-211)."""

    perm: np.ndarray
    valid_count: np.ndarray
    n_video_tiles: int
    n_ref_tiles: int
    n_global_tiles: int
    ref_tokens: int
    target_tokens: int
    used: int
    seq_len: int

    @property
    def n_tiles(self) -> int:
        return self.n_video_tiles + self.n_global_tiles

    @property
    def num_slots(self) -> int:
        return self.n_tiles * TILE

    @property
    def gather_index(self):
        return np.maximum(self.perm, 0)

    @property
    def scatter_index(self):
        return np.where(self.perm < 0, self.seq_len, self.perm)

    @property
    def pad_slots(self):
        return np.nonzero(self.perm < 0)[0]

    @property
    def partial_tiles(self):
        vc = self.valid_count
        return np.nonzero((vc > 0) & (vc < TILE))[0]

    @property
    def kv_ok(self):
        return self.valid_count > 0

    @property
    def full_tile(self):
        return self.valid_count == TILE

    @property
    def slot_valid(self):
        return (self.perm >= 0).astype(np.int32)


def build_tile_layout(spans, used: int, seq_len: int) -> Layout:
    """tiling.py:214-275: spans in packed order, the last is the target."""
    if not spans:
        raise ValueError('at least the target span must be tiled')
    covered = np.zeros(used, dtype=bool)
    tiles = []
    prev_stop = 0
    for span in spans:
        if span.start < prev_stop or span.start + span.num_rows > used:
            raise ValueError(f'span {span} overlaps or exceeds used={used}')
        prev_stop = span.start + span.num_rows
        covered[span.start:prev_stop] = True
        tiles.append(span_tiles(span))
    n_ref_tiles = sum(t.shape[0] for t in tiles[:-1])
    video = np.concatenate(tiles)
    global_rows = np.nonzero(~covered)[0]
    n_global = -(-global_rows.size // TILE)
    global_tiles = np.full(n_global * TILE, -1, dtype=np.int64)
    global_tiles[:global_rows.size] = global_rows
    perm = np.concatenate([video.reshape(-1), global_tiles])
    valid_count = (perm.reshape(-1, TILE) >= 0).sum(1).astype(np.int32)
    return Layout(perm=perm, valid_count=valid_count,
                  n_video_tiles=video.shape[0], n_ref_tiles=n_ref_tiles,
                  n_global_tiles=n_global,
                  ref_tokens=sum(s.num_rows for s in spans[:-1]),
                  target_tokens=spans[-1].num_rows, used=used,
                  seq_len=seq_len)


def gather_tiles(x: np.ndarray, layout: Layout, heads=None) -> np.ndarray:
    """tiling.py:278-297: [S,H,D] -> [N,H',D], padding slots zero."""
    out = x[layout.gather_index]
    if heads is not None:
        out = out[:, np.asarray(heads)]
    out = out.copy()
    out[layout.pad_slots] = 0
    return out


def scatter_tiles(out: np.ndarray, tiled: np.ndarray, layout: Layout,
                  heads=None) -> None:
    """tiling.py:300-312: writes into out[S+1,H,D]; padding -> row S."""
    if out.shape[0] != layout.seq_len + 1:
        raise ValueError(f'scatter buffer needs {layout.seq_len + 1} rows')
    idx = layout.scatter_index
    if heads is None:
        out[idx] = tiled
    else:
        heads = np.asarray(heads)
        out[idx[:, None], heads[None, :]] = tiled


def gather_lse(lse: np.ndarray, layout: Layout, heads) -> np.ndarray:
    """veda/attention.py:299-305: [S,H] -> [N,H'], 0 on padding slots."""
    out = lse[layout.gather_index][:, np.asarray(heads)].copy()
    out[layout.pad_slots] = 0.0
    return out


# ---------------------------------------------------------------------------
# a3/a4: pooling and predictor (miowtion/veda/predictor.py)
# ---------------------------------------------------------------------------

def pool_tiles(tiles: np.ndarray, layout: Layout, second=None) -> np.ndarray:
    """predictor.py:82-168: masked mean|max|min -> [H', n, 3D] fp32.

    `second='raw'` returns E[x^2], `'central'` the centred Var(x), each
    [H', n, D]; empty tiles are exactly 0.
    """
    n = layout.n_tiles
    heads, dim = tiles.shape[1], tiles.shape[2]
    x = tiles.reshape(n, TILE, heads, dim).astype(np.float64)
    vc = layout.valid_count.astype(np.int64)
    valid = np.arange(TILE)[None, :] < vc[:, None]            # [n, 128]
    count = np.maximum(vc, 1).astype(np.float64)
    mean = x.sum(1) / count[:, None, None]                     # [n, H, D]
    if second is None:
        vm = valid[:, :, None, None]
        tmax = np.where(vm, x, -np.inf).max(1)
        tmin = np.where(vm, x, np.inf).min(1)
        feats = np.concatenate([mean, tmax, tmin], axis=-1)
    elif second == 'raw':
        feats = (x * x).sum(1) / count[:, None, None]
    elif second == 'central':
        c = np.where(valid[:, :, None, None], x - mean[:, None], 0.0)
        feats = (c * c).sum(1) / count[:, None, None]
    else:
        raise ValueError(f'unknown second moment {second!r}')
    feats = np.where(layout.kv_ok[:, None, None], feats, 0.0)
    return np.ascontiguousarray(feats.transpose(1, 0, 2)).astype(np.float32)


def predictor_logits(feats_q: np.ndarray, feats_k: np.ndarray,
                     proj_q: np.ndarray, proj_k: np.ndarray,
                     heads) -> np.ndarray:
    """predictor.py:251-255 and :299-338 (no count / second-order terms).

    q_hat = feats_q @ proj_q[h] + mean_q, k_hat likewise, logits =
    q_hat . k_hat^T / sqrt(D), all fp32 (computed here in fp64).
    """
    heads = np.asarray(heads)
    dim = proj_q.shape[-1]
    fq = feats_q.astype(np.float64)
    fk = feats_k.astype(np.float64)
    pq = proj_q[heads].astype(np.float64)
    pk = proj_k[heads].astype(np.float64)
    q_hat = np.matmul(fq, pq) + fq[..., :dim]
    k_hat = np.matmul(fk, pk) + fk[..., :dim]
    logits = np.matmul(q_hat, k_hat.transpose(0, 2, 1)) / math.sqrt(dim)
    return logits.astype(np.float32)


# ---------------------------------------------------------------------------
# a5-a8: budgets, selection, block mask, index lists (miowtion/veda/mask.py,
# miowtion/kernels/fa4.py)
# ---------------------------------------------------------------------------

@dataclasses.dataclass(frozen=True)
class Budget:
    """mask.py:38-65."""

    ratio: float | None = None
    tiles: float | None = None

    @property
    def keeps_all(self) -> bool:
        return self.ratio is not None and self.ratio >= 1.0

    def per_row(self, real_tokens: int, n_tiles: int) -> float:
        if self.tiles is not None:
            return float(self.tiles)
        n_ideal = math.ceil(real_tokens / TILE)
        return self.ratio * n_ideal * n_ideal / n_tiles


def split_budget(budget: float, n_cols: int):
    """mask.py:68-76: (k_lo, k_hi, frac)."""
    if budget >= n_cols:
        return n_cols, n_cols, 0.0
    k_lo = min(max(1, math.floor(budget)), n_cols)
    frac = round(min(max(budget - k_lo, 0.0), 1.0), 12)
    return k_lo, min(k_lo + 1, n_cols), frac


def bresenham_extra(n_rows: int, frac: float) -> np.ndarray:
    """mask.py:79-93: row r keeps k_hi iff floor((r+1)f) > floor(r f), fp64."""
    ramp = np.floor(np.arange(n_rows + 1, dtype=np.float64) * frac)
    return ramp[1:] > ramp[:-1]


@dataclasses.dataclass(frozen=True)
class ColumnBlock:
    """mask.py:96-103."""

    start: int
    stop: int
    budget: Budget
    real_tokens: int


def column_blocks(layout: Layout, target_budget: Budget, ref_budget=None):
    """mask.py:106-120."""
    target = ColumnBlock(layout.n_ref_tiles, layout.n_video_tiles,
                         target_budget, layout.target_tokens)
    if layout.n_ref_tiles == 0:
        return [target]
    if ref_budget is None:
        raise ValueError('tiled references need their own budget')
    return [ColumnBlock(0, layout.n_ref_tiles, ref_budget, layout.ref_tokens),
            target]


def select_video_blocks(scores: np.ndarray, layout: Layout, blocks,
                        rows=None):
    """mask.py:200-285 (rule 'topk'): returns (index int64, keep bool).

    `scores` is [H', R, >= n_video]; rows are video query tile ids.
    """
    heads = scores.shape[0]
    n_video = layout.n_video_tiles
    rows = np.arange(n_video) if rows is None else np.asarray(rows)
    num_rows = rows.size
    if scores.shape[1] != num_rows:
        raise ValueError('scores rows must match `rows`')
    kv_ok = layout.kv_ok
    indices, keeps = [], []
    for block in blocks:
        n_cols = block.stop - block.start
        if block.budget.keeps_all:
            idx = np.broadcast_to(np.arange(block.start, block.stop),
                                  (heads, num_rows, n_cols))
            indices.append(idx)
            keeps.append(np.broadcast_to(kv_ok[block.start:block.stop],
                                         (heads, num_rows, n_cols)))
            continue
        s = scores[:, :, block.start:block.stop].astype(np.float32).copy()
        s[:, :, ~kv_ok[block.start:block.stop]] = -np.inf
        own = (rows >= block.start) & (rows < block.stop)
        for r_i in np.nonzero(own)[0]:
            s[:, r_i, rows[r_i] - block.start] = np.inf
        budget = block.budget.per_row(block.real_tokens, n_cols)
        k_lo, k_hi, frac = split_budget(budget, n_cols)
        # Descending by value, ties lowest column first.
        order = np.argsort(-s, axis=-1, kind='stable')[..., :k_hi]
        vals = np.take_along_axis(s, order, axis=-1)
        extra = bresenham_extra(n_video, frac)[rows]
        allowed = k_lo + extra.astype(np.int64)
        keep = ((np.arange(k_hi)[None, None, :] < allowed[None, :, None])
                & (vals > -np.inf))
        indices.append(order.astype(np.int64) + block.start)
        keeps.append(keep)
    return (np.concatenate(indices, -1).astype(np.int64),
            np.concatenate(keeps, -1))


def dense_block_mask(index: np.ndarray, keep: np.ndarray, layout: Layout,
                     global_rows: bool = True) -> np.ndarray:
    """mask.py:288-317: [H', n, n] (or [H', R, n]) bool."""
    heads, num_rows, _ = index.shape
    n, n_video = layout.n_tiles, layout.n_video_tiles
    if global_rows and num_rows != n_video:
        raise ValueError('global_rows needs a selection of all video rows')
    mask = np.zeros((heads, n if global_rows else num_rows, n), dtype=bool)
    h_i = np.arange(heads)[:, None, None]
    r_i = np.arange(num_rows)[None, :, None]
    mask[h_i, r_i, index] = keep
    mask[:, :, n_video:] = layout.kv_ok[n_video:]
    if global_rows:
        mask[:, n_video:, :] = layout.kv_ok
    return mask


def _pack_lists(member: np.ndarray):
    """fa4.py:266-272: left-packed ascending members, then non-members."""
    heads, rows, cols = member.shape
    order = np.argsort((~member).astype(np.int8), axis=-1, kind='stable')
    return (member.sum(-1)[None].astype(np.int32),
            order[None].astype(np.int32))


def index_lists(block_mask: np.ndarray, layout: Layout,
                transpose: bool = False):
    """fa4.py:275-296: (partial_cnt, partial_idx, full_cnt, full_idx)."""
    block_mask = block_mask & layout.kv_ok
    full = layout.full_tile
    if transpose:
        block_mask = block_mask.transpose(0, 2, 1)
        full = full[:, None]
    full_cnt, full_idx = _pack_lists(block_mask & full)
    part_cnt, part_idx = _pack_lists(block_mask & ~full)
    return part_cnt, part_idx, full_cnt, full_idx


# ---------------------------------------------------------------------------
# a9/a10: block-sparse attention (miowtion/kernels/reference.py:23-56) and its
# gradients (autograd of the same function, tests/gpu/test_kernels_gpu.py:200)
# ---------------------------------------------------------------------------

def _key_valid(valid_count: np.ndarray) -> np.ndarray:
    return (np.arange(TILE)[None, :] < valid_count[:, None]).reshape(-1)


def block_sparse_attention(q, k, v, block_mask, valid_count,
                           return_lse=False, q_tiles=None):
    """reference.py:23-56 restated per query tile (fp32 math).

    q: [R*128, H', D] (rows of query tiles `q_tiles`, default all), k, v:
    [N, H', D], block_mask [H', R, n]. Rows with no key output 0 and have
    lse -inf. Returns out [R*128, H', D] float32 (and lse [H', R*128]).
    """
    rows_total, heads, dim = q.shape
    n_q = rows_total // TILE
    scale = 1.0 / math.sqrt(dim)
    kvalid = _key_valid(np.asarray(valid_count))
    out = np.zeros((rows_total, heads, dim), dtype=np.float32)
    lse = np.full((heads, rows_total), -np.inf, dtype=np.float32)
    qf = q.astype(np.float32)
    kf = k.astype(np.float32)
    vf = v.astype(np.float32)
    for h in range(heads):
        for r in range(n_q):
            tiles = np.nonzero(block_mask[h, r])[0]
            if tiles.size == 0:
                continue
            cols = (tiles[:, None] * TILE + np.arange(TILE)[None]).reshape(-1)
            cols = cols[kvalid[cols]]
            if cols.size == 0:
                continue
            qr = qf[r * TILE:(r + 1) * TILE, h]
            s = (qr @ kf[cols, h].T) * np.float32(scale)
            m = s.max(-1, keepdims=True)
            p = np.exp(s - m)
            den = p.sum(-1, keepdims=True)
            out[r * TILE:(r + 1) * TILE, h] = (p / den) @ vf[cols, h]
            lse[h, r * TILE:(r + 1) * TILE] = (m + np.log(den))[:, 0]
    if return_lse:
        return out, lse
    return out


def block_sparse_attention_bwd(q, k, v, dout, block_mask, valid_count):
    """Gradients of reference.py:23-56 w.r.t. q, k, v (fp32 math).

    Every query row (padding rows included, exactly as autograd through the
    reference treats them) contributes to dK/dV of the keys it attends.
    """
    rows_total, heads, dim = q.shape
    n_q = rows_total // TILE
    scale = np.float32(1.0 / math.sqrt(dim))
    kvalid = _key_valid(np.asarray(valid_count))
    qf, kf, vf = (t.astype(np.float32) for t in (q, k, v))
    dof = dout.astype(np.float32)
    dq = np.zeros_like(qf)
    dk = np.zeros_like(kf)
    dv = np.zeros_like(vf)
    for h in range(heads):
        for r in range(n_q):
            tiles = np.nonzero(block_mask[h, r])[0]
            if tiles.size == 0:
                continue
            cols = (tiles[:, None] * TILE + np.arange(TILE)[None]).reshape(-1)
            cols = cols[kvalid[cols]]
            if cols.size == 0:
                continue
            sl = slice(r * TILE, (r + 1) * TILE)
            qr, do = qf[sl, h], dof[sl, h]
            kc, vc = kf[cols, h], vf[cols, h]
            s = (qr @ kc.T) * scale
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            o = p @ vc
            dp = do @ vc.T
            delta = (do * o).sum(-1, keepdims=True)
            ds = p * (dp - delta)
            dq[sl, h] += (ds @ kc) * scale
            np.add.at(dk[:, h], cols, (ds.T @ qr) * scale)
            np.add.at(dv[:, h], cols, p.T @ do)
    return dq, dk, dv


# ---------------------------------------------------------------------------
# a11: dense attention with LSE (miowtion/h3/attention.py:18-25, :28-102)
# ---------------------------------------------------------------------------

def dense_attention(q, k, v, used, return_lse=False, row_chunk=1024):
    """Full attention of rows [0, used); padding rows are 0 (lse 0)."""
    seq_len, heads, dim = q.shape
    scale = np.float32(1.0 / math.sqrt(dim))
    out = np.zeros((seq_len, heads, dim), dtype=np.float32)
    lse = np.zeros((seq_len, heads), dtype=np.float32)
    qf, kf, vf = (t[:used].astype(np.float32) for t in (q, k, v))
    for h in range(heads):
        for r0 in range(0, used, row_chunk):
            r1 = min(used, r0 + row_chunk)
            s = (qf[r0:r1, h] @ kf[:, h].T) * scale
            m = s.max(-1, keepdims=True)
            p = np.exp(s - m)
            den = p.sum(-1, keepdims=True)
            out[r0:r1, h] = (p / den) @ vf[:, h]
            lse[r0:r1, h] = (m + np.log(den))[:, 0]
    return (out, lse) if return_lse else (out, None)


# ---------------------------------------------------------------------------
# a13: teacher block heat (miowtion/veda/heatmap.py:36-99)
# ---------------------------------------------------------------------------

def teacher_heat(q, k, lse, layout: Layout, q_tiles, reduce='max',
                 round_scores=True):
    """heatmap.py:36-99: [H', R, n] fp32 heat, 0 on padding rows / empty keys.

    `round_scores` rounds every q.k to bf16 first, which is what the
    reference's bf16 `bmm` returns for bf16 inputs (leave False for fp32
    inputs, whose bmm is not rounded).
    """
    if reduce not in ('max', 'sum'):
        raise ValueError(f"reduce must be 'max' or 'sum': {reduce!r}")
    heads, dim = q.shape[1], q.shape[2]
    scale = np.float32(1.0 / math.sqrt(dim))
    valid = layout.slot_valid.astype(bool)
    q_tiles = np.asarray(q_tiles)
    n = layout.n_tiles
    heat = np.zeros((heads, q_tiles.size, n), dtype=np.float32)
    kf = k.astype(np.float32)
    for h in range(heads):
        for r_i, r in enumerate(q_tiles):
            sl = slice(r * TILE, (r + 1) * TILE)
            s = q[sl, h].astype(np.float32) @ kf[:, h].T      # [128, N]
            if round_scores:
                s = round_bf16(s)
            s = np.where(valid[None, :], s, -np.inf)
            blocks = s.reshape(TILE, n, TILE)
            lr = lse[sl, h].astype(np.float32)[:, None]
            if reduce == 'max':
                agg = blocks.max(-1)                            # [128, n]
                with np.errstate(invalid='ignore'):
                    rows_heat = np.exp(agg * scale - lr)
            else:
                with np.errstate(invalid='ignore'):
                    p = np.exp(blocks * scale - lr[:, :, None])
                rows_heat = p.sum(-1)
            rows_heat = np.where(valid[sl][:, None], rows_heat, 0.0)
            rows_heat = np.nan_to_num(rows_heat, nan=0.0)
            heat[h, r_i] = (rows_heat.max(0) if reduce == 'max'
                            else rows_heat.sum(0))
    return heat


# ---------------------------------------------------------------------------
# (f) zero-order compensation (miowtion/veda/attention.py:591-689; the Triton
# form miowtion/kernels/compensation_triton.py:84-245)
# ---------------------------------------------------------------------------

def zero_order_compensation(o_kept, lse_kept, q_tiles, k_tiles, v_tiles,
                            block_mask, layout: Layout,
                            bf16_summaries=False):
    """attention.py:591-689 (fp32): each dropped key tile with real rows
    becomes one key at its centroid (mean k over real rows) with value
    sum v, weighted by its real row count; the reference exponent is the
    kept LSE (0 where not finite). `bf16_summaries` rounds the centroid and
    the value sum to bf16 as the Triton form stores them. An empty key tile
    carries no mass in either form (zero value sum, zero weight).
    """
    rows, heads, dim = o_kept.shape
    n = layout.n_tiles
    scale = np.float32(1.0 / math.sqrt(dim))
    counts = layout.valid_count.astype(np.float32)
    kf = k_tiles.astype(np.float32).reshape(n, TILE, heads, dim)
    vf = v_tiles.astype(np.float32).reshape(n, TILE, heads, dim)
    real = (np.arange(TILE)[None, :] < layout.valid_count[:, None])
    k_mean = (kf * real[:, :, None, None]).sum(1) / np.maximum(
        counts, 1.0)[:, None, None]                        # [n, H, D]
    v_sum = (vf * real[:, :, None, None]).sum(1)
    if bf16_summaries:
        k_mean, v_sum = round_bf16(k_mean), round_bf16(v_sum)
    out = np.empty((rows, heads, dim), dtype=np.float32)
    owner = np.arange(rows) // TILE
    for h in range(heads):
        ref = lse_kept[h].astype(np.float32)
        safe = np.where(np.isfinite(ref), ref, 0.0).astype(np.float32)
        drop = (~block_mask[h][owner]) & (counts[None, :] > 0)   # [rows, n]
        s_hat = (q_tiles[:, h].astype(np.float32) @ k_mean[:, h].T) * scale
        with np.errstate(over='ignore'):
            p_hat = np.where(drop, np.exp(s_hat - safe[:, None]), 0.0)
        num = p_hat @ v_sum[:, h]
        den = p_hat @ counts
        out[:, h] = (o_kept[:, h].astype(np.float32) + num) / (
            1.0 + den)[:, None]
    return out


# ---------------------------------------------------------------------------
# stage-1 supervision: the seer KL (miowtion/veda/heatmap.py:113-180)
# ---------------------------------------------------------------------------

def seer_kl(logits, heat, kv_ok, direction='forward'):
    """heatmap.py:125-180 in float64: the student is softmax(logits) over
    the key tiles with kv_ok; the teacher is the heat clipped at 0 and
    normalised per row. forward: sum of t * (log t - log s) over t > 0;
    reverse: sum of s * (log s - log max(t, 1e-6)). Rows without heat are
    left out; the mean is over rows per head, then over heads."""
    if direction not in ('forward', 'reverse'):
        raise ValueError(direction)
    logits = np.asarray(logits, np.float64)
    cols = np.asarray(kv_ok, bool)[None, None, :]
    z = np.where(cols, logits, -np.inf)
    zmax = z.max(-1, keepdims=True)
    log_s = z - zmax - np.log(np.exp(z - zmax).sum(-1, keepdims=True))
    t = np.where(cols, np.maximum(np.asarray(heat, np.float64), 0.0), 0.0)
    total = t.sum(-1, keepdims=True)
    live = total[..., 0] > 0
    t = t / np.where(total > 0, total, 1.0)
    with np.errstate(divide='ignore', invalid='ignore'):
        if direction == 'forward':
            pos = cols & (t > 0)
            terms = np.where(pos, t * (np.log(np.where(pos, t, 1.0))
                                       - np.where(pos, log_s, 0.0)), 0.0)
        else:
            log_t = np.log(np.maximum(t, 1e-6))
            terms = np.where(cols, np.exp(log_s) * (log_s - log_t), 0.0)
    rows = terms.sum(-1)
    per_head = (rows * live).sum(-1) / np.maximum(live.sum(-1), 1)
    return float(per_head.mean())


# ---------------------------------------------------------------------------
# (f) tile search: oracle relative error (miowtion/veda/search.py:53-175)
# ---------------------------------------------------------------------------

def _slots(rows) -> np.ndarray:
    rows = np.asarray(rows, dtype=np.int64)
    return (rows[:, None] * TILE + np.arange(TILE)[None]).reshape(-1)


def _rel_err(o_sparse, o_dense, row_valid) -> np.ndarray:
    """search.py:122-126: per head sum of squared errors over sum of
    squares, real rows only (fp32 accumulation)."""
    diff = ((o_sparse - o_dense) ** 2).sum(-1)[row_valid]      # [rows, H]
    norm = (o_dense ** 2).sum(-1)[row_valid]
    tiny = np.finfo(np.float32).tiny
    return (diff.sum(0) / np.maximum(norm.sum(0), tiny)).astype(np.float32)


def oracle_rel_mse_reference(q, k, v, layout: Layout, blocks, rows,
                             round_scores=True) -> np.ndarray:
    """search.py:130-175: token-level fp32 restatement, head by head.

    q, k, v [S, H, D] (bf16 values); `rows` the sampled video query tiles.
    The dense probabilities of the sampled rows give the block score (the
    max of p inside each block), the selection keeps blocks by the training
    rules with every global key tile kept, and the sparse output is p
    renormalised on the kept blocks. `round_scores` rounds q.k to bf16 as
    the reference's bf16 matmul does.
    """
    heads, dim = q.shape[1], q.shape[2]
    scale = np.float32(1.0 / math.sqrt(dim))
    valid = layout.slot_valid.astype(bool)
    slots = _slots(rows)
    row_valid = valid[slots]
    n = layout.n_tiles
    rows = np.asarray(rows, dtype=np.int64)
    gi = layout.gather_index
    out = np.zeros(heads, dtype=np.float32)
    for h in range(heads):
        qt = q[gi[slots], h].astype(np.float32)
        kt = k[gi, h].astype(np.float32)
        vt = v[gi, h].astype(np.float32)
        s = qt @ kt.T
        if round_scores:
            s = round_bf16(s)
        s = np.where(valid[None, :], s * scale, -np.inf)
        m = s.max(-1, keepdims=True)
        p = np.exp(s - m)
        p /= p.sum(-1, keepdims=True)
        p[~row_valid] = 0.0
        o_dense = p @ vt
        block = p.reshape(rows.size, TILE, n, TILE).max(axis=(1, 3))
        index, keep = select_video_blocks(block[None], layout, blocks, rows)
        kept = np.zeros((rows.size, n), dtype=bool)
        np.put_along_axis(kept, index[0], keep[0], axis=1)
        kept[:, layout.n_video_tiles:] = True
        ps = (p.reshape(rows.size, TILE, n, TILE)
              * kept[:, None, :, None]).reshape(p.shape)
        ps /= np.maximum(ps.sum(-1, keepdims=True), np.finfo(np.float32).tiny)
        o_sparse = ps @ vt
        out[h] = _rel_err(o_sparse[:, None], o_dense[:, None],
                          row_valid)[0]
    return out


def oracle_rel_mse(q, k, v, layout: Layout, blocks, rows, dense_out,
                   lse) -> np.ndarray:
    """search.py:86-127, the kernel path: block scores from the teacher heat
    (reduce 'max') with the dense LSE, selection without global query rows,
    the block-sparse forward of the sampled query tiles alone (bf16 output),
    and the error against the bf16 dense output of those rows."""
    heads = np.arange(q.shape[1])
    qt = gather_tiles(q, layout, heads)
    kt = gather_tiles(k, layout, heads)
    vt = gather_tiles(v, layout, heads)
    lse_t = gather_lse(lse, layout, heads)
    rows = np.asarray(rows, dtype=np.int64)
    heat = teacher_heat(qt, kt, lse_t, layout, rows, 'max')
    index, keep = select_video_blocks(heat, layout, blocks, rows)
    mask = dense_block_mask(index, keep, layout, global_rows=False)
    slots = _slots(rows)
    o_sparse = round_bf16(block_sparse_attention(
        qt[slots], kt, vt, mask, layout.valid_count))
    o_dense = round_bf16(np.asarray(dense_out, np.float32))[
        layout.gather_index[slots]]
    return _rel_err(o_sparse, o_dense, layout.slot_valid.astype(bool)[slots])


# ---------------------------------------------------------------------------
# The whole SparseStudent layer (miowtion/veda/attention.py:724-794)
# ---------------------------------------------------------------------------

def sparse_student_layer(q, k, v, groups, proj_q, proj_k, target_budget,
                         ref_budget=None, *, used=None):
    """One sparse layer: gather/pool -> logits -> top-k -> attention -> scatter.

    `groups` is a list of (Layout, heads) pairs (plan.head_groups). Returns
    (out [S,H,D] float32, per-group dicts of intermediates).
    """
    seq_len, n_heads, dim = q.shape
    used = seq_len if used is None else used
    out = np.zeros((seq_len + 1, n_heads, dim), dtype=np.float32)
    info = []
    for layout, heads in groups:
        heads = np.asarray(heads)
        qt = gather_tiles(q, layout, heads)
        kt = gather_tiles(k, layout, heads)
        vt = gather_tiles(v, layout, heads)
        fq = pool_tiles(qt, layout)
        fk = pool_tiles(kt, layout)
        logits = predictor_logits(fq, fk, proj_q, proj_k, heads)
        blocks = column_blocks(layout, target_budget, ref_budget)
        index, keep = select_video_blocks(
            logits[:, :layout.n_video_tiles], layout, blocks)
        mask = dense_block_mask(index, keep, layout)
        ot = block_sparse_attention(qt, kt, vt, mask, layout.valid_count)
        scatter_tiles(out, ot.astype(np.float32), layout, heads)
        info.append(dict(feats_q=fq, feats_k=fk, logits=logits, index=index,
                         keep=keep, mask=mask))
    out = out[:seq_len]
    out[used:] = 0
    return out, info
