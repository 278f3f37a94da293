"""Tile-plan search on the B200 kernels: the oracle relative error of each
candidate tile shape per (layer, head), and the plan vote over those scores.

Mirror of the reference's `miowtion/veda/search.py` (names, arguments and
errors). For every scored layer, candidate shape and head
(search.py:1-22):

1. permute q, k, v with the candidate's tile layout (`gather_and_pool`);
2. sample video query tiles with one seed for every candidate;
3. block score = the peak probability of each (query tile, key tile) block,
   from the dense teacher's LSE (`teacher_heat`, reduce 'max');
4. keep blocks by the training rules (budget, Bresenham, diagonal, column
   blocks; global key tiles always kept), without global query rows, as
   the block lists of the sampled rows (`select_block_lists`);
5. the sparse output of the sampled query tiles alone (the row-subset
   forward of `block_sparse_attention`);
6. rel_mse = sum ||o_sparse - o_dense||^2 / sum ||o_dense||^2 over their real
   rows (`veda_rel_mse`).

Every step runs on the device; the fp32 token-level restatement of the same
quantity (search.py:130-175) lives in the CPU oracle, for the tests only.
"""

from __future__ import annotations

import dataclasses
import json
import os
from collections.abc import Iterable, Sequence

import torch

from miowtion_b200 import _lib
from miowtion_b200 import attention as veda_attention
from miowtion_b200 import heatmap
from miowtion_b200 import kernels
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import tiling

_TILE = tiling.TILE_SIZE

# Bound on the tile-ordered q / k / v copies held at once (search.py:80-83);
# heads are scored in chunks under it. Heads are independent throughout, so
# chunking does not change the result.
_ORACLE_GATHER_BYTES = 1 << 30


def rel_mse(o_sparse: torch.Tensor, o_dense: torch.Tensor,
            seq_row: torch.Tensor, heads: torch.Tensor) -> torch.Tensor:
    """[H'] relative MSE of o_sparse [R * 128, H', 128] (sampled slots)
    against rows seq_row of o_dense [S, H, 128], heads `heads`; slots with
    seq_row < 0 are padding and not scored (search.py:117-126)."""
    if o_sparse.dtype != torch.bfloat16 or o_dense.dtype != torch.bfloat16:
        raise ValueError('rel_mse takes bf16 outputs')
    if o_sparse.shape[-1] != 128 or o_dense.shape[-1] != 128:
        raise ValueError('rel_mse takes head_dim 128')
    if o_sparse.stride(-1) != 1 or o_dense.stride(-1) != 1:
        raise ValueError('outputs must be contiguous in head_dim')
    n_rows = o_sparse.shape[0] // _TILE
    n_heads = o_sparse.shape[1]
    if seq_row.numel() != n_rows * _TILE or heads.numel() != n_heads:
        raise ValueError('seq_row must cover every sampled slot and heads '
                         'every head of o_sparse')
    dev = o_sparse.device
    seq_row = seq_row.to(device=dev, dtype=torch.int64).contiguous()
    heads = heads.to(device=dev, dtype=torch.int64).contiguous()
    ws_bytes = _lib.load().veda_rel_mse_workspace(n_rows, n_heads)
    ws = torch.empty(max(1, ws_bytes // 4), dtype=torch.float32, device=dev)
    out = torch.empty(n_heads, dtype=torch.float32, device=dev)
    _lib.call('veda_rel_mse', o_sparse.data_ptr(), o_sparse.stride(0),
              o_sparse.stride(1), o_dense.data_ptr(), o_dense.stride(0),
              o_dense.stride(1), seq_row.data_ptr(), heads.data_ptr(), n_rows,
              n_heads, out.data_ptr(), ws.data_ptr(), ws.numel() * 4,
              _lib.stream_ptr(dev))
    return out


def oracle_rel_mse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   tile_layout: tiling.TileLayout,
                   blocks: list[veda_mask.ColumnBlock], rows: torch.Tensor,
                   dense_out: torch.Tensor | None = None,
                   lse: torch.Tensor | None = None) -> torch.Tensor:
    """Oracle relative MSE per head of one head group (search.py:53-77).

    Args:
        q, k, v: [S, H', D] bf16 packed rows of the heads to score.
        tile_layout: Candidate permutation.
        blocks: Column blocks (budgets).
        rows: [R] int64 sampled video query tiles.
        dense_out: [S, H', D] dense output of these heads; computed here
            (with `lse`) when either is missing.
        lse: [S, H'] fp32 natural-log dense LSE.

    Returns:
        [H'] fp32 relative MSE per head.

    Raises:
        NotImplementedError: Off B200 (there is no CPU path).
    """
    if dense_out is None or lse is None:
        dense_out, lse = kernels.dense_attention(
            q, k, v, q.shape[-1]**-0.5, return_lse=True,
            used=tile_layout.used)
    return _oracle_rel_mse_kernels(q, k, v, dense_out, lse, tile_layout,
                                   blocks, rows)


@torch.no_grad()
def _oracle_rel_mse_kernels(q, k, v, dense_out, lse, tile_layout, blocks,
                            rows):
    """Head chunks; never materialises [rows, N] probabilities
    (search.py:86-127)."""
    kernels._require(q, 'oracle_rel_mse')  # pylint: disable=protected-access
    num_heads = q.shape[1]
    per_head = 3 * tile_layout.num_slots * q.shape[-1] * q.element_size()
    chunk = max(1, min(num_heads, _ORACLE_GATHER_BYTES // per_head))
    rows = rows.to(device=q.device, dtype=torch.int64).contiguous()
    if rows.numel() and (int(rows.min()) < 0 or
                         int(rows.max()) >= tile_layout.n_video_tiles):
        raise ValueError('rows must be video query tiles')
    seq_row, _ = tiling.tile_rows_perm(tile_layout, rows)
    errors = []
    for start in range(0, num_heads, chunk):
        heads = torch.arange(start, min(start + chunk, num_heads),
                             device=q.device)
        k_t, v_t = (tiling.gather_tiles(t, tile_layout, heads) for t in (k, v))
        q_t = tiling.gather_tiles(q, tile_layout, heads)
        lse_t = tiling.gather_lse(lse, tile_layout, heads)
        heat = heatmap.teacher_heat(q_t, k_t, lse_t, tile_layout, rows)
        del q_t
        # The selection's block lists of the sampled rows, without global
        # query rows (dense_block_mask(global_rows=False) then index_lists,
        # in one kernel).
        lists = veda_mask.select_block_lists(heat, tile_layout, blocks, rows,
                                             global_rows=False)
        # The sampled query tiles alone, straight from the packed rows.
        q_s = tiling.gather_tile_rows(q, tile_layout, rows, heads)
        o_sparse = kernels.block_sparse_attention_lists(q_s, k_t, v_t, lists,
                                                        tile_layout)
        errors.append(rel_mse(o_sparse, dense_out, seq_row, heads))
    return torch.cat(errors)


class OracleScorer:
    """AttentionFn that returns the dense attention and, on the way, scores
    every candidate shape (search.py:195-243). Only the layers of scored
    steps should use it; the trajectory itself stays dense.

    `dense_backend` is accepted for the reference's signature; the dense
    teacher here is always this library's dense kernel. Scores accumulate
    in `scores[layer] = [candidates, heads]` fp32 on the host.
    """

    def __init__(self, layout: veda_attention.PackedLayout,
                 candidates: Sequence[tiling.TileShape],
                 config: veda_attention.VedaConfig, query_tiles: int,
                 seed: int, device: torch.device,
                 dense_backend: str = 'auto'):
        del dense_backend
        self.clip = veda_attention.ClipTiling(layout, config, device)
        self.layout, self.candidates = layout, list(candidates)
        self.query_tiles, self.seed = query_tiles, seed
        self.scores: dict[int, torch.Tensor] = {}

    def sample_rows(self, tile_layout: tiling.TileLayout,
                    layer_index: int) -> torch.Tensor:
        """The sampled video query tiles, ascending. The seed depends on
        the run seed and the layer only (seed * 1000 + layer), so every
        candidate of a layer is scored on the same draw: the first
        min(query_tiles, n_video) entries of a random permutation."""
        draw = torch.randperm(
            tile_layout.n_video_tiles,
            generator=torch.Generator().manual_seed(
                self.seed * 1000 + layer_index))
        return draw[:self.query_tiles].sort().values

    def __call__(self, q, k, v, layer_index):
        out, lse = kernels.dense_attention(q, k, v, q.shape[-1]**-0.5,
                                           return_lse=True,
                                           used=self.layout.used)
        per_candidate = []
        for shape in self.candidates:
            tile_layout = self.clip.get(shape)
            rows = self.sample_rows(tile_layout, layer_index).to(q.device)
            per_candidate.append(oracle_rel_mse(
                q, k, v, tile_layout, self.clip.blocks(tile_layout), rows,
                dense_out=out, lse=lse).float().cpu())
        self.scores[layer_index] = torch.stack(per_candidate)
        return out


@dataclasses.dataclass(frozen=True)
class ScoreEntry:
    """rel-MSE of every candidate shape for one (clip, step, layer):
    `table` [candidates, heads]."""

    clip: str
    step: int
    layer: int
    table: torch.Tensor


# Score files: one JSON object {"candidates": [shape strings], "meta": {...},
# "entries": [{"clip", "step", "layer", "table"}, ...]} (the reference's
# search.py:256-294), and beside it "<file>.done" = {"entries": count},
# written last: a file without it is an interrupted run.
_DONE = '.done'


def save_entries(path: str, entries: Iterable[ScoreEntry],
                 candidates: Sequence[tiling.TileShape], meta: dict) -> None:
    """Writes a score file (atomically), then its completion marker."""
    rows = [dict(clip=e.clip, step=e.step, layer=e.layer,
                 table=e.table.tolist()) for e in entries]
    body = dict(candidates=[str(c) for c in candidates], meta=meta,
                entries=rows)
    partial = path + '.tmp'
    with open(partial, 'w') as f:
        json.dump(body, f)
    os.replace(partial, path)
    with open(path + _DONE, 'w') as f:
        json.dump({'entries': len(rows)}, f)


def _read_score_file(path: str) -> dict:
    if not os.path.exists(path + _DONE):
        raise FileNotFoundError(
            f'{path} has no completion marker ({path + _DONE}): the run '
            'that wrote it did not finish')
    with open(path) as f:
        return json.load(f)


def load_entries(paths: Iterable[str]
                 ) -> tuple[list[tiling.TileShape], list[ScoreEntry], dict]:
    """The entries of completed score files, in file order; the menu and
    the meta come from the files (the meta of the last one).

    Raises:
        FileNotFoundError: A file without its completion marker.
        ValueError: Files scored against different candidate menus.
    """
    menu: list[tiling.TileShape] | None = None
    meta: dict = {}
    entries: list[ScoreEntry] = []
    for path in paths:
        body = _read_score_file(path)
        this_menu = [tiling.TileShape.parse(c) for c in body['candidates']]
        if menu is None:
            menu = this_menu
        elif this_menu != menu:
            raise ValueError(f'{path}: candidate menu {body["candidates"]} '
                             f'differs from the earlier files\'')
        meta = body['meta']
        entries.extend(ScoreEntry(r['clip'], r['step'], r['layer'],
                                  torch.tensor(r['table']))
                       for r in body['entries'])
    return menu, entries, meta


def _vote_layer(tables: torch.Tensor, max_shapes: int
                ) -> tuple[list[int], list[int], torch.Tensor]:
    """One layer's vote over `tables` [entries, shapes, heads] (allowed
    shapes only). Returns (kept shapes in rank order, each head's shape,
    each head's mean error under it).

    1. Every entry votes, per head, for its lowest-error shape; each head
       takes the most-voted shape (the lower mean error on a tie).
    2. Shapes rank by how many heads took them (the lower mean error over
       heads on a tie); the first `max_shapes` that some head took stay.
    3. Every head takes the staying shape with its lowest mean error.
    """
    n_shapes = tables.shape[1]
    mean = tables.mean(0)                                 # [shapes, heads]
    ballots = torch.nn.functional.one_hot(
        tables.argmin(1), n_shapes).sum(0).T.to(mean.dtype)  # [shapes, heads]
    # Integer vote counts first, mean error only to break a tie.
    head_pick = (ballots - 1e-6 * mean).argmax(0)
    heads_per_shape = torch.bincount(head_pick, minlength=n_shapes)
    order = sorted(range(n_shapes),
                   key=lambda a: (-int(heads_per_shape[a]),
                                  float(mean[a].mean())))
    kept = [a for a in order if heads_per_shape[a] > 0][:max_shapes]
    among = mean[kept]                                    # [kept, heads]
    choice = among.argmin(0)
    return kept, [kept[c] for c in choice.tolist()], \
        among.gather(0, choice[None])[0]


def build_plan(geometry_name: str, grid: tuple[int, int, int],
               candidates: Sequence[tiling.TileShape],
               entries: Sequence[ScoreEntry], num_layers: int,
               max_padding: float = 0.2, max_shapes_per_layer: int = 2,
               meta: dict | None = None) -> veda_plan.TilePlan:
    """A timestep-independent plan voted from oracle scores
    (search.py:297-368): candidates that pad the grid by more than
    `max_padding` are out; each layer votes as `_vote_layer` describes. The
    provenance records the entries used, the voting limits, the plan's mean
    error and the best single shape's.

    Raises:
        ValueError: No candidate within the padding limit, or a layer
            without scores.
    """
    allowed = [i for i, c in enumerate(candidates)
               if c.padding_ratio(grid) <= max_padding + 1e-12]
    if not allowed:
        raise ValueError('no candidate passes the padding limit')
    per_layer: dict[int, list[torch.Tensor]] = {}
    for e in entries:
        per_layer.setdefault(e.layer, []).append(e.table[allowed])
    absent = [layer for layer in range(num_layers) if layer not in per_layer]
    if absent:
        raise ValueError(f'no scores for layers {absent[:5]}')

    rows, errors, layer_shapes, means = [], [], [], []
    for layer in range(num_layers):
        tables = torch.stack(per_layer[layer])
        kept, picks, err = _vote_layer(tables, max_shapes_per_layer)
        rows.append([allowed[a] for a in picks])
        errors.append(err)
        layer_shapes.append([str(candidates[allowed[a]]) for a in kept])
        means.append(tables.mean(0))
    in_use = sorted({c for row in rows for c in row})
    slot = {c: i for i, c in enumerate(in_use)}
    by_shape = torch.stack(means).mean(dim=(0, 2))        # [allowed]
    provenance = {
        'entries': len(entries),
        'clips': sorted({e.clip for e in entries}),
        'steps': sorted({e.step for e in entries}),
        'max_padding': max_padding,
        'max_shapes_per_layer': max_shapes_per_layer,
        'plan_mse': torch.stack(errors).mean().item(),
        'best_single_shape_mse': by_shape.min().item(),
        'layer_shapes': layer_shapes,
    }
    provenance.update(meta or {})
    return veda_plan.TilePlan(geometry_name, tuple(grid),
                              [candidates[c] for c in in_use],
                              [[slot[c] for c in row] for row in rows],
                              provenance)
