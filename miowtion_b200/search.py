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

import collections
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
    """AttentionFn that returns dense attention and scores every candidate
    shape on the way (search.py:195-243). Only the layers of scored steps
    should use it; the trajectory itself stays dense. `dense_backend` is
    kept for the reference's signature: the dense teacher here is always
    this library's dense kernel."""

    def __init__(self, layout: veda_attention.PackedLayout,
                 candidates: Sequence[tiling.TileShape],
                 config: veda_attention.VedaConfig, query_tiles: int,
                 seed: int, device: torch.device,
                 dense_backend: str = 'auto'):
        self.layout = layout
        self.candidates = list(candidates)
        self.clip = veda_attention.ClipTiling(layout, config, device)
        self.query_tiles = query_tiles
        self.seed = seed
        self.dense_backend = dense_backend
        self.scores: dict[int, torch.Tensor] = {}

    def sample_rows(self, tile_layout: tiling.TileLayout,
                    layer_index: int) -> torch.Tensor:
        """Sorted sample of video query tiles, one seed per (run, layer) so
        every candidate is scored on paired samples (search.py:227-230)."""
        gen = torch.Generator().manual_seed(self.seed * 1000 + layer_index)
        count = min(self.query_tiles, tile_layout.n_video_tiles)
        rows = torch.randperm(tile_layout.n_video_tiles, generator=gen)
        return rows[:count].sort().values

    def __call__(self, q, k, v, layer_index):
        out, lse = kernels.dense_attention(q, k, v, q.shape[-1]**-0.5,
                                           return_lse=True,
                                           used=self.layout.used)
        table = torch.empty(len(self.candidates), q.shape[1],
                            dtype=torch.float32)
        for ci, shape in enumerate(self.candidates):
            tile_layout = self.clip.get(shape)
            rows = self.sample_rows(tile_layout, layer_index).to(q.device)
            table[ci] = oracle_rel_mse(q, k, v, tile_layout,
                                       self.clip.blocks(tile_layout), rows,
                                       dense_out=out, lse=lse).cpu()
        self.scores[layer_index] = table
        return out


@dataclasses.dataclass(frozen=True)
class ScoreEntry:
    """rel-MSE of every candidate for one (clip, step, layer): [C, H]."""

    clip: str
    step: int
    layer: int
    table: torch.Tensor


def save_entries(path: str, entries: Iterable[ScoreEntry],
                 candidates: Sequence[tiling.TileShape], meta: dict) -> None:
    """Writes the score file atomically, then its `.done` marker
    (search.py:256-273)."""
    entries = list(entries)
    payload = {'candidates': [str(c) for c in candidates], 'meta': meta,
               'entries': [{'clip': e.clip, 'step': e.step, 'layer': e.layer,
                            'table': e.table.tolist()} for e in entries]}
    tmp = path + '.tmp'
    with open(tmp, 'w') as f:
        json.dump(payload, f)
    os.replace(tmp, path)
    with open(path + '.done', 'w') as f:
        json.dump({'entries': len(entries)}, f)


def load_entries(paths: Iterable[str]
                 ) -> tuple[list[tiling.TileShape], list[ScoreEntry], dict]:
    """Completed score files (search.py:276-294).

    Raises:
        FileNotFoundError: A file without its completion marker.
        ValueError: Files with different candidate menus.
    """
    candidates, entries, meta = None, [], {}
    for path in paths:
        if not os.path.exists(path + '.done'):
            raise FileNotFoundError(f'{path} has no completion marker')
        with open(path) as f:
            payload = json.load(f)
        shapes = [tiling.TileShape.parse(s) for s in payload['candidates']]
        if candidates is not None and shapes != candidates:
            raise ValueError(f'{path}: candidate menu differs')
        candidates = shapes
        meta = payload['meta']
        entries += [ScoreEntry(e['clip'], e['step'], e['layer'],
                               torch.tensor(e['table']))
                    for e in payload['entries']]
    return candidates, entries, meta


def build_plan(geometry_name: str, grid: tuple[int, int, int],
               candidates: Sequence[tiling.TileShape],
               entries: Sequence[ScoreEntry], num_layers: int,
               max_padding: float = 0.2, max_shapes_per_layer: int = 2,
               meta: dict | None = None) -> veda_plan.TilePlan:
    """Votes a timestep-independent plan from oracle scores
    (search.py:297-368):

    - candidates padding the grid by more than `max_padding` are dropped;
    - per (layer, head), every entry votes for its lowest-error shape; the
      head picks the majority (ties to the lower mean error);
    - a layer keeps its `max_shapes_per_layer` most-picked shapes (ties to
      the lower mean error); heads of dropped shapes take the kept shape
      with their lowest mean error;
    - provenance records the plan's and the best single shape's mean error.

    Raises:
        ValueError: No candidate passes the padding limit, or a layer has
            no scores.
    """
    allowed = [i for i, c in enumerate(candidates)
               if c.padding_ratio(grid) <= max_padding + 1e-12]
    if not allowed:
        raise ValueError('no candidate passes the padding limit')
    allowed_t = torch.tensor(allowed)
    by_layer = collections.defaultdict(list)
    for e in entries:
        by_layer[e.layer].append(e.table[allowed_t])
    missing = [layer for layer in range(num_layers) if layer not in by_layer]
    if missing:
        raise ValueError(f'no scores for layers {missing[:5]}')
    head_shape, plan_mse, per_layer = [], [], []
    for layer in range(num_layers):
        tables = torch.stack(by_layer[layer])  # [E, A, H]
        mean = tables.mean(0)
        winners = tables.argmin(1)  # [E, H]
        votes = torch.zeros_like(mean).scatter_add_(
            0, winners, torch.ones_like(winners, dtype=mean.dtype))
        head_pick = (votes - 1e-6 * mean).argmax(0)
        counts = torch.bincount(head_pick, minlength=mean.shape[0]).float()
        ranking = sorted(range(mean.shape[0]),
                         key=lambda a: (-counts[a].item(),
                                        mean[a].mean().item()))
        kept = [a for a in ranking if counts[a] > 0][:max_shapes_per_layer]
        kept_t = torch.tensor(kept)
        final = kept_t[mean[kept_t].argmin(0)]
        head_shape.append([allowed[a] for a in final.tolist()])
        plan_mse.append(mean.gather(0, final[None])[0])
        per_layer.append([str(candidates[allowed[a]]) for a in kept])
    used = sorted({i for row in head_shape for i in row})
    remap = {old: new for new, old in enumerate(used)}
    layer_means = torch.stack([torch.stack(by_layer[layer]).mean(0)
                               for layer in range(num_layers)])
    provenance = {
        'entries': len(entries),
        'clips': sorted({e.clip for e in entries}),
        'steps': sorted({e.step for e in entries}),
        'max_padding': max_padding,
        'max_shapes_per_layer': max_shapes_per_layer,
        'plan_mse': torch.stack(plan_mse).mean().item(),
        'best_single_shape_mse': layer_means.mean(dim=(0, 2)).min().item(),
        'layer_shapes': per_layer,
        **(meta or {}),
    }
    return veda_plan.TilePlan(
        geometry=geometry_name, grid=tuple(grid),
        shapes=[candidates[i] for i in used],
        head_shape=[[remap[i] for i in row] for row in head_shape],
        provenance=provenance)
