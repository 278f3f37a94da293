"""Teacher block heat: drop-in for the reference's `miowtion/veda/heatmap.py`
heat entry points (`teacher_heat`, `teacher_heat_reference`), backed by the
tcgen05 kernel `veda_teacher_heat`, plus the two pieces of the stage-1
supervision the teacher collector runs by default: the seer KL and the
mask diagnostics. Both are small fp32 torch on the [H', R, n] tile grid
(about 1e-6 of the heat's cost); the reference's other losses
(transport_loss, gauge_fixed_kl, oracle_bce) are ablation objectives and
are not provided.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from miowtion_b200 import _lib
from miowtion_b200 import kernels
from miowtion_b200 import mask as veda_mask
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


# The reverse KL floors the teacher's block probability here, so a block the
# teacher gives no mass costs a finite penalty (heatmap.py:113-116).
REVERSE_FLOOR = 1e-6


def seer_kl(logits: torch.Tensor, heat: torch.Tensor,
            layout: tiling.TileLayout,
            direction: str = 'forward') -> torch.Tensor:
    """The seer KL over key tiles, averaged over rows then heads
    (heatmap.py:125-180).

    The student distribution is softmax(logits) over the non-empty key
    tiles; the teacher's is the heat, clipped at 0 and normalised per row.
    'forward' is KL(teacher || student) over the blocks the teacher gives
    mass; 'reverse' is KL(student || teacher) with the teacher floored at
    REVERSE_FLOOR. Rows whose heat sums to 0 do not count.

    Args:
        logits: [H', R, n_tiles] fp32 student logits (with grad).
        heat: [H', R, n_tiles] fp32 teacher heat.
        layout: Tile layout (its empty key tiles are excluded).
        direction: 'forward' or 'reverse'.

    Returns:
        Scalar loss.

    Raises:
        ValueError: On an unknown direction.
    """
    if direction not in ('forward', 'reverse'):
        raise ValueError(f"direction must be 'forward' or 'reverse': "
                         f'{direction!r}')
    cols = layout.kv_ok.view(1, 1, -1)
    log_student = F.log_softmax(
        logits.masked_fill(~cols, float('-inf')), dim=-1)
    teacher = torch.where(cols, heat.clamp(min=0.0), 0.0)
    row_mass = teacher.sum(-1, keepdim=True)
    live = row_mass.squeeze(-1) > 0
    teacher = teacher / row_mass.clamp(min=torch.finfo(torch.float32).tiny)
    if direction == 'forward':
        support = cols & (teacher > 0)
        safe_t = torch.where(support, teacher, 1.0)
        safe_s = torch.where(support, log_student, 0.0)
        terms = torch.where(support, teacher * (safe_t.log() - safe_s), 0.0)
    else:
        log_teacher = teacher.clamp(min=REVERSE_FLOOR).log()
        terms = torch.where(cols, log_student.exp()
                            * (log_student - log_teacher), 0.0)
    row_kl = terms.sum(-1)
    head_kl = (row_kl * live).sum(-1) / live.sum(-1).clamp(min=1)
    return head_kl.mean()


@torch.no_grad()
def mask_diagnostics(logits: torch.Tensor, heat: torch.Tensor,
                     layout: tiling.TileLayout,
                     blocks: list[veda_mask.ColumnBlock],
                     q_tiles: torch.Tensor) -> dict[str, torch.Tensor]:
    """Predictor against oracle on the video quadrant, as device scalars
    (heatmap.py:499-574): `recall` (off-diagonal overlap of the predicted
    and the heat's own top-k sets; NaN when the budget holds nothing but the
    diagonal), `heat_kept` / `heat_ceiling` (share of a row's video heat the
    predicted / the oracle's tiles carry, diagonal included, averaged over
    rows with heat), `retained` (per row, the predicted off-diagonal heat
    over the oracle's, averaged over rows with some). Nothing synchronises
    the host.

    Args:
        logits: [H', R, n_tiles] student logits of the rows `q_tiles`.
        heat: [H', R, n_tiles] teacher heat of the same rows.
        layout: Tile layout.
        blocks: Column blocks with their budgets.
        q_tiles: [R] int64 video query tiles.
    """
    n_video = layout.n_video_tiles
    q_tiles = q_tiles.to(device=logits.device, dtype=torch.int64)

    def chosen(scores: torch.Tensor) -> torch.Tensor:
        sel = veda_mask.select_video_blocks(scores.contiguous(), layout,
                                            blocks, q_tiles)
        out = torch.zeros(*sel.index.shape[:2], n_video, dtype=torch.bool,
                          device=logits.device)
        return out.scatter_(2, sel.index, sel.keep)

    predicted, oracle = chosen(logits.float()), chosen(heat.float())
    mass = heat[:, :, :n_video].float().clamp(min=0.0)
    total = mass.sum(-1)
    tiny = torch.finfo(torch.float32).tiny
    has_mass = total > 0

    def kept_share(selected: torch.Tensor) -> torch.Tensor:
        per_row = (mass * selected).sum(-1) / total.clamp(min=tiny)
        return (per_row * has_mass).sum() / has_mass.sum().clamp(min=1)

    diagonal = F.one_hot(q_tiles, n_video).bool()[None]
    pred_off = predicted & ~diagonal
    oracle_off = oracle & ~diagonal
    hits = (pred_off & oracle_off).sum()
    possible = oracle_off.sum()
    recall = torch.where(possible > 0, hits / possible.clamp(min=1),
                         torch.nan)
    off_mass = mass.masked_fill(diagonal, 0.0)
    ceiling = (off_mass * oracle_off).sum(-1)
    rows = ceiling > 0
    ratio = (off_mass * pred_off).sum(-1) / ceiling.clamp(min=tiny)
    retained = (ratio * rows).sum() / rows.sum().clamp(min=1)
    return {'recall': recall, 'heat_kept': kept_share(predicted),
            'heat_ceiling': kept_share(oracle), 'retained': retained}
