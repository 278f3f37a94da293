"""Teacher block heat: drop-in for the reference's `miowtion/veda/heatmap.py`
heat entry points (`teacher_heat`, `teacher_heat_reference`), backed by the
tcgen05 kernel `veda_teacher_heat`, plus the stage-1 supervision the
teacher collector trains the predictor with: the seer KL, the three
ablation objectives (`transport_loss`, `gauge_fixed_kl`, `oracle_bce`) and
the mask diagnostics. All of them are small fp32 torch on the [H', R, n]
tile grid (about 1e-6 of the heat's cost). The heat's own top-k, which
three of them compare against, is one launch of the selection kernel
(`oracle_set`); a caller that needs it more than once per head group
computes it once and passes it as `oracle=`.
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
    return _mean_rows_then_heads(row_kl, live)


def _mean_rows_then_heads(per_row: torch.Tensor,
                          live: torch.Tensor) -> torch.Tensor:
    """Mean over the live rows of each head, then over heads; a head
    without live rows counts as 0."""
    per_row = torch.where(live, per_row, 0.0)
    return (per_row.sum(-1) / live.sum(-1).clamp(min=1)).mean()


def _decision_columns(layout: tiling.TileLayout,
                      q_tiles: torch.Tensor) -> torch.Tensor:
    """[1, R, n_video] bool: the video key tiles a predictor decides on for
    each supervised row, i.e. the non-empty ones minus the row's own tile
    (the forced diagonal is a kernel rule, heatmap.py:283-289)."""
    n_video = layout.n_video_tiles
    own = F.one_hot(q_tiles, n_video).bool()[None]
    return layout.kv_ok[:n_video].view(1, 1, -1) & ~own


def _standardise(scores: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Per-row zero mean, unit variance over the columns where `weight` is
    1 (0 elsewhere): the projection that removes the per-row offset and
    scale a top-k read-out cannot see (heatmap.py:309-317)."""
    count = weight.sum(-1, keepdim=True).clamp(min=1.0)
    centred = (scores - (scores * weight).sum(-1, keepdim=True) / count) * weight
    var = (centred.square() * weight).sum(-1, keepdim=True) / count
    return centred / var.clamp(min=1e-12).sqrt()


def _video_mass(heat: torch.Tensor, columns: torch.Tensor) -> torch.Tensor:
    """The teacher's non-negative block heat on the decision columns."""
    mass = heat[:, :, :columns.shape[-1]].float()
    return torch.where(columns, mass, 0.0).clamp(min=0.0)


@torch.no_grad()
def oracle_set(heat: torch.Tensor, layout: tiling.TileLayout,
               blocks: list[veda_mask.ColumnBlock],
               q_tiles: torch.Tensor) -> torch.Tensor:
    """The heat's own top-k selection over the video key tiles at the
    clip's budgets, as a [H', R, n_video] bool mask: the oracle set that
    `transport_loss`, `oracle_bce` and `mask_diagnostics` compare against
    (heatmap.py:285-291, :462-466). One launch of the selection kernel."""
    n_video = layout.n_video_tiles
    q_tiles = q_tiles.to(device=heat.device, dtype=torch.int64)
    sel = veda_mask.select_video_blocks(heat.float().contiguous(), layout,
                                        blocks, q_tiles)
    chosen = torch.zeros(*sel.index.shape[:2], n_video, dtype=torch.bool,
                         device=heat.device)
    return chosen.scatter_(2, sel.index, sel.keep)


# Width of the soft top-k boundary in row-standardised score units
# (heatmap.py:183-190).
TRANSPORT_TAU = 0.15

# Masked columns sort below every standardised score at this value
# (heatmap.py:118-121). Where a row's budget reaches its last valid column
# the cut falls halfway down to it, and the sigmoid is then 1 at every
# valid column for any value this large.
_BELOW_EVERY_SCORE = 1e4


def transport_loss(logits: torch.Tensor, heat: torch.Tensor,
                   layout: tiling.TileLayout,
                   blocks: list[veda_mask.ColumnBlock],
                   q_tiles: torch.Tensor,
                   temperature: float = TRANSPORT_TAU,
                   oracle: torch.Tensor | None = None) -> torch.Tensor:
    """Minus the retained transport mass relative to the oracle's
    (heatmap.py:192-333).

    Per row: the student's scores over the decision columns are
    standardised, the row's cut is placed halfway between its k-th and
    (k+1)-th largest standardised score (k = the oracle's off-diagonal
    budget of the row; the cut carries no gradient), and the soft policy
    sigmoid((z - cut) / temperature) is rescaled to spend exactly k. The
    row's value is the policy's share of the teacher mass the oracle keeps;
    rows where the oracle keeps nothing or no mass do not count. -1 is the
    oracle's own choice; as temperature -> 0 the loss is minus the
    `retained` diagnostic of the student's hard top-k. Invariant to a
    per-row positive affine map of the logits.

    Args:
        logits: [H', R, n_tiles] fp32 student logits (with grad).
        heat: [H', R, n_tiles] teacher heat (the mass reduction).
        layout: Tile layout.
        blocks: Column blocks with their budgets.
        q_tiles: [R] int64 supervised video query tiles.
        temperature: Width of the soft boundary; > 0.
        oracle: The heat's own selection, `oracle_set(heat, ...)`, if the
            caller has it already.

    Returns:
        Scalar loss (rows averaged, then heads).

    Raises:
        ValueError: If temperature is not positive.
    """
    if temperature <= 0:
        raise ValueError(f'temperature must be > 0: {temperature}')
    n_video = layout.n_video_tiles
    q_tiles = q_tiles.to(device=logits.device, dtype=torch.int64)
    with torch.no_grad():
        if oracle is None:
            oracle = oracle_set(heat, layout, blocks, q_tiles)
        columns = _decision_columns(layout, q_tiles)
        kept = oracle & columns
        mass = _video_mass(heat, columns)
        ceiling = (mass * kept).sum(-1)
        budget = kept.sum(-1)
        live = (ceiling > 0) & (budget > 0)
    weight = columns.float()
    z = _standardise(logits[:, :, :n_video].float(), weight)
    with torch.no_grad():
        ranked = z.masked_fill(~columns, -_BELOW_EVERY_SCORE).sort(
            -1, descending=True).values
        last = n_video - 1
        kth = (budget - 1).clamp(min=0, max=last).unsqueeze(-1)
        cut = 0.5 * (ranked.gather(-1, kth)
                     + ranked.gather(-1, (kth + 1).clamp(max=last)))
    policy = torch.sigmoid((z - cut) / temperature) * weight
    spend = budget.unsqueeze(-1).float() / policy.sum(-1, keepdim=True).clamp(
        min=1e-6)
    retained = (policy * spend * mass).sum(-1) / ceiling.clamp(
        min=torch.finfo(torch.float32).tiny)
    return -_mean_rows_then_heads(retained, live)


# Floor of the teacher's block probability relative to the row's largest,
# for the logarithm that sets the row's scale (heatmap.py:336-340).
GAUGE_FLOOR = 1e-6


def gauge_fixed_kl(logits: torch.Tensor, heat: torch.Tensor,
                   layout: tiling.TileLayout,
                   q_tiles: torch.Tensor) -> torch.Tensor:
    """Forward KL(teacher || student) over the decision columns after
    moving the student's standardised scores onto the teacher's own
    log-probability scale (heatmap.py:341-430).

    Per row: t = the teacher's mass normalised over the decision columns,
    floored at GAUGE_FLOOR times its row maximum; the student's scores are
    standardised and mapped to mean(log t) + std(log t) * z; the row's term
    is sum t * (log t - log softmax). 0 when the student reproduces the
    teacher up to a per-row positive affine map; rows without teacher mass
    do not count.

    Args:
        logits: [H', R, n_tiles] fp32 student logits (with grad).
        heat: [H', R, n_tiles] teacher heat (the mass reduction).
        layout: Tile layout.
        q_tiles: [R] int64 supervised video query tiles.

    Returns:
        Scalar divergence (rows averaged, then heads).
    """
    n_video = layout.n_video_tiles
    q_tiles = q_tiles.to(device=logits.device, dtype=torch.int64)
    columns = _decision_columns(layout, q_tiles)
    weight = columns.float()
    count = weight.sum(-1, keepdim=True).clamp(min=1.0)
    tiny = torch.finfo(torch.float32).tiny
    with torch.no_grad():
        mass = _video_mass(heat, columns)
        total = mass.sum(-1, keepdim=True)
        live = total.squeeze(-1) > 0
        teacher = mass / total.clamp(min=tiny)
        floor = GAUGE_FLOOR * teacher.amax(-1, keepdim=True).clamp(min=tiny)
        log_teacher = torch.maximum(teacher, floor).log()
        level = (log_teacher * weight).sum(-1, keepdim=True) / count
        spread = (((log_teacher - level) * weight).square() * weight).sum(
            -1, keepdim=True) / count
    z = _standardise(logits[:, :, :n_video].float(), weight)
    moved = z * spread.sqrt() + level
    log_student = F.log_softmax(moved.masked_fill(~columns, float('-inf')),
                                dim=-1)
    # Excluded columns carry teacher weight 0; their log is -inf, so zero
    # it before the product (0 * -inf would be NaN).
    log_student = log_student.masked_fill(~columns, 0.0)
    per_row = (teacher * (log_teacher - log_student) * weight).sum(-1)
    return _mean_rows_then_heads(per_row, live)


def oracle_bce(logits: torch.Tensor, heat: torch.Tensor,
               layout: tiling.TileLayout,
               blocks: list[veda_mask.ColumnBlock],
               q_tiles: torch.Tensor,
               oracle: torch.Tensor | None = None) -> torch.Tensor:
    """Class-balanced BCE of the row-centred student logits against the
    oracle's top-k set over the decision columns (heatmap.py:433-496).

    Each row's logits are centred on their mean over the decision columns;
    the BCE terms of the oracle's members and of the other decision columns
    are averaged separately (over all heads and rows) and the two means
    halved. An indifferent predictor scores ln 2; 0 when no decision
    column exists.

    Args:
        logits: [H', R, n_tiles] fp32 student logits (with grad).
        heat: [H', R, n_tiles] teacher heat.
        layout: Tile layout.
        blocks: Column blocks with their budgets.
        q_tiles: [R] int64 supervised video query tiles.
        oracle: The heat's own selection, `oracle_set(heat, ...)`, if the
            caller has it already.

    Returns:
        Scalar loss.
    """
    n_video = layout.n_video_tiles
    q_tiles = q_tiles.to(device=logits.device, dtype=torch.int64)
    with torch.no_grad():
        if oracle is None:
            oracle = oracle_set(heat, layout, blocks, q_tiles)
        columns = _decision_columns(layout, q_tiles)
        members = oracle & columns
        others = ~oracle & columns
    weight = columns.float()
    scores = logits[:, :, :n_video].float()
    count = weight.sum(-1, keepdim=True).clamp(min=1.0)
    centred = scores - (scores * weight).sum(-1, keepdim=True) / count
    terms = F.binary_cross_entropy_with_logits(centred, oracle.float(),
                                               reduction='none')
    loss = 0.5 * ((terms * members).sum() / members.sum().clamp(min=1)
                  + (terms * others).sum() / others.sum().clamp(min=1))
    # Decided on the device, so the host never waits for the counts.
    return torch.where(columns.any(), loss, torch.zeros_like(loss))


@torch.no_grad()
def mask_diagnostics(logits: torch.Tensor, heat: torch.Tensor,
                     layout: tiling.TileLayout,
                     blocks: list[veda_mask.ColumnBlock],
                     q_tiles: torch.Tensor,
                     oracle: torch.Tensor | None = None
                     ) -> dict[str, torch.Tensor]:
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
        oracle: The heat's own selection, `oracle_set(heat, ...)`, if the
            caller has it already.
    """
    n_video = layout.n_video_tiles
    q_tiles = q_tiles.to(device=logits.device, dtype=torch.int64)
    predicted = oracle_set(logits, layout, blocks, q_tiles)
    if oracle is None:
        oracle = oracle_set(heat, layout, blocks, q_tiles)
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
