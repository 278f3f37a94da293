"""Veda attention functions: the pluggable `AttentionFn` callables.

Mirror of the reference's `miowtion/veda/attention.py` for the sparse
student: `SparseStudent(clip, plan, predictor)(q, k, v, layer_index)` with
q, k, v [S, H, D] bf16 returns [S, H, D] bf16 (the `AttentionFn` protocol of
miowtion/h3/model.py:40-45). Every stage is a CUDA kernel of this package:
    gather+pool q, k  ->  gather v  ->  predictor logits  ->  top-k lists
    ->  tcgen05 block-sparse attention  ->  inverse permutation.
The block lists go from the selection kernel straight to the attention
kernel; no dense block mask and no Selection are materialised, and nothing
synchronises the host. With gradients enabled (the stage-2 student step,
attention.py:335-359 of the reference) q, k and v receive gradients through
the permutation and the sparse attention (the selection itself is discrete);
the backward walks transposed key-tile lists built from the same selection.
"""

from __future__ import annotations

import dataclasses

import torch

from miowtion_b200 import compensation
from miowtion_b200 import heatmap
from miowtion_b200 import kernels
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import predictor as veda_predictor
from miowtion_b200 import tiling

# Default VedaConfig.collect_bytes (attention.py:30-34): bound on one
# tile-ordered copy. The B200's 180 GB make the default one group per launch.
DEFAULT_COLLECT_BYTES = 64 * 2**30


@dataclasses.dataclass(frozen=True)
class VedaConfig:
    """Sparsity settings (attention.py:37-135; the fields the sparse path
    and the stage-1 teacher read).

    The teacher's supervision: `heat_reduce` ('max' peak probability or
    'sum' mass per block), `kl_weight` and `kl_direction` of the seer KL,
    `teacher_q_tiles` (supervised video query tiles per layer and head
    group: a fraction of the video tiles when <= 1, else a count) and
    `recall_every` (diagnostics on every n-th layer). `transport_weight`
    and `gauge_kl_weight` add the retained-transport-mass loss and the
    gauge-fixed KL (`heatmap.transport_loss`, `heatmap.gauge_fixed_kl`)
    to the seer KL (attention.py:52-63)."""

    heat_reduce: str = 'max'
    transport_weight: float = 0.0
    gauge_kl_weight: float = 0.0
    kl_weight: float = 1.0
    kl_direction: str = 'forward'
    teacher_q_tiles: float = 1.0
    recall_every: int = 1
    target_budget: veda_mask.Budget = veda_mask.Budget(ratio=0.1)
    ref_budget: veda_mask.Budget | None = None
    tile_conditions: bool = False
    budget_rule: str = 'topk'
    # Sol's zero-order term for the dropped tiles (attention.py:70-94). The
    # torch form and the Triton form are one B200 kernel here
    # (compensation.py); the INT8 fused arm has none.
    zero_order_compensation: bool = False
    fused_compensation: bool = False
    triton_compensation: bool = False
    dense_layers: frozenset[int] = frozenset()
    collect_bytes: int = DEFAULT_COLLECT_BYTES

    @property
    def compensated(self) -> bool:
        return self.zero_order_compensation or self.triton_compensation


@dataclasses.dataclass(frozen=True)
class VideoSpan:
    """A run of video-like rows on a (T, H, W) grid (h3/layout.py:42-67)."""

    start: int
    grid: tuple[int, int, int]
    role: str = 'target'


@dataclasses.dataclass
class PackedLayout:
    """The parts of the reference's `h3.layout.PackedLayout`
    (h3/layout.py:70-108) the Veda path reads: packed length, real rows and
    the video spans (target last)."""

    seq_len: int
    used: int
    spans: tuple[VideoSpan, ...]

    @property
    def target(self) -> VideoSpan:
        return self.spans[-1]


class ClipTiling:
    """Tile layouts of one clip, one per target shape (attention.py:138-197)."""

    def __init__(self, layout: PackedLayout, config: VedaConfig,
                 device: torch.device,
                 condition_spans: tuple[tiling.TiledSpan, ...] = ()):
        chosen = [name for name in ('zero_order_compensation',
                                    'fused_compensation',
                                    'triton_compensation')
                  if getattr(config, name)]
        if len(chosen) > 1:
            raise ValueError(
                f'{" and ".join(chosen)} compute the same term; pick one, '
                'they are implementations of it')
        if config.budget_rule not in ('topk', 'threshold'):
            raise ValueError("budget_rule must be 'topk' or 'threshold': "
                             f'{config.budget_rule!r}')
        self.layout = layout
        self.config = config
        self.device = torch.device(device)
        spans = list(condition_spans)
        if config.tile_conditions:
            spans += [tiling.TiledSpan(s.start, s.grid,
                                       tiling.least_padding_shape(s.grid))
                      for s in layout.spans[:-1]]
        self._condition_spans = sorted(spans, key=lambda s: s.start)
        self._cache: dict[tiling.TileShape, tiling.TileLayout] = {}

    def get(self, shape: tiling.TileShape) -> tiling.TileLayout:
        if shape not in self._cache:
            target = self.layout.target
            spans = self._condition_spans + [
                tiling.TiledSpan(target.start, target.grid, shape)]
            self._cache[shape] = tiling.build_tile_layout(
                spans, self.layout.used, self.layout.seq_len, self.device)
        return self._cache[shape]

    def blocks(self, tile_layout: tiling.TileLayout
               ) -> list[veda_mask.ColumnBlock]:
        return veda_mask.column_blocks(tile_layout, self.config.target_budget,
                                       self.config.ref_budget)

    def num_supervised(self, tile_layout: tiling.TileLayout) -> int:
        """Supervised video query tiles per layer and head group
        (attention.py:193-197)."""
        n_video = tile_layout.n_video_tiles
        value = self.config.teacher_q_tiles
        count = round(value * n_video) if value <= 1 else int(value)
        return max(1, min(n_video, count))


_HEAD_DIM_BYTES = 128 * 2


def _chunk_heads(tile_layout: tiling.TileLayout, collect_bytes: int) -> int:
    """Heads per chunk so one tile-ordered copy stays under collect_bytes
    (attention.py:204-206)."""
    return max(1, collect_bytes // (tile_layout.num_slots * _HEAD_DIM_BYTES))


class StageEvents:
    """Optional per-stage CUDA events on the launching stream (for timing:
    the reference's docs time stages with torch.profiler labels). Records
    (name, start, stop) around each stage of `SparseStudent._attend`."""

    def __init__(self):
        self.records: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def start(self, name: str):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return name, ev

    def stop(self, token) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.records.append((token[0], token[1], ev))

    def totals_ms(self) -> dict[str, float]:
        torch.cuda.synchronize()
        out: dict[str, float] = {}
        for name, a, b in self.records:
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out

    def clear(self) -> None:
        self.records.clear()


class _NoEvents:
    def start(self, name):
        return None

    def stop(self, token):
        pass


_NO_EVENTS = _NoEvents()


class _SparseGroup(torch.autograd.Function):
    """One head group's sparse attention in sequence order, differentiable
    in q, k and v: gather -> block-sparse attention -> inverse permutation,
    and back. The tiles of q and k (gathered with the pooling the predictor
    needs) and both list directions are computed by the caller."""

    @staticmethod
    def forward(ctx, q, k, v, q_tiles, k_tiles, heads, layout, lists,
                t_lists):
        v_tiles = tiling.gather_tiles(v, layout, heads)
        o_tiles, lse = kernels.block_sparse_attention_lists(
            q_tiles, k_tiles, v_tiles, lists, layout, return_lse=True)
        local = torch.arange(heads.numel(), device=q.device)
        out = torch.zeros(q.shape[0], heads.numel(), q.shape[2],
                          dtype=q.dtype, device=q.device)
        tiling.scatter_rows_(out, o_tiles, layout, local)
        ctx.save_for_backward(q_tiles, k_tiles, v_tiles, o_tiles, lse, heads)
        ctx.layout, ctx.lists, ctx.t_lists = layout, lists, t_lists
        ctx.shape = q.shape
        return out

    @staticmethod
    def backward(ctx, dout):
        q_tiles, k_tiles, v_tiles, o_tiles, lse, heads = ctx.saved_tensors
        layout = ctx.layout
        local = torch.arange(heads.numel(), device=dout.device)
        dout = dout.contiguous()
        do_tiles = tiling.gather_tiles(dout, layout, local)
        grads = kernels.block_sparse_attention_bwd(
            q_tiles, k_tiles, v_tiles, o_tiles, do_tiles, lse, ctx.lists,
            ctx.t_lists, layout)
        outs = []
        for g in grads:
            full = torch.zeros(ctx.shape, dtype=g.dtype, device=g.device)
            tiling.scatter_rows_(full, g, layout, heads)
            outs.append(full)
        return (*outs, None, None, None, None, None, None)


def _extra_features(predictor: veda_predictor.TileScorePredictor,
                    tile_layout: tiling.TileLayout,
                    sq_q: torch.Tensor | None, var_k: torch.Tensor | None,
                    rows: torch.Tensor | None = None) -> dict:
    """Keyword inputs of the predictor's optional score terms
    (attention.py:251-288): log B_j from the layout for the count term, the
    pooled E[q^2] (query rows `rows` of it, if given) and Var(k) for the
    second-order head; {} for a plain predictor."""
    extra: dict = {}
    if predictor.count_term:
        extra['log_count'] = veda_predictor.log_tile_counts(tile_layout)
    if predictor.second_order_rank:
        if sq_q is None or var_k is None:
            raise ValueError('the second-order head needs the pooled '
                             'second moments; gather with second=True')
        extra['sq_q'] = sq_q if rows is None else sq_q[:, rows]
        extra['var_k'] = var_k
    return extra


def _gather_pool_moments(x: torch.Tensor, tile_layout: tiling.TileLayout,
                         heads: torch.Tensor, second: bool):
    """(tiles, features, E[x^2], Var(x)) of one gather/pool pass; the
    moments are None unless `second`."""
    if second:
        return tiling.gather_and_pool(x, tile_layout, heads, second=True)
    return (*tiling.gather_and_pool(x, tile_layout, heads), None, None)


# Diagnostic fields of LayerStats in the order resolve() transfers them
# (attention.py:308-310).
STAT_FIELDS = ('kl', 'topk_bce', 'transport', 'logit_std', 'recall',
               'gauge_kl', 'heat_kept', 'heat_ceiling', 'retained')


@dataclasses.dataclass
class LayerStats:
    """Stage-1 diagnostics kept on the device until `resolve()`
    (attention.py:313-347): `kl` one entry per layer, the others one per
    layer and head group (the diagnostics only on the layers they ran)."""

    kl: list = dataclasses.field(default_factory=list)
    topk_bce: list = dataclasses.field(default_factory=list)
    transport: list = dataclasses.field(default_factory=list)
    gauge_kl: list = dataclasses.field(default_factory=list)
    retained: list = dataclasses.field(default_factory=list)
    logit_std: list = dataclasses.field(default_factory=list)
    recall: list = dataclasses.field(default_factory=list)
    heat_kept: list = dataclasses.field(default_factory=list)
    heat_ceiling: list = dataclasses.field(default_factory=list)

    def resolve(self) -> dict[str, list[float]]:
        """Host values of every field, in one device-to-host transfer."""
        fields = {name: getattr(self, name) for name in STAT_FIELDS}
        flat = [t for values in fields.values() for t in values]
        if not flat:
            return {name: [] for name in fields}
        host = torch.stack([t.detach().float().reshape(())
                            for t in flat]).cpu().tolist()
        out, start = {}, 0
        for name, values in fields.items():
            out[name] = host[start:start + len(values)]
            start += len(values)
        return out


class TeacherCollector:
    """Stage-1 attention (attention.py:350-470): returns the dense output
    and, per layer and head group, trains the predictor against the
    teacher's block heat right away.

    Per call: the dense attention with its LSE over all heads (the B200
    dense kernel); per head group of the plan, a seeded sample of video
    query tiles, the group's q and k gathered and pooled, the heat of the
    sampled tiles (`veda_teacher_heat`, reduce `config.heat_reduce`), the
    predictor's logits of those tiles with gradients, the seer KL (plus,
    when their weights are non-zero, the transport loss, the gauge-fixed KL
    and `topk_weight` times the oracle BCE) and its backward, scaled so the
    sum over groups is the head-weighted mean times `grad_scale`. The heat's
    own top-k is selected once per group for the terms and diagnostics that
    compare against it. No graph outlives the call; diagnostics stay on the
    device in `stats`.
    """

    def __init__(self, clip: ClipTiling, plan: veda_plan.TilePlan,
                 predictor: veda_predictor.TileScorePredictor,
                 generator: torch.Generator, grad_scale: float,
                 dense_backend: str = 'auto', topk_weight: float = 0.0):
        config = clip.config
        if config.heat_reduce not in ('max', 'sum'):
            raise ValueError(f"heat_reduce must be 'max' or 'sum': "
                             f'{config.heat_reduce!r}')
        reason = kernels.unavailable_reason(clip.device)
        if reason is not None:
            raise RuntimeError(f'TeacherCollector needs the B200 kernels '
                               f'({reason}); refusing to fall back silently')
        self.clip = clip
        self.plan = plan
        self.predictor = predictor
        self.generator = generator
        self.grad_scale = grad_scale
        self.dense_backend = dense_backend
        self.topk_weight = topk_weight
        self.stats = LayerStats()
        self._num_heads = sum(
            g.heads.numel() for g in plan.head_groups(0, clip.device))

    def _sample_rows(self, tile_layout: tiling.TileLayout) -> torch.Tensor:
        """Sorted supervised video query tiles, drawn from the generator
        exactly as attention.py:385-389 draws them."""
        count = self.clip.num_supervised(tile_layout)
        rows = torch.randperm(tile_layout.n_video_tiles,
                              generator=self.generator)[:count]
        return rows.sort().values.to(self.clip.device)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 layer_index: int) -> torch.Tensor:
        config = self.clip.config
        out, lse = dense_attention(q, k, v, self.clip.layout.used,
                                   return_lse=True,
                                   backend=self.dense_backend)
        layer_kl = None
        for group in self.plan.head_groups(layer_index, self.clip.device):
            tile_layout = self.clip.get(group.shape)
            rows = self._sample_rows(tile_layout)
            for heads in group.heads.split(
                    _chunk_heads(tile_layout, config.collect_bytes)):
                second = bool(self.predictor.second_order_rank)
                with torch.no_grad():
                    q_tiles, feats_q, sq_q, _ = _gather_pool_moments(
                        q.detach(), tile_layout, heads, second)
                    k_tiles, feats_k, _, var_k = _gather_pool_moments(
                        k.detach(), tile_layout, heads, second)
                    heat = heatmap.teacher_heat(
                        q_tiles, k_tiles,
                        tiling.gather_lse(lse, tile_layout, heads),
                        tile_layout, rows, config.heat_reduce)
                del q_tiles, k_tiles
                weight = heads.numel() / self._num_heads
                blocks = self.clip.blocks(tile_layout)
                diagnose = layer_index % config.recall_every == 0
                # The heat's own top-k, selected once for every term that
                # compares against it.
                oracle = (heatmap.oracle_set(heat, tile_layout, blocks, rows)
                          if (config.transport_weight or self.topk_weight
                              or diagnose) else None)
                extra = _extra_features(self.predictor, tile_layout, sq_q,
                                        var_k, rows)
                with torch.enable_grad():
                    logits = self.predictor.layers[layer_index](
                        feats_q[:, rows], feats_k, heads, **extra)
                    kl = heatmap.seer_kl(logits, heat, tile_layout,
                                         config.kl_direction)
                    loss = config.kl_weight * kl
                    if config.transport_weight:
                        transport = heatmap.transport_loss(
                            logits, heat, tile_layout, blocks, rows,
                            oracle=oracle)
                        loss = loss + config.transport_weight * transport
                        self.stats.transport.append(transport.detach())
                    if config.gauge_kl_weight:
                        gauge = heatmap.gauge_fixed_kl(logits, heat,
                                                       tile_layout, rows)
                        loss = loss + config.gauge_kl_weight * gauge
                        self.stats.gauge_kl.append(gauge.detach())
                    if self.topk_weight:
                        bce = heatmap.oracle_bce(logits, heat, tile_layout,
                                                 blocks, rows, oracle=oracle)
                        loss = loss + self.topk_weight * bce
                        self.stats.topk_bce.append(bce.detach())
                    (loss * (weight * self.grad_scale)).backward()
                term = kl.detach() * weight
                layer_kl = term if layer_kl is None else layer_kl + term
                self.stats.logit_std.append(
                    logits.detach()[:, :, :tile_layout.n_video_tiles]
                    .std(dim=-1).mean())
                if diagnose:
                    values = heatmap.mask_diagnostics(
                        logits.detach(), heat, tile_layout, blocks, rows,
                        oracle=oracle)
                    for name, value in values.items():
                        getattr(self.stats, name).append(value)
        self.stats.kl.append(layer_kl)
        return out


def _rule_lists(scores: torch.Tensor, tile_layout: tiling.TileLayout,
                clip: ClipTiling, want_mask: bool = False
                ) -> veda_mask.BlockLists:
    """Block lists of the video rows' scores [H', n_video, n] under
    `clip.config.budget_rule`: 'topk' in one selection launch; 'threshold'
    through its Selection, the block mask and the mask's lists
    (attention.py:764-770 and, for the oracle student, :574-580)."""
    blocks = clip.blocks(tile_layout)
    if clip.config.budget_rule == 'topk':
        return veda_mask.select_block_lists(scores, tile_layout, blocks,
                                           want_mask=want_mask)
    selection = veda_mask.select_video_blocks(scores, tile_layout, blocks,
                                              rule='threshold')
    block_mask = veda_mask.dense_block_mask(selection, tile_layout)
    lists = kernels.index_lists_from_mask(block_mask, tile_layout,
                                          transpose=False)
    lists.mask = block_mask
    return lists


class SparseStudent:
    """Stage-2 / evaluation attention: predictor-masked block sparsity
    (attention.py:692-794)."""

    events = _NO_EVENTS  # set a StageEvents to time the stages
    # Called (once per head group on the inference path) before v is first
    # read; the head-parallel wrapper waits there for v's exchange.
    v_ready = None

    def __init__(self, clip: ClipTiling, plan: veda_plan.TilePlan,
                 predictor: veda_predictor.TileScorePredictor,
                 head_offset: int = 0):
        """`head_offset` (not in the reference, which runs every head of a
        layer on one GPU): the predictor's index of the first head of q,
        for a caller that hands this student a contiguous slice of the
        heads (head-parallel ranks, head chunks)."""
        reason = kernels.unavailable_reason(clip.device)
        if reason is not None:
            raise RuntimeError(
                f'SparseStudent needs the B200 block-sparse kernels '
                f'({reason}); refusing to fall back silently')
        if clip.config.fused_compensation:
            raise NotImplementedError(
                'fused_compensation is the INT8 Sol kernel (an external '
                'Triton kernel); use zero_order_compensation or '
                'triton_compensation, which run the B200 compensation '
                'kernel')
        self.clip = clip
        self.plan = plan
        self.predictor = predictor
        self.head_offset = head_offset
        self.calls = {'sparse': 0, 'dense': 0}

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 layer_index: int, out: torch.Tensor | None = None
                 ) -> torch.Tensor:
        """`out` (not in the reference's AttentionFn): an optional
        preallocated [S, H, D] output for the inference path, which the
        layer then writes in place (the head-parallel wrapper passes a
        buffer its peers read)."""
        used = self.clip.layout.used
        grad = torch.is_grad_enabled() and any(t.requires_grad
                                               for t in (q, k, v))
        if out is not None and (grad or out.shape != q.shape or
                                out.dtype != q.dtype or
                                out.device != q.device or
                                not out.is_contiguous()):
            raise ValueError('out must be a contiguous tensor like q, and '
                             'is for the inference path only')
        if layer_index in self.clip.config.dense_layers:
            self._wait_v()
            self.calls['dense'] += 1
            result = kernels.dense_attention(q, k, v, q.shape[-1] ** -0.5,
                                             False, used=used)[0]
            if out is None:
                return result
            out.copy_(result)
            return out
        self.calls['sparse'] += 1
        if grad:
            self._wait_v()
            return self._attend_grad(q, k, v, layer_index)
        seq_len = q.shape[0]
        if out is None:
            out = torch.empty_like(q)
        if used < seq_len:
            out[used:] = 0
        covered = 0
        for group in self.plan.head_groups(layer_index, self.clip.device):
            tile_layout = self.clip.get(group.shape)
            covered += group.heads.numel()
            for heads in group.heads.split(
                    _chunk_heads(tile_layout, self.clip.config.collect_bytes)):
                self._attend(q, k, v, layer_index, tile_layout, heads, out)
        if covered != q.shape[1]:
            raise ValueError(f'the plan covers {covered} heads, q has '
                             f'{q.shape[1]}')
        return out

    def _wait_v(self) -> None:
        if self.v_ready is not None:
            self.v_ready()

    def _attend(self, q, k, v, layer_index: int,
                tile_layout: tiling.TileLayout, heads: torch.Tensor,
                out: torch.Tensor) -> None:
        """Sparse attention of some heads of one group, scattered to out."""
        second = bool(self.predictor.second_order_rank)
        if (not self.clip.config.compensated and not second
                and self.clip.config.budget_rule == 'topk'
                and kernels.packed_supported(tile_layout)):
            self._attend_packed(q, k, v, layer_index, tile_layout, heads, out)
            return
        self._wait_v()
        ev = self.events
        t = ev.start('permute_pool')
        q_tiles, feats_q, sq_q, _ = _gather_pool_moments(q, tile_layout,
                                                         heads, second)
        k_tiles, feats_k, _, var_k = _gather_pool_moments(k, tile_layout,
                                                          heads, second)
        v_tiles = tiling.gather_tiles(v, tile_layout, heads)
        ev.stop(t)
        with torch.no_grad():
            t = ev.start('score')
            logits = self.predictor.layers[layer_index](
                feats_q, feats_k, heads + self.head_offset,
                **_extra_features(self.predictor, tile_layout, sq_q, var_k))
            ev.stop(t)
            t = ev.start('topk')
            lists = self._block_lists(logits, tile_layout)
            ev.stop(t)
        t = ev.start('attention')
        if self.clip.config.compensated:
            o_tiles, lse = kernels.block_sparse_attention_lists(
                q_tiles, k_tiles, v_tiles, lists, tile_layout,
                return_lse=True)
            compensation.compensate_lists(o_tiles, lse, q_tiles, k_tiles,
                                          v_tiles, lists, tile_layout,
                                          out=o_tiles)
        else:
            o_tiles = kernels.block_sparse_attention_lists(
                q_tiles, k_tiles, v_tiles, lists, tile_layout)
        ev.stop(t)
        t = ev.start('unpermute')
        tiling.scatter_rows_(out, o_tiles, tile_layout, heads)
        ev.stop(t)
        self.last_lists = lists

    def _block_lists(self, logits: torch.Tensor,
                     tile_layout: tiling.TileLayout,
                     want_mask: bool = False) -> veda_mask.BlockLists:
        """Lists of the logits under `config.budget_rule`: 'topk' in one
        selection launch; 'threshold' through its Selection, the block
        mask and the mask's lists (attention.py:764-770)."""
        return _rule_lists(logits[:, :tile_layout.n_video_tiles],
                           tile_layout, self.clip, want_mask)

    def _attend_packed(self, q, k, v, layer_index: int,
                       tile_layout: tiling.TileLayout, heads: torch.Tensor,
                       out: torch.Tensor) -> None:
        """`_attend` without the tile-ordered q and output: pooling reads q
        in place, and the attention kernel reads query tiles as boxes of the
        packed q and writes out directly (no gather of q, no scatter). Key
        and value tiles are gathered once into shared-memory images, which
        the kernel loads with one bulk copy each."""
        ev = self.events
        t = ev.start('permute_pool')
        feats_q = tiling.pool_features(q, tile_layout, heads)
        k_img, feats_k = tiling.gather_images(k, tile_layout, heads,
                                              pool=True)
        ev.stop(t)
        with torch.no_grad():
            t = ev.start('score')
            logits = self.predictor.layers[layer_index](
                feats_q, feats_k, heads + self.head_offset,
                **_extra_features(self.predictor, tile_layout, None, None))
            ev.stop(t)
            t = ev.start('topk')
            lists = veda_mask.select_block_lists(
                logits[:, :tile_layout.n_video_tiles], tile_layout,
                self.clip.blocks(tile_layout))
            ev.stop(t)
        # v is first read here, after the scoring: a caller that is still
        # receiving v (the head-parallel exchange) lets it arrive meanwhile.
        self._wait_v()
        t = ev.start('permute_pool')
        v_img = tiling.gather_images(v, tile_layout, heads)
        ev.stop(t)
        t = ev.start('attention')
        kernels.block_sparse_attention_packed(
            q, k_img, v_img, lists, tile_layout, heads, out,
            kv_tiles='images',
            order=kernels.work_order(tile_layout, heads.numel(),
                                     self.clip.blocks(tile_layout),
                                     q.device))
        ev.stop(t)
        self.last_lists = lists

    def _attend_grad(self, q, k, v, layer_index: int) -> torch.Tensor:
        """The differentiable layer: per head group, the forward of
        `_attend` inside `_SparseGroup`, plus the transposed lists the
        backward walks (fa4.py:353-359)."""
        if self.clip.config.compensated:
            raise NotImplementedError(
                'the zero-order compensation is an evaluation arm; it has '
                'no backward')
        parts, all_heads = [], []
        for group in self.plan.head_groups(layer_index, self.clip.device):
            tile_layout = self.clip.get(group.shape)
            heads = group.heads
            second = bool(self.predictor.second_order_rank)
            with torch.no_grad():
                q_tiles, feats_q, sq_q, _ = _gather_pool_moments(
                    q.detach(), tile_layout, heads, second)
                k_tiles, feats_k, _, var_k = _gather_pool_moments(
                    k.detach(), tile_layout, heads, second)
                logits = self.predictor.layers[layer_index](
                    feats_q, feats_k, heads + self.head_offset,
                    **_extra_features(self.predictor, tile_layout, sq_q,
                                      var_k))
                lists = self._block_lists(logits, tile_layout,
                                          want_mask=True)
                t_lists = kernels.index_lists_from_mask(lists.mask,
                                                        tile_layout)
            parts.append(_SparseGroup.apply(q, k, v, q_tiles, k_tiles, heads,
                                            tile_layout, lists, t_lists))
            all_heads.append(heads)
            self.last_lists = lists
        heads = torch.cat(all_heads)
        if heads.numel() != q.shape[1]:
            raise ValueError(f'the plan covers {heads.numel()} heads, q has '
                             f'{q.shape[1]}')
        out = torch.zeros_like(q)
        return out.index_copy(1, heads, torch.cat(parts, 1))


DENSE_BACKENDS = ('auto', 'b200', 'fa4', 'sdpa')


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    used: int, return_lse: bool = False,
                    backend: str = 'auto'
                    ) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Full attention of rows [0, used) among themselves, the reference's
    `h3.attention.dense_attention` (h3/attention.py:28-102): out [S, H, D]
    zero on padding rows, lse [S, H] fp32 natural log (0 on padding rows).

    Every CUDA backend name runs the B200 dense kernel; 'math' (the
    reference's fp32 CPU path) has none here.

    Raises:
        ValueError: On an unknown backend.
        NotImplementedError: For 'math', or off B200.
    """
    if backend == 'math':
        raise NotImplementedError("backend 'math' is the reference's fp32 "
                                  'CPU path; this package runs on B200 only')
    if backend not in DENSE_BACKENDS:
        raise ValueError(f'unknown dense backend {backend!r}')
    return kernels.dense_attention(q, k, v, q.shape[-1] ** -0.5, return_lse,
                                   used=used)


class DenseAttention:
    """The dense teacher AttentionFn (h3/model.py:48-58)."""

    def __init__(self, used: int, backend: str = 'auto'):
        self.used = used
        self.backend = backend

    def __call__(self, q, k, v, layer_index):
        del layer_index
        return dense_attention(q, k, v, self.used, backend=self.backend)[0]


ORACLE_TARGETS = ('mass', 'max', 'mean')


class OracleStudent:
    """Block sparsity masked by the true block statistic instead of a
    predictor (attention.py:474-588): an upper bound for the router.

    Targets: 'mass' (the block's summed attention probability), 'max' (its
    peak probability), 'mean' (mass per real key row). Per head group, one
    fused pass gives the dense teacher's normalisation and the block heat of
    every query tile (`heatmap.fused_dense_heat`; its dense output is not
    used), the training rules select the blocks from the video rows' heat,
    and the sparse kernel attends over them. Cost is dense plus sparse per
    layer: an analysis mode, never an inference path.

    `allow_reference_kernel` is accepted for the reference's signature; there
    is no reference kernel here, so it changes nothing.
    """

    def __init__(self, clip: ClipTiling, plan: veda_plan.TilePlan,
                 target: str = 'mass', allow_reference_kernel: bool = False):
        del allow_reference_kernel
        if target not in ORACLE_TARGETS:
            raise ValueError(f'target must be one of {ORACLE_TARGETS}: '
                             f'{target!r}')
        reason = kernels.unavailable_reason(clip.device)
        if reason is not None:
            raise RuntimeError(
                f'OracleStudent needs the B200 block-sparse kernels '
                f'({reason}); refusing to fall back silently')
        self.clip = clip
        self.plan = plan
        self.target = target
        self.calls = {'sparse': 0, 'dense': 0}

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 layer_index: int) -> torch.Tensor:
        used = self.clip.layout.used
        if layer_index in self.clip.config.dense_layers:
            self.calls['dense'] += 1
            return dense_attention(q, k, v, used)[0]
        self.calls['sparse'] += 1
        seq_len = q.shape[0]
        out = torch.empty_like(q)
        if used < seq_len:
            out[used:] = 0
        for group in self.plan.head_groups(layer_index, self.clip.device):
            tile_layout = self.clip.get(group.shape)
            for heads in group.heads.split(
                    _chunk_heads(tile_layout, self.clip.config.collect_bytes)):
                self._attend(q, k, v, tile_layout, heads, out)
        return out

    @torch.no_grad()
    def _attend(self, q, k, v, tile_layout: tiling.TileLayout,
                heads: torch.Tensor, out: torch.Tensor) -> None:
        q_tiles = tiling.gather_tiles(q, tile_layout, heads)
        k_tiles = tiling.gather_tiles(k, tile_layout, heads)
        v_tiles = tiling.gather_tiles(v, tile_layout, heads)
        reduce = 'max' if self.target == 'max' else 'sum'
        _, _, heat = heatmap.fused_dense_heat(q_tiles, k_tiles, v_tiles,
                                              tile_layout, reduce)
        heat = heat[:, :tile_layout.n_video_tiles]
        if self.target == 'mean':
            counts = tile_layout.valid_count.clamp(min=1).to(heat.dtype)
            heat = heat / counts[None, None, :]
        lists = _rule_lists(heat, tile_layout, self.clip, want_mask=True)
        o_tiles = kernels.block_sparse_attention_lists(
            q_tiles, k_tiles, v_tiles, lists, tile_layout)
        tiling.scatter_rows_(out, o_tiles, tile_layout, heads)
        self.last_lists = lists
