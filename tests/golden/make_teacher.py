"""Golden vectors of the reference's TeacherCollector (stage-1 attention),
run on CPU in the build container:

    PYTHONPATH=<path to the reference checkout> python tests/golden/make_teacher.py

For each case of `inputs.TEACHER` it runs the reference's
`TeacherCollector(clip, plan, predictor, generator, grad_scale)` over two
layers of the same q, k, v (bf16; its dense teacher on the fp32 'math'
backend, its heat through `teacher_heat_reference`) and stores the dense
output (rows [::4]), the per-layer KL and the per-(layer, group)
diagnostics `LayerStats.resolve()` returns, and the predictor's gradients
(feature rows [::12]).
A case may add the ablation losses' weights; its stats then hold the
`transport`, `gauge_kl` and `topk_bce` values too. It also stores `seer_kl`
of seeded logits and heat on the padded layout, in both directions, and
`transport_loss` (at each temperature of `inputs.LOSSES`), `gauge_fixed_kl`
and `oracle_bce` of seeded logits and heat there, each with its gradient
with respect to the logits, and the heat's own top-k set they compare
against. Writes `tests/golden/teacher.npz`.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import inputs  # noqa: E402

from miowtion.h3 import layout as h3_layout  # noqa: E402
from miowtion.veda import attention as veda_attention  # noqa: E402
from miowtion.veda import heatmap  # noqa: E402
from miowtion.veda import mask as veda_mask  # noqa: E402
from miowtion.veda import plan as veda_plan  # noqa: E402
from miowtion.veda import predictor as veda_predictor  # noqa: E402
from miowtion.veda import tiling  # noqa: E402

STATS = ('kl', 'logit_std', 'recall', 'heat_kept', 'heat_ceiling',
         'retained')


def packed_layout(spec):
    text, grid, seq_len = spec['text'], spec['grid'], spec['seq_len']
    used = text + grid[0] * grid[1] * grid[2]
    return h3_layout.PackedLayout(
        seq_len=seq_len, used=used, text_len=text,
        img_pos=torch.arange(text, used),
        audio_pos=torch.zeros(0, dtype=torch.long),
        update_mask=torch.ones(used - text, dtype=torch.bool),
        audio_update_mask=torch.zeros(0, dtype=torch.bool),
        position_ids=torch.zeros(seq_len, 3, dtype=torch.float64),
        token_tags=torch.zeros(seq_len, dtype=torch.long),
        cu_seqlens=torch.tensor([0, used, seq_len], dtype=torch.int32),
        spans=(h3_layout.VideoSpan(text, grid, 'target'),),
        visual_cond_shapes=(), audio_cond_lengths=())


ABLATION_STATS = ('transport', 'gauge_kl', 'topk_bce')


def run_case(spec, heat_reduce, direction, q_tiles, weights=None):
    weights = dict(weights or {})
    topk_weight = weights.pop('topk_weight', 0.0)
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.bfloat16)
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=spec['ratio']),
        heat_reduce=heat_reduce, kl_direction=direction,
        teacher_q_tiles=q_tiles, **weights)
    clip = veda_attention.ClipTiling(packed_layout(spec), config,
                                     torch.device('cpu'))
    plan = veda_plan.TilePlan(
        'teacher', spec['grid'], [tiling.TileShape(*s) for s in
                                  spec['shapes']],
        [spec['head_shape']] * spec['layers'])
    predictor = veda_predictor.TileScorePredictor(
        spec['layers'], spec['heads'], spec['dim'])
    with torch.no_grad():
        for i, layer in enumerate(predictor.layers):
            pq, pk = inputs.predictor_weights(
                spec['heads'], spec['dim'], spec['pred_seed'] + i,
                spec['pred_std'])
            layer.proj_q.copy_(pq)
            layer.proj_k.copy_(pk)
    gen = torch.Generator().manual_seed(spec['gen_seed'])
    teacher = veda_attention.TeacherCollector(
        clip, plan, predictor, gen, spec['grad_scale'], dense_backend='math',
        topk_weight=topk_weight)
    outs = [teacher(q, k, v, layer) for layer in range(spec['layers'])]
    stats = teacher.stats.resolve()
    arrays = {'out_rows': outs[0][::4].float().numpy().astype(np.float16)}
    for name in STATS + ABLATION_STATS:
        if stats[name] or name in STATS:
            arrays[name] = np.asarray(stats[name], dtype=np.float64)
    for i, layer in enumerate(predictor.layers):
        # Rows [::12] of the 384 feature rows keep the fixture small.
        arrays[f'grad_q{i}'] = layer.proj_q.grad[:, ::12].numpy()
        arrays[f'grad_k{i}'] = layer.proj_k.grad[:, ::12].numpy()
    return arrays


def kl_cases():
    """seer_kl of seeded logits / heat on the padded layout (its empty key
    tiles excluded), both directions, plus rows with no heat at all."""
    spec = inputs.PADDED
    spans = [tiling.TiledSpan(s, g, tiling.TileShape(*sh))
             for s, g, sh in spec['spans']]
    lay = tiling.build_tile_layout(spans, spec['used'], spec['seq_len'])
    gen = torch.Generator().manual_seed(91)
    heads, rows, n = 3, 9, lay.n_tiles
    logits = torch.randn(heads, rows, n, generator=gen) * 2.0
    heat = torch.rand(heads, rows, n, generator=gen) ** 4
    heat[:, 2] = 0.0                          # a row without heat
    heat[1, 5, ::3] = -1e-3                   # negative heat is clipped
    arrays = {'kl_logits': logits.numpy(), 'kl_heat': heat.numpy(),
              'kl_kv_ok': lay.kv_ok.numpy()}
    for direction in ('forward', 'reverse'):
        arrays[f'kl_{direction}'] = np.array(heatmap.seer_kl(
            logits, heat, lay, direction).item())
    return arrays


def loss_cases():
    """The ablation losses of seeded logits / heat on the padded layout:
    values and logit gradients, plus the heat's own top-k set. Row 1 has no
    mass (distinct negative heat, clipped to 0, so its top-k is still free
    of ties); one row of head 2 has some negative heat."""
    spec, pad = inputs.LOSSES, inputs.PADDED
    spans = [tiling.TiledSpan(s, g, tiling.TileShape(*sh))
             for s, g, sh in pad['spans']]
    lay = tiling.build_tile_layout(spans, pad['used'], pad['seq_len'])
    blocks = veda_mask.column_blocks(lay, veda_mask.Budget(
        ratio=spec['ratio']))
    rows = torch.tensor(spec['rows'], dtype=torch.int64)
    gen = torch.Generator().manual_seed(spec['seed'])
    shape = (spec['heads'], rows.numel(), lay.n_tiles)
    logits = torch.randn(*shape, generator=gen) * 1.5
    heat = torch.rand(*shape, generator=gen) ** 3
    heat[:, 1] = -1e-3 * torch.rand(*heat[:, 1].shape, generator=gen)
    heat[2, 3, ::4] = -1e-3
    sel = veda_mask.select_video_blocks(heat, lay, blocks, rows)
    chosen = torch.zeros(*sel.index.shape[:2], lay.n_video_tiles,
                         dtype=torch.bool)
    chosen.scatter_(2, sel.index, sel.keep)
    arrays = {'loss_logits': logits.numpy(), 'loss_heat': heat.numpy(),
              'loss_oracle': chosen.numpy()}

    def record(name, fn):
        x = logits.clone().requires_grad_(True)
        value = fn(x)
        value.backward()
        arrays[f'loss_{name}'] = np.array(value.item())
        arrays[f'loss_{name}_grad'] = x.grad.numpy()

    for tau in spec['temperatures']:
        record(f'transport_{tau:g}', lambda x, tau=tau: heatmap.transport_loss(
            x, heat, lay, blocks, rows, temperature=tau))
    record('gauge', lambda x: heatmap.gauge_fixed_kl(x, heat, lay, rows))
    record('bce', lambda x: heatmap.oracle_bce(x, heat, lay, blocks, rows))
    return arrays


def main() -> None:
    spec = inputs.TEACHER
    out = kl_cases()
    out.update(loss_cases())
    for case, args in spec['cases'].items():
        for name, value in run_case(spec, *args).items():
            out[f'{case}__{name}'] = value
    path = os.path.join(HERE, 'teacher.npz')
    np.savez_compressed(path, **out)
    print(f'wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)')


if __name__ == '__main__':
    main()
