"""TeacherCollector (stage 1) on the B200 kernels against the reference's
own collector run on the CPU (tests/golden/make_teacher.py): the dense
output, the per-layer seer KL, the diagnostics, the ablation losses and
the predictor's gradients, for a heat reduction / KL direction /
supervision share / loss weighting each."""

import os

import numpy as np
import pytest
import torch

import inputs
from miowtion_b200 import _lib
from miowtion_b200 import attention as veda_attention
from miowtion_b200 import heatmap
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import predictor as veda_predictor
from miowtion_b200 import tiling

pytestmark = pytest.mark.gpu

DEV = torch.device('cuda')
GOLDEN = os.path.join(os.path.dirname(__file__), 'golden', 'teacher.npz')


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0, 'a kernel wait timed out'


def run_case(spec, heat_reduce, direction, q_tiles, weights=None):
    weights = dict(weights or {})
    topk_weight = weights.pop('topk_weight', 0.0)
    text, grid, seq_len = spec['text'], spec['grid'], spec['seq_len']
    used = text + grid[0] * grid[1] * grid[2]
    q, k, v = (t.to(DEV) for t in inputs.qkv(seq_len, spec['heads'],
                                             spec['dim'], spec['seed'],
                                             torch.bfloat16))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=spec['ratio']),
        heat_reduce=heat_reduce, kl_direction=direction,
        teacher_q_tiles=q_tiles, **weights)
    layout = veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),))
    clip = veda_attention.ClipTiling(layout, config, DEV)
    plan = veda_plan.TilePlan(
        'teacher', grid, [tiling.TileShape(*s) for s in spec['shapes']],
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
    predictor = predictor.to(DEV)
    gen = torch.Generator().manual_seed(spec['gen_seed'])
    teacher = veda_attention.TeacherCollector(clip, plan, predictor, gen,
                                              spec['grad_scale'],
                                              topk_weight=topk_weight)
    outs = [teacher(q, k, v, layer) for layer in range(spec['layers'])]
    torch.cuda.synchronize()
    return outs, teacher.stats.resolve(), predictor


@pytest.mark.parametrize('case', sorted(inputs.TEACHER['cases']))
def test_teacher_collector_matches_reference(case):
    spec = inputs.TEACHER
    golden = np.load(GOLDEN)
    want = {name[len(case) + 2:]: golden[name] for name in golden.files
            if name.startswith(case + '__')}
    outs, stats, predictor = run_case(spec, *spec['cases'][case])
    # Dense output: the reference's fp32 'math' teacher, rows [::4].
    got = outs[0][::4].float().cpu().numpy()
    np.testing.assert_allclose(got, want['out_rows'].astype(np.float32),
                               rtol=2e-2, atol=2e-2)
    # One KL per layer: the head-weighted seer KL, within the heat's own
    # tolerance.
    np.testing.assert_allclose(stats['kl'], want['kl'], rtol=3e-2,
                               atol=1e-4)
    # The logits are fp32 on both sides.
    np.testing.assert_allclose(stats['logit_std'], want['logit_std'],
                               rtol=1e-4)
    for name in ('recall', 'heat_kept', 'heat_ceiling', 'retained'):
        np.testing.assert_allclose(stats[name], want[name], rtol=0,
                                   atol=0.05, equal_nan=True, err_msg=name)
    # The ablation losses, where the case weights them: one value per
    # layer and head group, from the heat within its tolerance.
    for name in ('transport', 'gauge_kl', 'topk_bce'):
        if name in want:
            np.testing.assert_allclose(stats[name], want[name], rtol=0,
                                       atol=0.05, err_msg=name)
        else:
            assert stats[name] == [], name
    # Gradients of the projections (feature rows [::12]).
    for i, layer in enumerate(predictor.layers):
        for side, param in (('q', layer.proj_q), ('k', layer.proj_k)):
            g = param.grad[:, ::12].cpu().numpy()
            w = want[f'grad_{side}{i}']
            scale = np.abs(w).max()
            np.testing.assert_allclose(g, w, rtol=0, atol=5e-2 * scale,
                                       err_msg=f'grad_{side}{i}')


def test_ablation_losses_select_the_oracle_set_on_the_gpu():
    """`oracle_set` on the selection kernel reproduces the reference's own
    top-k set of the heat, and the losses that select it themselves match
    the reference's values and gradients (tests/golden/make_teacher.py)."""
    golden = np.load(GOLDEN)
    pad, spec = inputs.PADDED, inputs.LOSSES
    layout = tiling.build_tile_layout(
        [tiling.TiledSpan(s, g, tiling.TileShape(*sh))
         for s, g, sh in pad['spans']], pad['used'], pad['seq_len'], DEV)
    blocks = veda_mask.column_blocks(layout,
                                     veda_mask.Budget(ratio=spec['ratio']))
    rows = torch.tensor(spec['rows'], device=DEV)
    heat = torch.from_numpy(golden['loss_heat']).to(DEV)
    oracle = heatmap.oracle_set(heat, layout, blocks, rows)
    assert np.array_equal(oracle.cpu().numpy(), golden['loss_oracle'])
    cases = {f'transport_{t:g}': lambda x, t=t: heatmap.transport_loss(
        x, heat, layout, blocks, rows, temperature=t)
        for t in spec['temperatures']}
    cases['gauge'] = lambda x: heatmap.gauge_fixed_kl(x, heat, layout, rows)
    cases['bce'] = lambda x: heatmap.oracle_bce(x, heat, layout, blocks,
                                                rows)
    for name, fn in cases.items():
        logits = torch.from_numpy(golden['loss_logits']).to(
            DEV).requires_grad_(True)
        value = fn(logits)
        value.backward()
        np.testing.assert_allclose(value.item(), golden[f'loss_{name}'],
                                   rtol=1e-4, atol=1e-6, err_msg=name)
        want = golden[f'loss_{name}_grad']
        np.testing.assert_allclose(logits.grad.cpu().numpy(), want, rtol=0,
                                   atol=1e-4 * max(1.0, np.abs(want).max()),
                                   err_msg=name)


def test_teacher_output_is_the_dense_attention_and_trains_only_the_predictor():
    """The collector's output is the dense teacher's, bit for bit, and its
    backward reaches only the predictor (the reference's
    tests/unit/test_veda_heatmap_attention.py:108-137)."""
    spec = inputs.TEACHER
    text, grid, seq_len = spec['text'], spec['grid'], spec['seq_len']
    used = text + grid[0] * grid[1] * grid[2]
    q, k, v = (t.to(DEV).requires_grad_(True)
               for t in inputs.qkv(seq_len, spec['heads'], spec['dim'],
                                   spec['seed'], torch.bfloat16))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=spec['ratio']))
    layout = veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),))
    clip = veda_attention.ClipTiling(layout, config, DEV)
    plan = veda_plan.TilePlan(
        'teacher', grid, [tiling.TileShape(*s) for s in spec['shapes']],
        [spec['head_shape']])
    predictor = veda_predictor.TileScorePredictor(1, spec['heads'],
                                                  spec['dim']).to(DEV)
    teacher = veda_attention.TeacherCollector(
        clip, plan, predictor, torch.Generator().manual_seed(3), 1.0)
    out = teacher(q, k, v, 0)
    want = veda_attention.dense_attention(q.detach(), k.detach(), v.detach(),
                                          used)[0]
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert q.grad is None and k.grad is None and v.grad is None
    for layer in predictor.layers:
        assert layer.proj_q.grad is not None and layer.proj_k.grad is not None
        assert layer.proj_q.grad.abs().sum() > 0
