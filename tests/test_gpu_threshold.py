"""The 'threshold' budget rule on the B200: `select_video_blocks(...,
rule='threshold')` against the reference's selection
(tests/golden/make_threshold.py) and SparseStudent under
`budget_rule='threshold'`."""

import os

import numpy as np
import pytest
import torch

import inputs
from miowtion_b200 import _lib
from miowtion_b200 import attention as veda_attention
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import predictor as veda_predictor
from miowtion_b200 import tiling

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda')
GOLDEN = os.path.join(os.path.dirname(__file__), 'golden', 'threshold.npz')


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0, 'a kernel wait timed out'


def _layout(spec):
    return tiling.build_tile_layout(
        [tiling.TiledSpan(s, tuple(g), tiling.TileShape(*sh))
         for s, g, sh in spec['spans']], spec['used'], spec['seq_len'], DEV)


@pytest.mark.parametrize('case', ['padded', 'padded_rows', 'segmented'])
def test_threshold_selection_matches_reference(case):
    golden = np.load(GOLDEN)
    pad, seg = inputs.PADDED, inputs.SEGMENTED
    rows = None
    if case == 'segmented':
        lay = _layout(seg)
        blocks = veda_mask.column_blocks(
            lay, veda_mask.Budget(ratio=seg['target_ratio']),
            veda_mask.Budget(ratio=seg['ref_ratio']))
    else:
        lay = _layout(pad)
        blocks = veda_mask.column_blocks(lay,
                                         veda_mask.Budget(ratio=pad['ratio']))
        if case == 'padded_rows':
            rows = torch.tensor(inputs.THRESHOLD['rows'], device=DEV)
    scores = torch.from_numpy(golden[f'{case}_scores']).to(DEV)
    sel = veda_mask.select_video_blocks(scores, lay, blocks, rows,
                                        rule='threshold')
    assert np.array_equal(sel.keep.cpu().numpy(), golden[f'{case}_keep'])
    assert np.array_equal(sel.index.cpu().numpy(), golden[f'{case}_index'])


def test_student_with_threshold_rule():
    heads, seq_len, text, grid = 4, 1100, 130, (4, 12, 20)
    used = text + grid[0] * grid[1] * grid[2]
    q, k, v = (x.to(DEV) for x in inputs.qkv(seq_len, heads, 128, 85,
                                             torch.bfloat16))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=0.4), budget_rule='threshold')
    clip = veda_attention.ClipTiling(veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),)), config, DEV)
    plan = veda_plan.TilePlan('thr', grid, [tiling.TileShape(2, 8, 8)],
                              [[0] * heads])
    pred = veda_predictor.TileScorePredictor(1, heads, 128)
    with torch.no_grad():
        pq, pk = inputs.predictor_weights(heads, 128, 86, 0.02)
        pred.layers[0].proj_q.copy_(pq)
        pred.layers[0].proj_k.copy_(pk)
    student = veda_attention.SparseStudent(clip, plan, pred.to(DEV))
    out = student(q, k, v, 0)
    lay = clip.get(tiling.TileShape(2, 8, 8))
    all_heads = torch.arange(heads, device=DEV)
    _, fq = tiling.gather_and_pool(q, lay, all_heads)
    _, fk = tiling.gather_and_pool(k, lay, all_heads)
    with torch.no_grad():
        logits = pred.layers[0](fq, fk, all_heads)
    sel = veda_mask.select_video_blocks(
        logits[:, :lay.n_video_tiles], lay, clip.blocks(lay),
        rule='threshold')
    want = veda_mask.dense_block_mask(sel, lay)
    torch.cuda.synchronize()
    assert torch.equal(student.last_lists.mask.bool(), want)
    kept = want[:, :lay.n_video_tiles, :lay.n_video_tiles].sum(-1)
    assert kept.float().std() > 0, 'the rule should keep uneven counts'
    assert torch.isfinite(out[:used].float()).all()


def test_oracle_student_with_threshold_rule():
    """OracleStudent passes the clip's budget rule to the selection, as the
    reference does (attention.py:574-580): under 'threshold' its block mask
    is the threshold selection of the true block mass of the video rows."""
    from miowtion_b200 import heatmap
    heads, seq_len, text, grid = 3, 1100, 130, (4, 12, 20)
    used = text + grid[0] * grid[1] * grid[2]
    q, k, v = (x.to(DEV) for x in inputs.qkv(seq_len, heads, 128, 87,
                                             torch.bfloat16))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=0.4), budget_rule='threshold')
    clip = veda_attention.ClipTiling(veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),)), config, DEV)
    plan = veda_plan.TilePlan('thr', grid, [tiling.TileShape(2, 8, 8)],
                              [[0] * heads])
    student = veda_attention.OracleStudent(clip, plan, 'mass')
    out = student(q, k, v, 0)
    lay = clip.get(tiling.TileShape(2, 8, 8))
    all_heads = torch.arange(heads, device=DEV)
    qt, kt, vt = (tiling.gather_tiles(t, lay, all_heads) for t in (q, k, v))
    _, _, heat = heatmap.fused_dense_heat(qt, kt, vt, lay, 'sum')
    sel = veda_mask.select_video_blocks(
        heat[:, :lay.n_video_tiles], lay, clip.blocks(lay), rule='threshold')
    want = veda_mask.dense_block_mask(sel, lay)
    torch.cuda.synchronize()
    assert torch.equal(student.last_lists.mask.bool(), want)
    kept = want[:, :lay.n_video_tiles, :lay.n_video_tiles].sum(-1)
    assert kept.float().std() > 0, 'the rule should keep uneven counts'
    assert torch.isfinite(out[:used].float()).all()
