"""The predictor's optional score terms on the B200: the layer's logits
(scoring kernel plus the count and second-order terms) and their parameter
gradients against the reference's LayerPredictor
(tests/golden/make_predictor_terms.py), and the terms' inputs reaching the
predictor inside SparseStudent (tile path for the second-order head, packed
path for the count term) and TeacherCollector."""

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
SPEC = inputs.PREDICTOR_TERMS
GOLDEN = os.path.join(os.path.dirname(__file__), 'golden',
                      'predictor_terms.npz')


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0, 'a kernel wait timed out'


def test_layer_with_terms_matches_reference():
    golden = np.load(GOLDEN)
    t = {n: x.to(DEV) for n, x in inputs.predictor_term_inputs(SPEC).items()}
    layer = veda_predictor.LayerPredictor(SPEC['heads'], SPEC['dim'],
                                          SPEC['rank'], count_term=True)
    with torch.no_grad():
        for name in ('proj_q', 'proj_k', 'so_q', 'so_k', 'count_gain'):
            getattr(layer, name).copy_(t[name])
    layer = layer.to(DEV)
    logits = layer(t['feats_q'], t['feats_k'], t['heads'], sq_q=t['sq_q'],
                   var_k=t['var_k'], log_count=t['log_count'])
    want = golden['logits']
    np.testing.assert_allclose(logits.detach().cpu().numpy(), want,
                               rtol=1e-4, atol=1e-4 * np.abs(want).max())
    (logits * t['probe']).sum().backward()
    for name in ('so_q', 'so_k', 'count_gain'):
        ref = golden[f'grad_{name}']
        np.testing.assert_allclose(getattr(layer, name).grad.cpu().numpy(),
                                   ref, rtol=0,
                                   atol=1e-4 * np.abs(ref).max(),
                                   err_msg=name)
    assert torch.isfinite(layer.proj_q.grad).all()


def _predictor(heads, rank, count):
    pred = veda_predictor.TileScorePredictor(1, heads, 128, rank,
                                             count_term=count)
    gen = torch.Generator().manual_seed(71)
    with torch.no_grad():
        layer = pred.layers[0]
        layer.proj_q.normal_(0.0, 0.02, generator=gen)
        layer.proj_k.normal_(0.0, 0.02, generator=gen)
        if rank:
            layer.so_q.normal_(0.0, 0.05, generator=gen)
            layer.so_k.normal_(0.0, 0.05, generator=gen)
        if count:
            layer.count_gain.fill_(2.0)
    return pred.to(DEV)


@pytest.mark.parametrize('rank,count', [(8, True), (0, True), (8, False)])
def test_student_scores_with_the_optional_terms(rank, count):
    """The lists the student builds are those of the layer's logits with
    the terms' inputs pooled from the same tiles."""
    heads, seq_len, text, grid = 4, 1100, 130, (4, 12, 20)
    used = text + grid[0] * grid[1] * grid[2]
    q, k, v = (x.to(DEV) for x in inputs.qkv(seq_len, heads, 128, 83,
                                             torch.bfloat16))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=0.4))
    clip = veda_attention.ClipTiling(veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),)), config, DEV)
    plan = veda_plan.TilePlan('terms', grid, [tiling.TileShape(2, 8, 8)],
                              [[0] * heads])
    pred = _predictor(heads, rank, count)
    student = veda_attention.SparseStudent(clip, plan, pred)
    out = student(q, k, v, 0)
    lay = clip.get(tiling.TileShape(2, 8, 8))
    all_heads = torch.arange(heads, device=DEV)
    _, fq, sq, _ = tiling.gather_and_pool(q, lay, all_heads, second=True)
    _, fk, _, var = tiling.gather_and_pool(k, lay, all_heads, second=True)
    extra = {}
    if count:
        extra['log_count'] = veda_predictor.log_tile_counts(lay)
    if rank:
        extra.update(sq_q=sq, var_k=var)
    with torch.no_grad():
        logits = pred.layers[0](fq, fk, all_heads, **extra)
    want = veda_mask.select_block_lists(logits[:, :lay.n_video_tiles], lay,
                                        clip.blocks(lay))
    got = student.last_lists
    torch.cuda.synchronize()
    for name in ('part_cnt', 'full_cnt'):
        assert torch.equal(getattr(got, name), getattr(want, name)), name
    for cnt, name in (('part_cnt', 'part_idx'), ('full_cnt', 'full_idx')):
        c = getattr(want, cnt)
        n = getattr(want, name).shape[-1]
        live = torch.arange(n, device=DEV) < c[..., None]
        assert torch.equal(getattr(got, name)[live],
                           getattr(want, name)[live]), name
    assert torch.isfinite(out[:used].float()).all()


def test_teacher_trains_the_optional_terms():
    heads, seq_len, text, grid = 4, 1100, 130, (4, 12, 20)
    used = text + grid[0] * grid[1] * grid[2]
    q, k, v = (x.to(DEV) for x in inputs.qkv(seq_len, heads, 128, 84,
                                             torch.bfloat16))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=0.4), heat_reduce='sum')
    clip = veda_attention.ClipTiling(veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),)), config, DEV)
    plan = veda_plan.TilePlan('terms', grid, [tiling.TileShape(2, 8, 8)],
                              [[0] * heads])
    pred = _predictor(heads, 8, True)
    teacher = veda_attention.TeacherCollector(
        clip, plan, pred, torch.Generator().manual_seed(5), 1.0)
    teacher(q, k, v, 0)
    torch.cuda.synchronize()
    layer = pred.layers[0]
    for name in ('proj_q', 'proj_k', 'so_q', 'so_k', 'count_gain'):
        grad = getattr(layer, name).grad
        assert grad is not None and torch.isfinite(grad).all(), name
        assert grad.abs().sum() > 0, name
