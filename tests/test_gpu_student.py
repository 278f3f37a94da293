"""The whole sparse layer (SparseStudent) against the oracle's restatement of
the reference's SparseStudent (veda/attention.py:724-794)."""

import numpy as np
import pytest
import torch

import inputs
import parity
from miowtion_b200 import attention as veda_attention
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import predictor as veda_predictor
from miowtion_b200 import tiling
from oracle import veda_oracle as vo

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def make_student(seq_len, used, spans, shapes, head_shape, budget, weights):
    layout = veda_attention.PackedLayout(seq_len, used, tuple(
        veda_attention.VideoSpan(s, g) for s, g in spans))
    config = veda_attention.VedaConfig(target_budget=budget)
    clip = veda_attention.ClipTiling(layout, config, torch.device(DEV))
    plan = veda_plan.TilePlan('test', spans[-1][1], shapes, [head_shape])
    pred = veda_predictor.TileScorePredictor(1, len(head_shape), 128)
    with torch.no_grad():
        pred.layers[0].proj_q.copy_(weights[0])
        pred.layers[0].proj_k.copy_(weights[1])
    return veda_attention.SparseStudent(clip, plan, pred.to(DEV)), clip, plan


def oracle_groups(clip, plan, spans_np):
    groups = []
    for g in plan.head_groups(0, 'cpu'):
        lay = vo.build_tile_layout(
            [vo.Span(s, tuple(grid), (g.shape.t, g.shape.h, g.shape.w))
             for s, grid in spans_np], clip.layout.used, clip.layout.seq_len)
        groups.append((lay, g.heads.numpy()))
    return groups


def run_case(seq_len, used, spans, shapes, head_shape, ratio, seed):
    heads = len(head_shape)
    q, k, v = inputs.qkv(seq_len, heads, 128, seed, torch.bfloat16)
    w = inputs.predictor_weights(heads, 128, seed + 100, 0.02)
    student, clip, plan = make_student(
        seq_len, used, spans, shapes, head_shape,
        veda_mask.Budget(ratio=ratio), w)
    out = student(q.to(DEV), k.to(DEV), v.to(DEV), 0)
    torch.cuda.synchronize()
    want, info = vo.sparse_student_layer(
        q.float().numpy(), k.float().numpy(), v.float().numpy(),
        oracle_groups(clip, plan, spans), w[0].numpy(), w[1].numpy(),
        vo.Budget(ratio=ratio), used=used)
    return out.float().cpu().numpy(), want, info, student, clip, plan, (q, k,
                                                                       v)


def test_cfg1_layer_matches_oracle():
    spec = inputs.CFG1
    got, want, info, student, clip, plan, _ = run_case(
        spec['seq_len'], spec['used'], [(0, spec['grid'])],
        [tiling.TileShape(*spec['shape'])], [0] * spec['heads'],
        spec['ratio'], spec['seed'])
    assert (info[0]['mask'].sum(-1) == 4).all()
    np.testing.assert_allclose(got, want, rtol=2e-2, atol=2e-2)
    parity.assert_rel(got, want, parity.FWD, 'SparseStudent layer, cfg1')
    assert student.calls == {'sparse': 1, 'dense': 0}


def test_two_shapes_text_rows_and_padding_match_oracle():
    """Two head groups, a padded grid (partial tiles), global text rows and
    padding rows [used, seq_len)."""
    text, grid = 300, (8, 12, 20)
    used = text + grid[0] * grid[1] * grid[2]
    got, want, info, student, clip, plan, (q, k, v) = run_case(
        used + 40, used, [(text, grid)],
        [tiling.TileShape(2, 8, 8), tiling.TileShape(1, 8, 16)],
        [0, 1, 0, 1], 0.3, 9)
    assert (got[used:] == 0).all()
    # Logit near-ties could flip a selection between fp32 orderings; the
    # inputs here have none, so the masks agree exactly and so do outputs.
    for g, (grp, (lay, heads)) in zip(plan.head_groups(0, DEV),
                                      zip(info, oracle_groups(clip, plan,
                                                              [(text, grid)]))):
        tl = clip.get(g.shape)
        qt, fq = tiling.gather_and_pool(q.to(DEV), tl, g.heads)
        kt, fk = tiling.gather_and_pool(k.to(DEV), tl, g.heads)
        logits = student.predictor.layers[0](fq, fk, g.heads)
        np.testing.assert_allclose(logits.detach().cpu().numpy(),
                                   grp['logits'],
                                   rtol=1e-4, atol=1e-5)
        lists = veda_mask.select_block_lists(
            logits[:, :tl.n_video_tiles], tl, clip.blocks(tl),
            want_mask=True)
        np.testing.assert_array_equal(lists.mask.cpu().numpy().astype(bool),
                                      grp['mask'])
    np.testing.assert_allclose(got[:used], want[:used], rtol=2e-2,
                               atol=2e-2)
    parity.assert_rel(got[:used], want[:used], parity.FWD,
                      'SparseStudent layer, two shapes with text rows')


def test_student_backward_matches_oracle():
    """Gradients of the whole layer (two head groups, partial tiles, text
    rows, padding rows) against the oracle: per group, the tile-level
    backward of the reference's attention on the oracle's own selection,
    mapped back through the permutation. Tolerance: the reference's
    backward test elementwise (3e-2) and a normalized error of at most
    2e-2."""
    text, grid = 300, (8, 12, 20)
    used = text + grid[0] * grid[1] * grid[2]
    seq_len = used + 40
    spans = [(text, grid)]
    head_shape = [0, 1, 0, 1]
    ratio, seed = 0.3, 9
    q, k, v = inputs.qkv(seq_len, len(head_shape), 128, seed, torch.bfloat16)
    w = inputs.predictor_weights(len(head_shape), 128, seed + 100, 0.02)
    student, clip, plan = make_student(
        seq_len, used, spans,
        [tiling.TileShape(2, 8, 8), tiling.TileShape(1, 8, 16)], head_shape,
        veda_mask.Budget(ratio=ratio), w)
    gen = torch.Generator().manual_seed(4)
    dout = torch.randn(q.shape, generator=gen).to(torch.bfloat16)
    ts = [t.to(DEV).requires_grad_(True) for t in (q, k, v)]
    out = student(*ts, 0)
    out.backward(dout.to(DEV))
    got = [t.grad.float().cpu().numpy() for t in ts]

    qf, kf, vf, df = (t.float().numpy() for t in (q, k, v, dout))
    _, info = vo.sparse_student_layer(
        qf, kf, vf, oracle_groups(clip, plan, spans), w[0].numpy(),
        w[1].numpy(), vo.Budget(ratio=ratio), used=used)
    want = [np.zeros((seq_len + 1,) + q.shape[1:], np.float32)
            for _ in range(3)]
    for (lay, heads), inf in zip(oracle_groups(clip, plan, spans), info):
        tiles = [vo.gather_tiles(x, lay, heads) for x in (qf, kf, vf, df)]
        grads = vo.block_sparse_attention_bwd(*tiles, inf['mask'],
                                              lay.valid_count)
        for buf, g in zip(want, grads):
            vo.scatter_tiles(buf, g, lay, heads)
    for name, g, wnt in zip('qkv', got, want):
        np.testing.assert_allclose(g[:used], wnt[:used], rtol=3e-2, atol=3e-2,
                                   err_msg=f'd{name}')
        parity.assert_rel(g[:used], wnt[:used], parity.GRAD,
                          f'SparseStudent layer backward d{name}')
        assert (g[used:] == 0).all()
        assert not (g[:used] == 0).all()


@pytest.mark.parametrize('target', ['max', 'mass', 'mean'])
def test_oracle_student_matches_oracle(target):
    """OracleStudent (attention.py:474-588): blocks chosen by the true block
    statistic of the dense teacher, then the sparse kernel. The oracle
    follows the same steps (heat of every video query tile, the training
    selection rules, block-sparse attention, scatter); the heat's sum mode
    is the unrounded one the fused pass computes."""
    from miowtion_b200 import attention as veda_attention
    from miowtion_b200 import mask as veda_mask
    from miowtion_b200 import plan as veda_plan
    spec = dict(inputs.PADDED, heads=3)
    (start, grid, shape), = spec['spans']
    packed = veda_attention.PackedLayout(
        spec['seq_len'], spec['used'],
        (veda_attention.VideoSpan(start, tuple(grid)),))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=spec['ratio']))
    clip = veda_attention.ClipTiling(packed, config, DEV)
    plan = veda_plan.TilePlan('o', tuple(grid), [tiling.TileShape(*shape)],
                              [[0] * spec['heads']])
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], 128, spec['seed'],
                         torch.bfloat16)
    student = veda_attention.OracleStudent(clip, plan, target)
    got = student(*(t.to(DEV) for t in (q, k, v)), 0)
    ref = vo.build_tile_layout([vo.Span(start, tuple(grid), tuple(shape))],
                               spec['used'], spec['seq_len'])
    qf, kf, vf = (t.float().numpy() for t in (q, k, v))
    _, lse = vo.dense_attention(qf, kf, vf, spec['used'], return_lse=True)
    heads = np.arange(spec['heads'])
    qt, kt, vt = (vo.gather_tiles(x, ref, heads) for x in (qf, kf, vf))
    rows = np.arange(ref.n_video_tiles)
    heat = vo.teacher_heat(qt, kt, vo.gather_lse(lse, ref, heads), ref, rows,
                           'max' if target == 'max' else 'sum',
                           round_scores=(target == 'max'))
    if target == 'mean':
        heat = heat / np.maximum(ref.valid_count, 1)[None, None, :]
    blocks = vo.column_blocks(ref, vo.Budget(ratio=spec['ratio']))
    index, keep = vo.select_video_blocks(heat, ref, blocks, rows)
    mask = vo.dense_block_mask(index, keep, ref)
    ot = vo.block_sparse_attention(qt, kt, vt, mask, ref.valid_count)
    want = np.zeros((spec['seq_len'] + 1, spec['heads'], 128), np.float32)
    vo.scatter_tiles(want, ot, ref, heads)
    used = spec['used']
    np.testing.assert_allclose(got.float().cpu().numpy()[:used], want[:used],
                               rtol=2e-2, atol=2e-2)
    parity.assert_rel(got.float().cpu().numpy()[:used], want[:used],
                      parity.FWD, 'OracleStudent layer')
    assert student.calls == {'sparse': 1, 'dense': 0}


def test_dense_attention_fn_matches_oracle():
    from miowtion_b200 import attention as veda_attention
    spec = inputs.PADDED
    q, k, v = inputs.qkv(spec['seq_len'], 2, 128, spec['seed'],
                         torch.bfloat16)
    fn = veda_attention.DenseAttention(spec['used'])
    got = fn(*(t.to(DEV) for t in (q, k, v)), 3)
    want, _ = vo.dense_attention(*(t.float().numpy() for t in (q, k, v)),
                                 spec['used'])
    np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=2e-2,
                               atol=2e-2)
    parity.assert_rel(got, want, parity.FWD, 'DenseAttention layer')
    with pytest.raises(ValueError):
        veda_attention.dense_attention(q.to(DEV), k.to(DEV), v.to(DEV),
                                       spec['used'], backend='nope')


def test_head_chunks_are_exact():
    """A group processed one head at a time (collect_bytes below one head's
    copy, attention.py:204-206) gives the same bits as one launch per group
    (heads are independent in every kernel); the reference's head-chunking
    test is tests/unit/test_veda_heatmap_attention.py:175-235."""
    text, grid = 300, (8, 12, 20)
    used = text + grid[0] * grid[1] * grid[2]
    seq_len = used + 40
    heads = 4
    q, k, v = (t.to(DEV) for t in inputs.qkv(seq_len, heads, 128, 27,
                                             torch.bfloat16))
    w = inputs.predictor_weights(heads, 128, 127, 0.02)
    outs = []
    for collect in (veda_attention.DEFAULT_COLLECT_BYTES, 1):
        layout = veda_attention.PackedLayout(
            seq_len, used, (veda_attention.VideoSpan(text, grid),))
        config = veda_attention.VedaConfig(
            target_budget=veda_mask.Budget(ratio=0.3), collect_bytes=collect)
        clip = veda_attention.ClipTiling(layout, config, torch.device(DEV))
        plan = veda_plan.TilePlan('chunks', grid,
                                  [tiling.TileShape(2, 8, 8),
                                   tiling.TileShape(1, 8, 16)], [[0, 1, 1, 0]])
        pred = veda_predictor.TileScorePredictor(1, heads, 128)
        with torch.no_grad():
            pred.layers[0].proj_q.copy_(w[0])
            pred.layers[0].proj_k.copy_(w[1])
        student = veda_attention.SparseStudent(clip, plan, pred.to(DEV))
        with torch.no_grad():
            outs.append(student(q, k, v, 0))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
