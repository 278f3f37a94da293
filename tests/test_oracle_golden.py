"""Pins the CPU oracle (oracle/veda_oracle.py) to the reference's own outputs.

The golden vectors were produced by importing the reference implementation
(tests/golden/make_golden.py). Integer and index outputs must match exactly;
floating-point outputs within the reference's own tolerances.
"""

import hashlib
import os

import numpy as np
import pytest
import torch

import inputs
from oracle import veda_oracle as vo

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden')


def load(name):
    return np.load(os.path.join(GOLDEN, f'{name}.npz'))


def digest(t):
    return hashlib.sha256(t.contiguous().view(-1).float().numpy()
                          .tobytes()).hexdigest()


def layout(spec):
    spans = [vo.Span(s, tuple(g), tuple(sh)) for s, g, sh in spec['spans']]
    return vo.build_tile_layout(spans, spec['used'], spec['seq_len'])


def check_layout(g, lay, prefix=''):
    np.testing.assert_array_equal(lay.perm, g[f'{prefix}perm'])
    np.testing.assert_array_equal(lay.valid_count, g[f'{prefix}valid_count'])
    np.testing.assert_array_equal(
        [lay.n_video_tiles, lay.n_ref_tiles, lay.n_global_tiles,
         lay.ref_tokens, lay.target_tokens, lay.used, lay.seq_len],
        g[f'{prefix}scalars'])


def check_lists(g, mask, lay, prefix):
    for transpose, tag in ((False, 'lists'), (True, 'tlists')):
        got = vo.index_lists(mask, lay, transpose=transpose)
        for name, arr in zip(('part_cnt', 'part_idx', 'full_cnt',
                              'full_idx'), got):
            np.testing.assert_array_equal(arr, g[f'{tag}_{name}'],
                                          err_msg=f'{prefix}{tag}_{name}')


@pytest.mark.parametrize('name', sorted(inputs.SMALL_LAYOUTS))
def test_small_layouts_match_reference(name):
    g = load('layouts')
    check_layout(g, layout(inputs.SMALL_LAYOUTS[name]), f'{name}_')


@pytest.mark.parametrize('name', sorted(inputs.BENCH_LAYOUTS))
def test_bench_layouts_and_budgets_match_reference(name):
    g = load('layouts')
    spec = inputs.BENCH_LAYOUTS[name]
    lay = layout(spec)
    assert hashlib.sha256(lay.perm.tobytes()).hexdigest() == str(
        g[f'{name}_perm_sha256'])
    np.testing.assert_array_equal(lay.valid_count, g[f'{name}_valid_count'])
    np.testing.assert_array_equal(
        [lay.n_video_tiles, lay.n_ref_tiles, lay.n_global_tiles,
         lay.ref_tokens, lay.target_tokens, lay.used, lay.seq_len],
        g[f'{name}_scalars'])


def test_budget_facts_match_reference():
    g = load('layouts')
    facts = []
    for spec in inputs.BENCH_LAYOUTS.values():
        lay = layout(spec)
        for ref_ratio, target_ratio in spec['budgets']:
            blocks = vo.column_blocks(
                lay, vo.Budget(ratio=target_ratio),
                None if ref_ratio is None else vo.Budget(ratio=ref_ratio))
            for b in blocks:
                per_row = b.budget.per_row(b.real_tokens, b.stop - b.start)
                k_lo, k_hi, frac = vo.split_budget(per_row, b.stop - b.start)
                extra = vo.bresenham_extra(lay.n_video_tiles, frac)
                facts.append([b.start, b.stop, b.real_tokens, per_row, k_lo,
                              k_hi, frac, int(extra.sum())])
    np.testing.assert_array_equal(np.array(facts), g['budget_facts'])
    kat = []
    for budget in g['split_kat'][:, 0]:
        k_lo, k_hi, frac = vo.split_budget(float(budget), 64)
        extra = vo.bresenham_extra(400, frac)
        kat.append([budget, k_lo, k_hi, frac, int(extra.sum()),
                    int((extra[:7].astype(np.int64) * 2**np.arange(7)).sum())])
    np.testing.assert_array_equal(np.array(kat), g['split_kat'])
    assert vo.Budget(ratio=0.1).per_row(37296, 330) == g['equal_cost'][0]


def test_segmented_selection_matches_reference():
    g = load('segmented')
    spec = inputs.SEGMENTED
    lay = layout(spec)
    check_layout(g, lay)
    scores_t = inputs.scores(spec['heads'], lay.n_tiles, spec['score_seed'])
    assert digest(scores_t) == str(g['s_digest'])
    scores = scores_t.numpy()
    blocks = vo.column_blocks(lay, vo.Budget(ratio=spec['target_ratio']),
                              vo.Budget(ratio=spec['ref_ratio']))
    index, keep = vo.select_video_blocks(scores[:, :lay.n_video_tiles], lay,
                                         blocks)
    np.testing.assert_array_equal(index, g['sel_index'])
    np.testing.assert_array_equal(keep, g['sel_keep'])
    mask = vo.dense_block_mask(index, keep, lay)
    np.testing.assert_array_equal(mask, g['mask'])
    rows = np.array(spec['subset_rows'])
    sub_index, sub_keep = vo.select_video_blocks(scores[:, rows], lay,
                                                 blocks, rows)
    np.testing.assert_array_equal(sub_index, g['sub_index'])
    np.testing.assert_array_equal(sub_keep, g['sub_keep'])
    np.testing.assert_array_equal(
        vo.dense_block_mask(sub_index, sub_keep, lay, global_rows=False),
        g['sub_mask'])
    check_lists(g, mask, lay, 'segmented ')


@pytest.fixture(scope='module')
def padded_case():
    spec = inputs.PADDED
    g = load('padded')
    lay = layout(spec)
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.bfloat16)
    assert digest(q) == str(g['q_digest'])
    heads = np.array(spec['group_heads'])
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    return spec, g, lay, heads, qn, kn, vn


def test_padded_layout_pool_and_logits_match_reference(padded_case):
    spec, g, lay, heads, q, k, _ = padded_case
    check_layout(g, lay)
    qt = vo.gather_tiles(q, lay, heads)
    kt = vo.gather_tiles(k, lay, heads)
    fq = vo.pool_tiles(qt, lay)
    d = spec['dim']
    # max/min are exact; the mean sums in another order (reference tol).
    np.testing.assert_array_equal(fq[..., d:], g['feats_q'][..., d:])
    np.testing.assert_allclose(fq[..., :d], g['feats_q'][..., :d],
                               rtol=1e-5, atol=1e-6)
    fk = vo.pool_tiles(kt, lay)
    np.testing.assert_allclose(fk, g['feats_k'], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(vo.pool_tiles(qt, lay, 'raw'), g['sq_q'],
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(vo.pool_tiles(kt, lay, 'central'),
                               g['var_k'], rtol=1e-4, atol=1e-6)
    proj_q, proj_k = inputs.predictor_weights(spec['heads'], d,
                                              spec['pred_seed'], 0.02)
    logits = vo.predictor_logits(fq, fk, proj_q.numpy(), proj_k.numpy(),
                                 heads)
    np.testing.assert_allclose(logits, g['logits'], rtol=1e-4, atol=1e-5)


def test_padded_selection_lists_match_reference(padded_case):
    spec, g, lay, heads, *_ = padded_case
    scores_t = inputs.scores(len(heads), lay.n_tiles, spec['score_seed'])
    assert digest(scores_t) == str(g['s_digest'])
    blocks = vo.column_blocks(lay, vo.Budget(ratio=spec['ratio']))
    index, keep = vo.select_video_blocks(
        scores_t.numpy()[:, :lay.n_video_tiles], lay, blocks)
    np.testing.assert_array_equal(index, g['sel_index'])
    np.testing.assert_array_equal(keep, g['sel_keep'])
    mask = vo.dense_block_mask(index, keep, lay)
    np.testing.assert_array_equal(mask, g['mask'])
    check_lists(g, mask, lay, 'padded ')


def test_padded_attention_fwd_bwd_match_reference(padded_case):
    spec, g, lay, heads, q, k, v = padded_case
    qt, kt, vt = (vo.gather_tiles(t, lay, heads) for t in (q, k, v))
    mask = g['mask']
    out, lse = vo.block_sparse_attention(qt, kt, vt, mask, lay.valid_count,
                                         return_lse=True)
    real = lay.slot_valid.astype(bool)
    sub = np.zeros_like(real)
    sub[::4] = True
    # The reference casts its fp32 output to bf16.
    got = vo.round_bf16(out)[::4][real[::4]]
    want = g['attn_out'].astype(np.float32)[real[::4]]
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(lse[:, real], g['attn_lse'][:, real],
                               rtol=1e-5, atol=1e-5)
    dout_t = inputs.dout(qt.shape, spec['dout_seed'])
    assert digest(dout_t) == str(g['d_digest'])
    dq, dk, dv = vo.block_sparse_attention_bwd(qt, kt, vt,
                                               dout_t.float().numpy(), mask,
                                               lay.valid_count)
    for name, arr in (('dq', dq), ('dk', dk), ('dv', dv)):
        np.testing.assert_allclose(
            vo.round_bf16(arr)[::4][real[::4]],
            g[name].astype(np.float32)[real[::4]], rtol=2e-2, atol=2e-2,
            err_msg=name)


def test_padded_dense_heat_scatter_match_reference(padded_case):
    spec, g, lay, heads, q, k, v = padded_case
    out, lse = vo.dense_attention(q, k, v, lay.used, return_lse=True)
    np.testing.assert_allclose(vo.round_bf16(out)[::4],
                               g['dense_out'].astype(np.float32), rtol=1e-2,
                               atol=1e-2)
    np.testing.assert_allclose(lse, g['dense_lse'], rtol=1e-5, atol=1e-5)
    qt, kt = (vo.gather_tiles(t, lay, heads) for t in (q, k))
    lse_t = vo.gather_lse(g['dense_lse'], lay, heads)
    rows = np.array(spec['heat_rows'])
    for reduce in ('max', 'sum'):
        heat = vo.teacher_heat(qt, kt, lse_t, lay, rows, reduce)
        np.testing.assert_allclose(heat, g[f'heat_{reduce}'], rtol=1e-4,
                                   atol=1e-7, err_msg=reduce)
    # Scatter of the (bf16) attention output into [S+1, H, D].
    vt = vo.gather_tiles(v, lay, heads)
    attn = vo.round_bf16(vo.block_sparse_attention(
        qt, kt, vt, g['mask'], lay.valid_count))
    buf = np.zeros((lay.seq_len + 1, spec['heads'], spec['dim']),
                   dtype=np.float32)
    vo.scatter_tiles(buf, attn, lay, heads)
    np.testing.assert_allclose(buf[::4], g['scatter'].astype(np.float32),
                               rtol=1e-2, atol=1e-2)


def test_cfg1_sparse_student_layer_matches_reference():
    spec = inputs.CFG1
    g = load('cfg1')
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.float32)
    assert digest(q) == str(g['q_digest'])
    proj_q, proj_k = inputs.predictor_weights(spec['heads'], spec['dim'],
                                              spec['pred_seed'],
                                              spec['pred_std'])
    assert digest(proj_q) == str(g['p_digest'])
    lay = vo.build_tile_layout(
        [vo.Span(0, spec['grid'], spec['shape'])], spec['used'],
        spec['seq_len'])
    check_layout(g, lay)
    heads = np.arange(spec['heads'])
    out, info = vo.sparse_student_layer(
        q.numpy(), k.numpy(), v.numpy(), [(lay, heads)], proj_q.numpy(),
        proj_k.numpy(), vo.Budget(ratio=spec['ratio']))
    (grp,) = info
    np.testing.assert_allclose(grp['feats_q'], g['feats_q'], rtol=1e-5,
                               atol=1e-6)
    np.testing.assert_allclose(grp['logits'], g['logits'], rtol=1e-4,
                               atol=1e-5)
    np.testing.assert_array_equal(grp['index'], g['sel_index'])
    np.testing.assert_array_equal(grp['keep'], g['sel_keep'])
    np.testing.assert_array_equal(grp['mask'], g['mask'])
    check_lists(g, grp['mask'], lay, 'cfg1 ')
    # Budget 0.5 of 8 tiles keeps 4 per row, the diagonal among them.
    assert (grp['mask'].sum(-1) == 4).all()
    np.testing.assert_allclose(out[::8], g['out_rows'], rtol=1e-4,
                               atol=1e-5)
