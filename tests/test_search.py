"""Tile search on CPU: the oracle's restatements of the oracle relative
error against the reference's own fp32 `oracle_rel_mse_reference`, and the
plan vote and score files against the reference's `build_plan`
(fixtures from tests/golden/make_search.py)."""

import json
import os

import numpy as np
import pytest
import torch

import inputs
from miowtion_b200 import search
from miowtion_b200 import tiling
from oracle import veda_oracle as vo

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden')


def _case(ci):
    spec = inputs.SEARCH
    lay = vo.build_tile_layout(
        [vo.Span(spec['text'], spec['grid'], spec['candidates'][ci])],
        spec['used'], spec['seq_len'])
    blocks = vo.column_blocks(lay, vo.Budget(ratio=spec['ratio']))
    rows = inputs.search_rows(lay.n_video_tiles, spec['query_tiles'],
                              spec['sample_seed']).numpy()
    return lay, blocks, rows


@pytest.fixture(scope='module')
def qkv():
    spec = inputs.SEARCH
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.bfloat16)
    return tuple(t.float().numpy() for t in (q, k, v))


@pytest.mark.parametrize('ci', range(len(inputs.SEARCH['candidates'])))
def test_oracle_rel_mse_matches_reference(qkv, ci):
    g = np.load(os.path.join(GOLDEN, 'search.npz'))
    lay, blocks, rows = _case(ci)
    np.testing.assert_array_equal(lay.perm, g[f'c{ci}_perm'])
    np.testing.assert_array_equal(rows, g[f'c{ci}_rows'])
    want = g[f'c{ci}_rel_mse']
    # The token-level restatement: fp32 sums in another order only.
    got = vo.oracle_rel_mse_reference(*qkv, lay, blocks, rows)
    np.testing.assert_allclose(got, want, rtol=1e-4)
    # The kernel path's restatement (heat-based selection, bf16 outputs).
    spec = inputs.SEARCH
    out, lse = vo.dense_attention(*qkv, spec['used'], return_lse=True)
    got = vo.oracle_rel_mse(*qkv, lay, blocks, rows, out, lse)
    np.testing.assert_allclose(got, want, rtol=1e-2)


def _entries():
    spec = inputs.SEARCH
    out = []
    for e, per_layer in enumerate(inputs.vote_tables(spec)):
        for layer, table in enumerate(per_layer):
            out.append(search.ScoreEntry(f'clip{e % 2}', 10 * e, layer,
                                         table))
    return out


def test_build_plan_matches_reference():
    spec = inputs.SEARCH
    with open(os.path.join(GOLDEN, 'search_plan.json')) as f:
        want = json.load(f)
    cands = [tiling.TileShape.parse(s) for s in spec['vote_candidates']]
    for key, plan_json in want.items():
        max_padding, max_shapes = key.split('_')
        kwargs = dict(max_padding=float(max_padding),
                      max_shapes_per_layer=int(max_shapes),
                      meta={'keep_ratio': 0.1})
        if 'error' in plan_json:
            with pytest.raises(ValueError):
                search.build_plan('16x9_t37', spec['vote_grid'], cands,
                                  _entries(), spec['vote_layers'], **kwargs)
            continue
        plan = search.build_plan('16x9_t37', spec['vote_grid'], cands,
                                 _entries(), spec['vote_layers'], **kwargs)
        assert plan.to_json() == plan_json


def test_score_files_round_trip(tmp_path):
    spec = inputs.SEARCH
    cands = [tiling.TileShape.parse(s) for s in spec['vote_candidates']]
    entries = _entries()
    path = str(tmp_path / 'scores.json')
    search.save_entries(path, entries, cands, {'seed': 0})
    got_cands, got, meta = search.load_entries([path])
    assert got_cands == cands and meta == {'seed': 0}
    assert len(got) == len(entries)
    for a, b in zip(got, entries):
        assert (a.clip, a.step, a.layer) == (b.clip, b.step, b.layer)
        torch.testing.assert_close(a.table, b.table)
    os.remove(path + '.done')
    with pytest.raises(FileNotFoundError):
        search.load_entries([path])
    other = str(tmp_path / 'other.json')
    search.save_entries(other, entries, cands[::-1], {})
    search.save_entries(path, entries, cands, {})
    with pytest.raises(ValueError, match='menu'):
        search.load_entries([path, other])
    with pytest.raises(ValueError, match='no scores'):
        search.build_plan('g', spec['vote_grid'], cands, entries[:1], 3)
