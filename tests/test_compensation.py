"""Zero-order compensation on CPU: the oracle's restatement against the
reference's own torch form (tests/golden/make_compensation.py), and the
host-side argument checks of the drop-in functions."""

import os

import numpy as np
import pytest
import torch

import inputs
from miowtion_b200 import compensation
from oracle import veda_oracle as vo

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden')


def case():
    spec = inputs.COMPENSATION
    lay = vo.build_tile_layout(
        [vo.Span(s, tuple(g), tuple(sh)) for s, g, sh in spec['spans']],
        spec['used'], spec['seq_len'])
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.float32)
    heads = np.arange(spec['heads'])
    tiles = [vo.gather_tiles(t.numpy(), lay, heads) for t in (q, k, v)]
    return spec, lay, tiles


def test_oracle_compensation_matches_reference():
    spec, lay, (qt, kt, vt) = case()
    g = np.load(os.path.join(GOLDEN, 'compensation.npz'))
    scores = inputs.scores(spec['heads'], lay.n_tiles,
                           spec['score_seed']).numpy()
    blocks = vo.column_blocks(lay, vo.Budget(ratio=spec['ratio']))
    index, keep = vo.select_video_blocks(scores[:, :lay.n_video_tiles], lay,
                                         blocks)
    mask = vo.dense_block_mask(index, keep, lay)
    np.testing.assert_array_equal(mask, g['mask'])
    o_kept, lse = vo.block_sparse_attention(qt, kt, vt, mask,
                                            lay.valid_count, return_lse=True)
    w = inputs.projection(spec['dim'], spec['proj_seed']).numpy()
    np.testing.assert_allclose(o_kept @ w, g['check_kept'], rtol=1e-4,
                               atol=1e-5)
    out = vo.zero_order_compensation(o_kept, lse, qt, kt, vt, mask, lay)
    np.testing.assert_allclose(out @ w, g['check_out'], rtol=1e-4, atol=1e-5)
    t = spec['full_tile']
    np.testing.assert_allclose(out[t * 128:(t + 1) * 128],
                               g['tile_out'].astype(np.float32), rtol=2e-3,
                               atol=2e-3)
    # The term does something where tiles were dropped ...
    assert np.abs(out - o_kept).max() > 1e-2
    # ... and nothing when every tile is kept.
    full = np.ones_like(mask)
    o_all, lse_all = vo.block_sparse_attention(qt, kt, vt, full,
                                               lay.valid_count,
                                               return_lse=True)
    same = vo.zero_order_compensation(o_all, lse_all, qt, kt, vt, full, lay)
    np.testing.assert_array_equal(same, o_all)


class _Layout:
    """The fields the argument checks read before touching the device."""

    def __init__(self, n_tiles):
        self.n_tiles = n_tiles
        self.valid_count = torch.full((n_tiles,), 128, dtype=torch.int32)


def test_compensate_rejects_a_mismatched_lse():
    rows, heads, dim, tiles = 256, 2, 128, 2
    zeros = torch.zeros(rows, heads, dim)
    mask = torch.ones(heads, tiles, tiles, dtype=torch.bool)
    with pytest.raises(ValueError, match='lse_kept'):
        compensation.compensate(zeros, torch.zeros(rows, heads), zeros, zeros,
                                zeros, mask, _Layout(tiles))


def test_compensate_rejects_a_query_tile_subset():
    rows, heads, dim, tiles = 256, 2, 128, 4
    zeros = torch.zeros(rows, heads, dim)
    mask = torch.ones(heads, rows // 128, tiles, dtype=torch.bool)
    with pytest.raises(ValueError, match='same id'):
        compensation.compensate(zeros, torch.zeros(heads, rows), zeros, zeros,
                                zeros, mask, _Layout(tiles))


def test_config_allows_one_compensation_arm():
    from miowtion_b200 import attention as veda_attention
    cfg = veda_attention.VedaConfig(zero_order_compensation=True,
                                    triton_compensation=True)
    layout = veda_attention.PackedLayout(
        1024, 1024, (veda_attention.VideoSpan(0, (4, 16, 16)),))
    with pytest.raises(ValueError, match='pick one'):
        veda_attention.ClipTiling(layout, cfg, torch.device('cpu'))
