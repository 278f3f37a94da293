"""GPU parity of the teacher block heat (a13) against the CPU oracle.

The oracle restates `miowtion/veda/heatmap.py:36-99` (scores rounded to
bf16 as the reference's bf16 bmm returns them). Tolerances are the
reference's own for its fused heat kernel (tests/gpu/test_kernels_gpu.py
:44-78: rtol 3e-2, atol 1e-5 for max and 1e-4 for sum). Both sides get the
same tile-ordered dense LSE, computed by the oracle.
"""

import numpy as np
import pytest
import torch

import inputs
import parity
from miowtion_b200 import _lib
from miowtion_b200 import heatmap
from miowtion_b200 import tiling
from oracle import veda_oracle as vo

pytestmark = pytest.mark.gpu

DEV = 'cuda'


def np32(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0, 'a kernel wait timed out'


@pytest.fixture(scope='module')
def teacher():
    spec = dict(inputs.PADDED, heads=4, group_heads=[0, 2, 3])
    lay = tiling.build_tile_layout(
        [tiling.TiledSpan(s, tuple(g), tiling.TileShape(*sh))
         for s, g, sh in spec['spans']], spec['used'], spec['seq_len'], DEV)
    ref = vo.build_tile_layout(
        [vo.Span(s, tuple(g), tuple(sh)) for s, g, sh in spec['spans']],
        spec['used'], spec['seq_len'])
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], 128, spec['seed'],
                         torch.bfloat16)
    heads = spec['group_heads']
    _, lse = vo.dense_attention(np32(q), np32(k), np32(v), spec['used'],
                                return_lse=True)
    lse_t = vo.gather_lse(lse, ref, heads)
    hd = torch.tensor(heads, device=DEV)
    qt, kt = (tiling.gather_tiles(t.to(DEV), lay, hd) for t in (q, k))
    return lay, ref, qt, kt, lse_t


@pytest.mark.parametrize('reduce', ['max', 'sum'])
def test_heat_matches_oracle(teacher, reduce):
    lay, ref, qt, kt, lse_t = teacher
    q_tiles = np.arange(lay.n_tiles)
    got = heatmap.teacher_heat(qt, kt, torch.from_numpy(lse_t).to(DEV), lay,
                               torch.from_numpy(q_tiles), reduce)
    want = vo.teacher_heat(np32(qt), np32(kt), lse_t, ref, q_tiles, reduce,
                           round_scores=True)
    atol = 1e-5 if reduce == 'max' else 1e-4
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=3e-2, atol=atol)
    parity.assert_rel(got, want, 3e-2, f'teacher heat ({reduce})')
    assert (got > 0).any()


def test_heat_row_subset_and_order(teacher):
    """q_tiles may be any subset in any order (heatmap.py:48-49)."""
    lay, ref, qt, kt, lse_t = teacher
    q_tiles = np.array([lay.n_tiles - 1, 3, 0, 7])
    got = heatmap.teacher_heat(qt, kt, torch.from_numpy(lse_t).to(DEV), lay,
                               torch.from_numpy(q_tiles), 'max')
    want = vo.teacher_heat(np32(qt), np32(kt), lse_t, ref, q_tiles, 'max',
                           round_scores=True)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=3e-2, atol=1e-5)
    parity.assert_rel(got, want, 3e-2, 'teacher heat (max), query subset')


def test_heat_mass_rows_sum_to_valid_rows(teacher):
    """With the true dense LSE every valid query row's probabilities over
    all keys sum to 1, so a query tile's masses sum to its valid rows."""
    lay, _, qt, kt, lse_t = teacher
    got = heatmap.teacher_heat(qt, kt, torch.from_numpy(lse_t).to(DEV), lay,
                               torch.arange(lay.n_tiles), 'sum')
    rows = got.sum(-1).cpu().numpy()  # [H', n]
    want = np.broadcast_to(lay.valid_count.cpu().numpy().astype(np.float64),
                           rows.shape)
    np.testing.assert_allclose(rows, want, rtol=2e-2, atol=1e-3)


def test_heat_rejects_bad_reduce(teacher):
    lay, _, qt, kt, lse_t = teacher
    with pytest.raises(ValueError):
        heatmap.teacher_heat(qt, kt, torch.from_numpy(lse_t).to(DEV), lay,
                             torch.arange(2), 'mean')


@pytest.fixture(scope='module')
def fused_case():
    """The padded layout with v too, and the oracle's dense teacher in tile
    order."""
    spec = dict(inputs.PADDED, heads=4, group_heads=[0, 2, 3])
    lay = tiling.build_tile_layout(
        [tiling.TiledSpan(s, tuple(g), tiling.TileShape(*sh))
         for s, g, sh in spec['spans']], spec['used'], spec['seq_len'], DEV)
    ref = vo.build_tile_layout(
        [vo.Span(s, tuple(g), tuple(sh)) for s, g, sh in spec['spans']],
        spec['used'], spec['seq_len'])
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], 128, spec['seed'],
                         torch.bfloat16)
    heads = spec['group_heads']
    out, lse = vo.dense_attention(np32(q), np32(k), np32(v), spec['used'],
                                  return_lse=True)
    hd = torch.tensor(heads, device=DEV)
    qt, kt, vt = (tiling.gather_tiles(t.to(DEV), lay, hd) for t in (q, k, v))
    out_t = vo.gather_tiles(out, ref, heads)
    lse_t = vo.gather_lse(lse, ref, heads)
    return lay, ref, qt, kt, vt, out_t, lse_t


@pytest.mark.parametrize('reduce', ['max', 'sum'])
def test_fused_dense_heat_matches_oracle(fused_case, reduce):
    """One pass gives the dense teacher (out, LSE) and the heat. The max
    mode follows the reference's bf16 score rounding exactly (it rounds the
    row maximum); the sum mode uses the fp32 scores of the softmax, so it
    is compared with the unrounded oracle."""
    lay, ref, qt, kt, vt, out_t, lse_t = fused_case
    out, lse, heat = heatmap.fused_dense_heat(qt, kt, vt, lay, reduce)
    valid = ref.slot_valid.astype(bool)
    np.testing.assert_allclose(np32(out)[valid], out_t[valid], rtol=2e-2,
                               atol=2e-2)
    parity.assert_rel(np32(out), out_t, parity.FWD,
                      f'fused dense + heat ({reduce}): output', where=valid)
    np.testing.assert_allclose(np32(lse).T[valid], lse_t[valid], atol=2e-3)
    want = vo.teacher_heat(np32(qt), np32(kt), lse_t, ref,
                           np.arange(lay.n_tiles), reduce,
                           round_scores=(reduce == 'max'))
    atol = 1e-5 if reduce == 'max' else 1e-4
    np.testing.assert_allclose(heat.cpu().numpy(), want, rtol=3e-2,
                               atol=atol)
    parity.assert_rel(heat, want, 3e-2, f'fused dense + heat ({reduce}): heat')
    # The separate heat kernel on the fused pass's own LSE agrees closely.
    sep = heatmap.teacher_heat(qt, kt, lse.T.contiguous(), lay,
                               torch.arange(lay.n_tiles), reduce)
    if reduce == 'max':
        torch.testing.assert_close(heat, sep, rtol=1e-3, atol=1e-6)
    else:
        torch.testing.assert_close(heat, sep, rtol=3e-2, atol=1e-4)


@pytest.mark.parametrize('reduce', ['max', 'sum'])
def test_fused_pass_pairs_equal_single_tiles(fused_case, reduce):
    """With two softmax groups the fused pass runs query tiles in pairs that
    share every key and value tile (one group per tile); with one group each
    tile runs alone. Same output, LSE and heat up to fp32 summation order;
    the padded layout has an odd number of tiles, so the last pair has one."""
    from miowtion_b200 import kernels
    lay, ref, qt, kt, vt, _, _ = fused_case
    assert lay.n_tiles % 2 == 1
    runs = {}
    try:
        for g in (1, 2):
            kernels.set_fwd_groups(g)
            runs[g] = heatmap.fused_dense_heat(qt, kt, vt, lay, reduce)
    finally:
        kernels.set_fwd_groups(kernels.DEFAULT_FWD_GROUPS)
    valid = ref.slot_valid.astype(bool)
    (o1, l1, h1), (o2, l2, h2) = runs[1], runs[2]
    parity.assert_rel(np32(o2), np32(o1), 1e-2,
                      f'fused pass ({reduce}): pairs against single tiles',
                      where=valid)
    np.testing.assert_allclose(np32(l2).T[valid], np32(l1).T[valid],
                               atol=1e-3)
    parity.assert_rel(h2, h1, 1e-2,
                      f'fused pass ({reduce}): heat, pairs against single '
                      'tiles')
