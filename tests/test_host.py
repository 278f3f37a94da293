"""Host-side logic of the mirror (no GPU): tile shapes, layout counts,
budgets, plans. Checked against the oracle, which is pinned to the reference.
"""

import json

import numpy as np
import pytest
import torch

import inputs
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import tiling
from oracle import veda_oracle as vo

_GRID = (37, 24, 42)


def test_shape_menu_and_padding():
    # tests/unit/test_veda_tiling_plan.py:13-21 of the reference
    assert len(tiling.all_shapes()) == 36
    assert tiling.TileShape(1, 8, 16).num_tiles(_GRID) == 333
    assert tiling.TileShape(8, 4, 4).num_tiles(_GRID) == 330
    assert tiling.TileShape(8, 4, 4).padded_grid(_GRID) == (40, 24, 44)
    assert tiling.least_padding_shape((1, 64, 112)).t == 1
    with pytest.raises(ValueError):
        tiling.TileShape(2, 2, 2)
    assert tiling.least_padding_shape((4, 45, 80)) == tiling.TileShape(4, 2, 16)


def spans_of(spec):
    return [tiling.TiledSpan(s, tuple(g), tiling.TileShape(*sh))
            for s, g, sh in spec['spans']]


@pytest.mark.parametrize('name', sorted({**inputs.SMALL_LAYOUTS,
                                         **inputs.BENCH_LAYOUTS}))
def test_layout_counts_match_oracle(name):
    spec = {**inputs.SMALL_LAYOUTS, **inputs.BENCH_LAYOUTS}[name]
    lay = vo.build_tile_layout(
        [vo.Span(s, tuple(g), tuple(sh)) for s, g, sh in spec['spans']],
        spec['used'], spec['seq_len'])
    assert tiling.layout_counts(spans_of(spec), spec['used']) == (
        lay.n_video_tiles, lay.n_ref_tiles, lay.n_global_tiles)


def test_layout_rejects_bad_spans_and_cpu():
    span = tiling.TiledSpan(10, (2, 8, 8), tiling.TileShape(2, 8, 8))
    with pytest.raises(ValueError):
        tiling.layout_counts([span], 100)
    with pytest.raises(ValueError):
        tiling.layout_counts([], 100)
    with pytest.raises(RuntimeError, match='CUDA'):
        tiling.build_tile_layout([span], 200, 200, 'cpu')


@pytest.mark.parametrize('budget', [1.0, 2.3, 3.75, 5.5, 68.695384615385,
                                    0.5, 100.0])
def test_split_budget_and_bresenham_match_oracle(budget):
    assert veda_mask.split_budget(budget, 64) == vo.split_budget(budget, 64)
    frac = veda_mask.split_budget(budget, 64)[2]
    np.testing.assert_array_equal(
        veda_mask.bresenham_extra(400, frac, 'cpu').numpy(),
        vo.bresenham_extra(400, frac))


def test_budget_rules():
    budget = veda_mask.Budget(ratio=0.1)
    assert budget.per_row(37296, 330) == pytest.approx(0.1 * 292**2 / 330)
    assert veda_mask.Budget(tiles=7).per_row(37296, 330) == 7.0
    assert veda_mask.Budget(ratio=1.0).keeps_all
    with pytest.raises(ValueError):
        veda_mask.Budget()
    with pytest.raises(ValueError):
        veda_mask.Budget(ratio=-1)


def test_resolved_blocks_carry_the_reference_budget():
    class Lay:
        n_ref_tiles, n_video_tiles = 120, 900
        ref_tokens, target_tokens = 14400, 93600
    blocks = veda_mask.column_blocks(Lay, veda_mask.Budget(ratio=0.1),
                                     veda_mask.Budget(ratio=0.05))
    arr = veda_mask.resolve_blocks(blocks)
    # cfg4 facts: ref per_row 5.3204, target 68.695
    assert (arr[0].start, arr[0].stop, arr[0].k_lo, arr[0].k_hi) == (
        0, 120, 5, 6)
    assert arr[0].frac == round(0.05 * 113**2 / 120 - 5, 12)
    assert (arr[1].k_lo, arr[1].k_hi) == (68, 69)
    assert arr[1].frac == round(0.1 * 732**2 / 780 - 68, 12)
    with pytest.raises(ValueError):
        veda_mask.column_blocks(Lay, veda_mask.Budget(ratio=0.1))


def test_plan_groups_and_json(tmp_path):
    shapes = [tiling.TileShape(4, 8, 4), tiling.TileShape(8, 8, 2),
              tiling.TileShape(2, 8, 8)]
    with pytest.raises(ValueError):
        veda_plan.TilePlan('g', (5, 8, 8), shapes, [[0, 1, 2, 0]])
    plan = veda_plan.TilePlan('g', (5, 8, 8), shapes,
                              [[0, 1, 1, 0], [2, 2, 2, 2]])
    groups = plan.head_groups(0, 'cpu')
    assert [g.heads.tolist() for g in groups] == [[0, 3], [1, 2]]
    path = tmp_path / 'p.json'
    plan.save(str(path))
    again = veda_plan.TilePlan.load(str(path))
    assert again.to_json() == plan.to_json()
    assert json.loads(path.read_text())['shapes'] == ['4x8x4', '8x8x2',
                                                      '2x8x8']


def test_fma_exp2_polynomial_error_bound():
    """The cubic the attention and heat kernels evaluate on the FMA pipes
    (exp2_poly2 of csrc/exp2_poly.cuh) stays within 1e-4 relative error of
    2^x over the softmax's argument range, emulated in float32 exactly as the
    kernel computes it."""
    import os
    import re
    import sys
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    csrc = os.path.join(here, 'miowtion_b200', 'csrc')
    sys.path.insert(0, csrc)
    import fit_exp2_poly
    src = open(os.path.join(csrc, 'exp2_poly.cuh')).read()
    body = src[src.index('float2 exp2_poly2'):]
    lits = re.findall(r'(0x1\.[0-9a-f]+p-?\d+)f', body)[:8:2]
    c3, c2, c1, c0 = (float.fromhex(x) for x in lits)
    coef = np.array([c0, c1, c2, c3])
    np.testing.assert_allclose(coef, fit_exp2_poly.remez(), rtol=1e-6)
    # The emulation clamps where the kernel does, so the bound below is the
    # kernel's own.
    clamps = {float(c) for c in re.findall(r'fmaxf\(x\.[xy], (-[0-9.]+)f\)',
                                           body)}
    assert clamps == {fit_exp2_poly.CLAMP}
    x = np.linspace(-130.0, 8.0, 1 << 21).astype(np.float32)
    x = x[x >= fit_exp2_poly.CLAMP + 0.5]
    got = fit_exp2_poly.exp2_emulated(x, coef).astype(np.float64)
    rel = np.abs(got / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() < 1e-4


def test_balanced_order_deals_every_item_once_and_evens_the_load():
    """kernels.balanced_order (the forward's work order) on the host: every
    (head, query tile) once, the dense global rows on distinct CTAs first,
    and no CTA more than one item's weight above the mean (the greedy
    least-loaded bound)."""
    from miowtion_b200 import kernels
    heads, n_tiles, n_video, ctas = 6, 788, 780, 148
    gw, vw = 788.0, 76.7
    order = kernels.balanced_order(heads, n_tiles, n_video, gw, vw, ctas)
    assert order.shape[1] == ctas and order.dtype == torch.int32
    items = order[order >= 0]
    assert sorted(items.tolist()) == list(range(heads * n_tiles))
    first = order[0]
    assert int(((first % n_tiles) >= n_video).sum()) == min(
        ctas, heads * (n_tiles - n_video))
    weight = torch.where((order % n_tiles) >= n_video, gw, vw)
    load = torch.where(order >= 0, weight, 0.0).sum(0)
    assert float(load.max()) <= float(load.mean()) + gw
    # Against striding the default order over the CTAs, the spread shrinks.
    stride = torch.zeros(ctas)
    for i in range(heads * n_tiles):
        qt = n_tiles - 1 - i % n_tiles
        stride[i % ctas] += gw if qt >= n_video else vw
    assert float(load.max()) < float(stride.max())


def test_bench_roofline_peak_follows_timed_region():
    """A timed region of a second or more is compared with the sustained
    bf16 peak (it runs under the power cap), a shorter one with the burst
    peak; both fractions are reported either way."""
    import importlib.util
    import pathlib
    path = pathlib.Path(__file__).resolve().parents[1] / 'bench.py'
    spec = importlib.util.spec_from_file_location('bench_under_test', path)
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    peaks = {'bf16_tflops': 1600.0, 'bf16_tflops_sustained': 1400.0,
             'source': 'measured'}
    short = bench.tensor_roofline(peaks, 800.0, 0.5, 'k', None)
    assert short['peak'] == 1600.0 and short['frac'] == 0.5
    assert 'burst' in short['peak_source']
    long = bench.tensor_roofline(peaks, 700.0, 12.0, 'k', 1e9)
    assert long['peak'] == 1400.0 and long['frac'] == 0.5
    assert 'sustained' in long['peak_source'] and long['traffic'] == 1e9
    assert long['frac_of_burst'] == 700.0 / 1600.0
    assert long['frac_of_sustained'] == 0.5
