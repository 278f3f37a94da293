"""The stage-1 losses on the CPU: the seer KL (the oracle's restatement and
the package's torch form) and the ablation losses (transport, gauge-fixed
KL, oracle BCE) against the reference's values and gradients
(tests/golden/make_teacher.py), plus the reference's own properties of
those losses. The collector itself runs on the GPU
(tests/test_gpu_teacher.py)."""

import math
import os
import types

import numpy as np
import pytest
import torch

import inputs
from miowtion_b200 import heatmap
from oracle import veda_oracle as vo

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden', 'teacher.npz')


@pytest.fixture(scope='module')
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize('direction', ['forward', 'reverse'])
def test_oracle_seer_kl_matches_reference(golden, direction):
    got = vo.seer_kl(golden['kl_logits'], golden['kl_heat'],
                     golden['kl_kv_ok'], direction)
    np.testing.assert_allclose(got, golden[f'kl_{direction}'], rtol=1e-5)


@pytest.mark.parametrize('direction', ['forward', 'reverse'])
def test_seer_kl_matches_reference_and_has_gradients(golden, direction):
    layout = types.SimpleNamespace(
        kv_ok=torch.from_numpy(golden['kl_kv_ok']))
    logits = torch.from_numpy(golden['kl_logits']).requires_grad_(True)
    heat = torch.from_numpy(golden['kl_heat'])
    kl = heatmap.seer_kl(logits, heat, layout, direction)
    np.testing.assert_allclose(kl.item(), golden[f'kl_{direction}'],
                               rtol=1e-5)
    kl.backward()
    assert torch.isfinite(logits.grad).all()
    # Empty key tiles take no gradient.
    assert (logits.grad[..., ~layout.kv_ok] == 0).all()


def test_seer_kl_rejects_unknown_direction(golden):
    layout = types.SimpleNamespace(kv_ok=torch.ones(4, dtype=torch.bool))
    with pytest.raises(ValueError, match='direction'):
        heatmap.seer_kl(torch.zeros(1, 1, 4), torch.ones(1, 1, 4), layout,
                        'sideways')


# --- the ablation losses ---------------------------------------------------
#
# The package's torch forms run on the CPU when the heat's own top-k set is
# passed in (`oracle=`); on the GPU the selection kernel makes it
# (tests/test_gpu_teacher.py). Here the set is the reference's own
# (`loss_oracle`), or the oracle restatement's selection for new inputs.

def _loss_layout():
    pad = inputs.PADDED
    lay = vo.build_tile_layout([vo.Span(s, g, sh)
                                for s, g, sh in pad['spans']],
                               pad['used'], pad['seq_len'])
    blocks = vo.column_blocks(lay, vo.Budget(ratio=inputs.LOSSES['ratio']))
    view = types.SimpleNamespace(kv_ok=torch.from_numpy(lay.kv_ok.copy()),
                                 n_video_tiles=lay.n_video_tiles)
    return lay, blocks, view, torch.tensor(inputs.LOSSES['rows'])


def _oracle_set(heat, lay, blocks, rows):
    idx, keep = vo.select_video_blocks(np.asarray(heat), lay, blocks,
                                       np.asarray(rows))
    chosen = np.zeros(idx.shape[:2] + (lay.n_video_tiles,), dtype=bool)
    np.put_along_axis(chosen, idx, keep, axis=2)
    return torch.from_numpy(chosen)


def _losses(view, rows, oracle):
    """name -> loss of logits, for every recorded loss."""
    out = {f'transport_{tau:g}': (
        lambda x, heat, tau=tau: heatmap.transport_loss(
            x, heat, view, None, rows, temperature=tau, oracle=oracle))
        for tau in inputs.LOSSES['temperatures']}
    out['gauge'] = lambda x, heat: heatmap.gauge_fixed_kl(x, heat, view,
                                                          rows)
    out['bce'] = lambda x, heat: heatmap.oracle_bce(x, heat, view, None,
                                                    rows, oracle=oracle)
    return out


def test_oracle_selection_reproduces_the_references_loss_set(golden):
    lay, blocks, _, rows = _loss_layout()
    got = _oracle_set(golden['loss_heat'], lay, blocks, rows)
    assert np.array_equal(got.numpy(), golden['loss_oracle'])


@pytest.mark.parametrize('name', [f'transport_{t:g}' for t in
                                  inputs.LOSSES['temperatures']]
                         + ['gauge', 'bce'])
def test_ablation_loss_and_gradient_match_reference(golden, name):
    _, _, view, rows = _loss_layout()
    oracle = torch.from_numpy(golden['loss_oracle'])
    heat = torch.from_numpy(golden['loss_heat'])
    logits = torch.from_numpy(golden['loss_logits']).requires_grad_(True)
    value = _losses(view, rows, oracle)[name](logits, heat)
    np.testing.assert_allclose(value.item(), golden[f'loss_{name}'],
                               rtol=1e-5, atol=1e-7)
    value.backward()
    want = golden[f'loss_{name}_grad']
    np.testing.assert_allclose(logits.grad.numpy(), want, rtol=0,
                               atol=1e-5 * max(1.0, np.abs(want).max()))


def _transport_case(seed):
    lay, blocks, view, rows = _loss_layout()
    gen = torch.Generator().manual_seed(seed)
    shape = (2, rows.numel(), view.kv_ok.numel())
    heat = torch.rand(*shape, generator=gen) + 0.01
    logits = torch.randn(*shape, generator=gen)
    return lay, blocks, view, rows, heat, logits


def _decision(view, rows):
    n_video = view.n_video_tiles
    own = torch.nn.functional.one_hot(rows, n_video).bool()[None]
    return view.kv_ok[None, None, :n_video] & ~own


def test_transport_loss_is_invariant_to_a_per_row_affine_map():
    """The reference's own property (tests/unit/
    test_veda_heatmap_attention.py:632-649)."""
    lay, blocks, view, rows, heat, logits = _transport_case(0)
    oracle = _oracle_set(heat, lay, blocks, rows)
    base = heatmap.transport_loss(logits, heat, view, blocks, rows,
                                  oracle=oracle).item()
    shift = torch.arange(rows.numel(), dtype=logits.dtype)[None, :, None]
    for moved in (logits + 7.0, logits * 3.0, logits * 0.01,
                  logits * 5.0 + shift * 100.0):
        got = heatmap.transport_loss(moved, heat, view, blocks, rows,
                                     oracle=oracle).item()
        assert got == pytest.approx(base, rel=1e-5, abs=1e-6)


def test_transport_loss_at_zero_temperature_is_the_retained_share():
    """tau -> 0: minus the attainable off-diagonal mass the student's own
    hard top-k keeps, and exactly -1 for the oracle's scores (the
    reference's tests/unit/test_veda_heatmap_attention.py:652-688)."""
    lay, blocks, view, rows, heat, logits = _transport_case(3)
    oracle = _oracle_set(heat, lay, blocks, rows)
    valid = _decision(view, rows)
    n_video = view.n_video_tiles
    mass = heat[:, :, :n_video].masked_fill(~valid, 0.0)
    budget = (oracle & valid).sum(-1)
    ceiling = (mass * (oracle & valid)).sum(-1)
    ranked = logits[:, :, :n_video].masked_fill(~valid, -1e4).argsort(
        -1, descending=True)
    kept = torch.zeros_like(oracle)
    for h in range(kept.shape[0]):
        for r in range(kept.shape[1]):
            kept[h, r, ranked[h, r, :int(budget[h, r])]] = True
    live = ceiling > 0
    want = -((mass * kept).sum(-1)[live] / ceiling[live]).mean().item()
    got = heatmap.transport_loss(logits, heat, view, blocks, rows,
                                 temperature=1e-4, oracle=oracle).item()
    assert got == pytest.approx(want, abs=1e-4)
    perfect = mass.masked_fill(~valid, -1e4)
    assert heatmap.transport_loss(perfect, heat, view, blocks, rows,
                                  temperature=1e-4, oracle=oracle).item() \
        == pytest.approx(-1.0, abs=1e-4)


def test_transport_loss_orders_masks_and_rejects_bad_temperature():
    lay, blocks, view, rows, heat, logits = _transport_case(4)
    oracle = _oracle_set(heat, lay, blocks, rows)
    valid = _decision(view, rows)
    n_video = view.n_video_tiles
    good = torch.zeros_like(logits)
    good[:, :, :n_video] = heat[:, :, :n_video].masked_fill(~valid, -1e4)
    losses = [heatmap.transport_loss(x, heat, view, blocks, rows,
                                     oracle=oracle).item()
              for x in (good, torch.zeros_like(logits), -good)]
    assert losses[0] < losses[1] < losses[2]
    for tau in (0.0, -1.0):
        with pytest.raises(ValueError, match='temperature must be'):
            heatmap.transport_loss(logits, heat, view, blocks, rows,
                                   temperature=tau, oracle=oracle)


def test_transport_loss_gradient_is_orthogonal_to_the_gauge():
    """Standardising removes the constant and the scale direction: the
    gradient sums to 0 over the decision columns and is orthogonal to the
    centred scores (the reference's test at :706-728)."""
    lay, blocks, view, rows, heat, logits = _transport_case(7)
    oracle = _oracle_set(heat, lay, blocks, rows)
    logits = logits.clone().requires_grad_(True)
    heatmap.transport_loss(logits, heat, view, blocks, rows,
                           oracle=oracle).backward()
    valid = _decision(view, rows)[0]
    n_video = view.n_video_tiles
    for r in range(rows.numel()):
        cols = valid[r]
        grad = logits.grad[0, r, :n_video][cols]
        x = logits.detach()[0, r, :n_video][cols]
        assert grad.sum().item() == pytest.approx(0.0, abs=1e-6)
        assert (grad * (x - x.mean())).sum().item() == pytest.approx(
            0.0, abs=1e-5)
    # Columns outside the decision (global tiles, the diagonal) get none.
    assert (logits.grad[:, :, n_video:] == 0).all()


def test_transport_loss_ignores_excluded_columns_and_massless_rows():
    lay, blocks, view, rows, heat, logits = _transport_case(5)
    view.kv_ok[1] = False
    oracle = _oracle_set(heat, lay, blocks, rows)
    base = heatmap.transport_loss(logits, heat, view, blocks, rows,
                                  oracle=oracle).item()
    moved = logits.clone()
    moved[:, :, 1] = 500.0
    assert heatmap.transport_loss(moved, heat, view, blocks, rows,
                                  oracle=oracle).item() == pytest.approx(
                                      base, rel=1e-6)
    heat = heat.clone()
    heat[:, 0] = 0.0
    assert torch.isfinite(heatmap.transport_loss(logits, heat, view, blocks,
                                                 rows, oracle=oracle))


def test_gauge_fixed_kl_is_zero_at_the_truth_and_gauge_invariant():
    """The reference's own property (:779-801)."""
    _, _, view, rows, heat, logits = _transport_case(4)
    n_video = view.n_video_tiles
    truth = heat.clone()
    truth[:, :, :n_video] = heat[:, :, :n_video].clamp(min=1e-20).log()
    assert heatmap.gauge_fixed_kl(truth, heat, view, rows).item() == \
        pytest.approx(0.0, abs=1e-6)
    shift = torch.arange(rows.numel(), dtype=logits.dtype)[None, :, None]
    for moved in (truth + 7.0, truth * 3.0, truth * 0.01,
                  truth * 5.0 + shift * 100.0):
        assert heatmap.gauge_fixed_kl(moved, heat, view, rows).item() == \
            pytest.approx(0.0, abs=1e-6)
    worse = heatmap.gauge_fixed_kl(logits, heat, view, rows).item()
    assert worse > 1e-3
    assert heatmap.gauge_fixed_kl(-truth, heat, view, rows).item() > worse


def test_oracle_bce_saturates_on_the_oracle_and_is_ln2_when_flat():
    """The reference's own properties (:324-345, :587-619)."""
    lay, blocks, view, rows, heat, logits = _transport_case(1)
    oracle = _oracle_set(heat, lay, blocks, rows)
    n_video = view.n_video_tiles
    confident = torch.zeros_like(logits)
    confident[:, :, :n_video] = torch.where(oracle, 30.0, -30.0)

    def bce(x):
        return heatmap.oracle_bce(x, heat, view, blocks, rows,
                                  oracle=oracle).item()

    assert bce(confident) < 1e-5
    assert bce(-confident) > 10
    assert bce(torch.zeros_like(logits)) == pytest.approx(math.log(2.0),
                                                          abs=1e-6)
    base = bce(logits)
    per_row = logits + torch.arange(
        rows.numel(), dtype=logits.dtype)[None, :, None] * 100.0
    assert bce(logits + 500.0) == pytest.approx(base, rel=1e-4)
    assert bce(per_row) == pytest.approx(base, rel=1e-4)
    # Descent raises the oracle's blocks and lowers the others.
    x = torch.zeros_like(logits).requires_grad_(True)
    heatmap.oracle_bce(x, heat, view, blocks, rows, oracle=oracle).backward()
    valid = _decision(view, rows)
    grad = x.grad[:, :, :n_video]
    assert (grad[oracle & valid] < 0).all()
    assert (grad[~oracle & valid] > 0).all()
