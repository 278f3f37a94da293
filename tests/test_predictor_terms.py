"""The predictor's optional score terms (count term, low-rank second-order
head) and their initialisations against the reference's LayerPredictor
(tests/golden/make_predictor_terms.py), on the CPU: the terms the package
adds to its kernel's logits, their parameter gradients, the argument rules
and `init_*_second_order_`. The kernel side runs in
tests/test_gpu_kernels.py."""

import os

import numpy as np
import pytest
import torch

import inputs
from miowtion_b200 import predictor as veda_predictor

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden',
                      'predictor_terms.npz')
SPEC = inputs.PREDICTOR_TERMS


@pytest.fixture(scope='module')
def golden():
    return np.load(GOLDEN)


def _layer(tensors, rank=SPEC['rank'], count=True):
    layer = veda_predictor.LayerPredictor(SPEC['heads'], SPEC['dim'], rank,
                                          count_term=count)
    with torch.no_grad():
        for name in ('proj_q', 'proj_k', 'so_q', 'so_k', 'count_gain'):
            if hasattr(layer, name):
                getattr(layer, name).copy_(tensors[name])
    return layer


def test_optional_terms_and_gradients_match_reference(golden):
    t = inputs.predictor_term_inputs(SPEC)
    layer = _layer(t)
    terms = layer.optional_terms(t['heads'], t['sq_q'], t['var_k'],
                                 t['log_count'])
    want = golden['logits'] - golden['plain']
    np.testing.assert_allclose(terms.detach().numpy(), want, rtol=1e-4,
                               atol=1e-4 * np.abs(want).max())
    # d/d(params) of <probe, logits>: the plain logits carry none of them.
    (terms * t['probe']).sum().backward()
    for name in ('so_q', 'so_k', 'count_gain'):
        got = getattr(layer, name).grad.numpy()
        ref = golden[f'grad_{name}']
        np.testing.assert_allclose(got, ref, rtol=0,
                                   atol=1e-5 * np.abs(ref).max(),
                                   err_msg=name)


def test_each_term_alone():
    t = inputs.predictor_term_inputs(SPEC)
    both = _layer(t).optional_terms(t['heads'], t['sq_q'], t['var_k'],
                                    t['log_count'])
    count = _layer(t, rank=0).optional_terms(t['heads'],
                                             log_count=t['log_count'])
    second = _layer(t, count=False).optional_terms(t['heads'], t['sq_q'],
                                                   t['var_k'])
    torch.testing.assert_close(count + second, both, rtol=1e-6, atol=1e-5)
    # The count term is a per-head gain on a per-key-tile constant.
    gain = t['count_gain'][t['heads']]
    torch.testing.assert_close(
        count, (gain[:, None, None] * t['log_count'][None, None, :]).expand(
            count.shape))
    assert _layer(t, rank=0, count=False).optional_terms(t['heads']) is None


def test_term_arguments_follow_the_reference_rules():
    t = inputs.predictor_term_inputs(SPEC)
    feats_q, feats_k, heads = t['feats_q'], t['feats_k'], t['heads']
    with pytest.raises(ValueError, match='log_count and count_term'):
        _layer(t, rank=0)(feats_q, feats_k, heads)
    with pytest.raises(ValueError, match='log_count and count_term'):
        _layer(t, rank=0, count=False)(feats_q, feats_k, heads,
                                       log_count=t['log_count'])
    with pytest.raises(ValueError, match='second-order features'):
        _layer(t, count=False)(feats_q, feats_k, heads)
    with pytest.raises(ValueError, match='second-order features'):
        _layer(t, rank=0, count=False)(feats_q, feats_k, heads,
                                       sq_q=t['sq_q'], var_k=t['var_k'])
    for rank in (-1, SPEC['dim'] + 1):
        with pytest.raises(ValueError, match='second_order_rank'):
            veda_predictor.LayerPredictor(2, SPEC['dim'], rank)


def test_parameter_names_and_initial_values():
    layer = veda_predictor.LayerPredictor(3, 128, 4, count_term=True)
    names = {n: tuple(p.shape) for n, p in layer.named_parameters()}
    assert names == {'proj_q': (3, 384, 128), 'proj_k': (3, 384, 128),
                     'so_q': (3, 128, 4), 'so_k': (3, 128, 4),
                     'count_gain': (3,)}
    assert torch.equal(layer.count_gain, torch.ones(3))
    pred = veda_predictor.TileScorePredictor(2, 3, 128, 4, count_term=True)
    assert pred.second_order_rank == 4 and pred.count_term
    assert 'layers.1.so_k' in dict(pred.named_parameters())


def test_exact_second_order_init_is_the_diagonal_cumulant():
    layer = veda_predictor.LayerPredictor(2, 128, 128)
    layer.init_exact_second_order_()
    product = torch.bmm(layer.so_q, layer.so_k.transpose(1, 2))
    torch.testing.assert_close(product,
                               torch.eye(128).expand(2, 128, 128) / 256.0)
    with pytest.raises(ValueError, match='exact term'):
        veda_predictor.LayerPredictor(2, 128, 8).init_exact_second_order_()


@pytest.mark.parametrize('rank', [SPEC['rank'], SPEC['dim']])
def test_low_rank_init_matches_reference(golden, rank):
    c_u, c_v = inputs.predictor_term_moments(SPEC)
    layer = veda_predictor.LayerPredictor(c_u.shape[0], SPEC['dim'], rank)
    layer.init_low_rank_second_order_(c_u, c_v)
    got = torch.bmm(layer.so_q, layer.so_k.transpose(1, 2)).detach().numpy()
    want = golden[f'low_rank_{rank}']
    np.testing.assert_allclose(got, want, rtol=0,
                               atol=1e-4 * np.abs(want).max())


def test_low_rank_init_rejects_bad_arguments():
    c_u, c_v = inputs.predictor_term_moments(SPEC)
    with pytest.raises(ValueError, match='no second-order head'):
        veda_predictor.LayerPredictor(2, 128).init_low_rank_second_order_(
            c_u, c_v)
    with pytest.raises(ValueError, match='shape'):
        veda_predictor.LayerPredictor(3, 128, 8).init_low_rank_second_order_(
            c_u, c_v)
    pred = veda_predictor.TileScorePredictor(2, 2, 128, 8)
    pred.init_low_rank_second_order_(torch.stack([c_u, c_u]),
                                     torch.stack([c_v, c_v]))
    torch.testing.assert_close(pred.layers[0].so_q, pred.layers[1].so_q)
    with pytest.raises(ValueError, match='one moment per layer'):
        veda_predictor.TileScorePredictor(
            3, 2, 128, 8).init_low_rank_second_order_(
                torch.stack([c_u, c_u]), torch.stack([c_v, c_v]))
