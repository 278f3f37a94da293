"""The stage-1 seer KL: the oracle's restatement and the package's torch
form against the reference's values (tests/golden/make_teacher.py), on
the CPU. The collector itself runs on the GPU (tests/test_gpu_teacher.py)."""

import os
import types

import numpy as np
import pytest
import torch

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
