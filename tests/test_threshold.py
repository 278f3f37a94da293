"""The 'threshold' budget rule's per-head threshold (`threshold_allowed`)
against the reference's (tests/golden/make_threshold.py), on the CPU. The
selection itself runs on the GPU (tests/test_gpu_threshold.py)."""

import os

import numpy as np
import torch

from miowtion_b200 import mask as veda_mask

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden', 'threshold.npz')


def test_threshold_allowed_matches_reference():
    golden = np.load(GOLDEN)
    vals = torch.from_numpy(golden['allowed_vals'])
    before = list(veda_mask.SATURATED)
    got = veda_mask.threshold_allowed(vals, vals > float('-inf'), 2.6, 9)
    assert np.array_equal(got.numpy(), golden['allowed'])
    # Every row is counted; none of these reaches the cap of 9.
    assert veda_mask.SATURATED[1] - before[1] == vals.shape[0] * vals.shape[1]
    assert veda_mask.SATURATED[0] == before[0]


def test_threshold_spends_the_head_total_unevenly():
    gen = torch.Generator().manual_seed(3)
    vals = torch.randn(2, 40, 12, generator=gen).sort(
        -1, descending=True).values
    allowed = veda_mask.threshold_allowed(vals, torch.ones_like(
        vals, dtype=torch.bool), 4.0, 12)
    # round(4.0 * 40) candidates clear each head's threshold (no ties).
    assert allowed.sum(-1).tolist() == [160, 160]
    assert int(allowed.min()) >= 1 and allowed.float().std() > 0
