"""Normalized parity errors for the floating-point GPU tests.

The bar for attention outputs, gradients and scores is stated on the
normalized error max|got - want| / max|want| over the compared elements:
at most 2e-2 against the fp32 oracle for forward outputs and for
gradients (the tests also keep the reference's own elementwise bars,
rtol = atol = 2e-2 forward and 3e-2 for gradients). Every
check is recorded, printed, and summarised at the end of the test session
(conftest.py) so a run's log carries the measured values, not only a pass.
"""

from __future__ import annotations

import numpy as np

RECORDS: list[tuple[str, float, float]] = []

FWD = 2e-2   # attention outputs against the fp32 oracle
GRAD = 2e-2  # dq, dk, dv against the fp32 oracle


def _np(x):
    if hasattr(x, 'detach'):
        x = x.detach().float().cpu().numpy()
    return np.asarray(x, dtype=np.float64)


def max_rel_err(got, want, where=None) -> float:
    """max|got - want| / max|want| (over `where` when given)."""
    got, want = _np(got), _np(want)
    if where is not None:
        got, want = got[where], want[where]
    if got.shape != want.shape:
        raise ValueError(f'shapes differ: {got.shape} vs {want.shape}')
    if got.size == 0:
        raise ValueError('nothing to compare')
    scale = float(np.abs(want).max())
    diff = float(np.abs(got - want).max())
    return diff / scale if scale > 0 else diff


def assert_rel(got, want, bound: float, what: str, where=None) -> float:
    """Asserts the normalized error is within `bound`; records and prints
    the measured value."""
    err = max_rel_err(got, want, where)
    RECORDS.append((what, err, bound))
    print(f'parity {what}: max|got-want|/max|want| = {err:.2e} '
          f'(bound {bound:.0e})')
    assert err <= bound, (f'{what}: normalized error {err:.3e} above '
                          f'{bound:.0e}')
    return err
