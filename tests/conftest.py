import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for path in (ROOT, os.path.join(ROOT, 'tests'),
             os.path.join(ROOT, 'tests', 'golden')):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line(
        'markers', 'gpu: needs a B200 (sm_100a) and the built CUDA library')


def pytest_collection_modifyitems(config, items):
    """GPU tests fail loudly without CUDA when explicitly selected (-m gpu);
    in a default run on a CPU-only machine they are skipped."""
    markexpr = config.getoption('-m') or ''
    if 'gpu' in markexpr and 'not gpu' not in markexpr:
        return
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason='no CUDA device')
    for item in items:
        if 'gpu' in item.keywords:
            item.add_marker(skip)


def pytest_terminal_summary(terminalreporter):
    """The normalized parity errors the GPU tests measured, worst (relative
    to its bound) first."""
    import parity
    if not parity.RECORDS:
        return
    rows = sorted(parity.RECORDS, key=lambda r: r[1] / r[2], reverse=True)
    worst = rows[0]
    terminalreporter.write_line(
        f'parity: {len(rows)} normalized-error checks '
        '(max|got-want|/max|want|); worst against its bound: '
        f'{worst[0]} {worst[1]:.2e} (bound {worst[2]:.0e})')
    for what, err, bound in rows[:10]:
        terminalreporter.write_line(f'  {err:.2e} / {bound:.0e}  {what}')
