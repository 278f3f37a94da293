import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for path in (ROOT, os.path.join(ROOT, 'tests', 'golden')):
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
