"""The C-ABI library loads and exports exactly what include/veda_b200.h
declares; argument validation runs on the host (no GPU needed)."""

import ctypes
import os
import re

import pytest

from miowtion_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), 'include',
                      'veda_b200.h')


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r'^\s*(?:int|int64_t)\s+(veda_\w+)\s*\(',
                                 text, flags=re.M)))


@pytest.fixture(scope='module')
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from miowtion_b200 import build
        build.build()
    return _lib.load()


def test_header_declares_the_bound_entry_points():
    assert declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert getattr(lib, name).restype is not None


def test_host_side_validation_needs_no_gpu(lib):
    # n_spans == 0 is rejected before any CUDA call.
    rc = lib.veda_build_layout(None, 0, 10, 10, 1, None, None, None)
    assert rc == _lib.VEDA_ERR_INVALID
    assert 'target span' in _lib.last_error()
    with pytest.raises(ValueError, match='target span'):
        _lib.check(rc, 'veda_build_layout')
    assert lib.veda_predict_workspace(2, 10, 12) == 2 * 22 * 128 * 4
    # Sizes whose byte count would not fit in 64 bits are refused, not
    # wrapped into a small (or negative) size.
    assert lib.veda_predict_workspace(2, 1 << 60, 12) == -1
    assert lib.veda_predict_workspace(0, 10, 12) == -1
    rc = lib.veda_predict_logits_noalloc(None, None, None, None, None, 2,
                                         1 << 60, 1 << 60, None, None)
    assert rc == _lib.VEDA_ERR_INVALID
    assert '2^31' in _lib.last_error()


def test_column_block_struct_layout():
    assert ctypes.sizeof(_lib.ColumnBlockC) == 32
    assert ctypes.sizeof(_lib.Span) == 32


def test_sm_reserve_is_validated_on_the_host(lib):
    with pytest.raises(ValueError, match='reserve'):
        _lib.call('veda_set_sm_reserve', -1)
    with pytest.raises(ValueError, match='reserve'):
        _lib.call('veda_set_sm_reserve', 1000)
    _lib.call('veda_set_sm_reserve', 0)
