"""The allocation-free predictor entry point, called through the C ABI.

Some callers cannot allocate device memory themselves: a host framework that
owns all GPU memory through its own pool, or a plugin interface that hands a
kernel only its inputs and outputs. `veda_predict_logits_noalloc` serves them
with a fixed scratch array inside the library instead of a caller-provided
workspace. These tests check that it computes exactly what the workspace
entry point `veda_predict_logits` computes, on two calls in a row (the
second call reuses scratch the first one left behind), and that it rejects
problems larger than its fixed scratch. This file is collected last.
"""

import pytest
import torch

from miowtion_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def _inputs(n_heads, n_q, n_k, seed):
    gen = torch.Generator().manual_seed(seed)
    feats_q = torch.randn(n_heads, n_q, 384, generator=gen)
    feats_k = torch.randn(n_heads, n_k, 384, generator=gen)
    proj_q = torch.randn(n_heads + 2, 384, 128, generator=gen) * 0.02
    proj_k = torch.randn(n_heads + 2, 384, 128, generator=gen) * 0.02
    heads = torch.randperm(n_heads + 2, generator=gen)[:n_heads]
    return [t.to(DEV).contiguous() for t in (feats_q, feats_k, proj_q,
                                             proj_k, heads)]


def _with_workspace(fq, fk, pq, pk, heads):
    n_heads, n_q, n_k = fq.shape[0], fq.shape[1], fk.shape[1]
    ws_bytes = _lib.load().veda_predict_workspace(n_heads, n_q, n_k)
    ws = torch.empty(ws_bytes // 4, dtype=torch.float32, device=DEV)
    out = torch.empty(n_heads, n_q, n_k, dtype=torch.float32, device=DEV)
    _lib.call('veda_predict_logits', fq.data_ptr(), fk.data_ptr(),
              pq.data_ptr(), pk.data_ptr(), heads.data_ptr(), n_heads, n_q,
              n_k, out.data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_ptr())
    return out


def _no_alloc(fq, fk, pq, pk, heads):
    n_heads, n_q, n_k = fq.shape[0], fq.shape[1], fk.shape[1]
    out = torch.empty(n_heads, n_q, n_k, dtype=torch.float32, device=DEV)
    _lib.call('veda_predict_logits_noalloc', fq.data_ptr(), fk.data_ptr(),
              pq.data_ptr(), pk.data_ptr(), heads.data_ptr(), n_heads, n_q,
              n_k, out.data_ptr(), _lib.stream_ptr())
    return out


def test_no_alloc_matches_workspace_entry_point_twice():
    # A larger call with other inputs first fills the shared scratch with
    # values that mean nothing to the calls after it. Then two calls in a
    # row with different shapes, each over what the one before left. Both
    # entry points run the same kernels and differ only in where the
    # scratch lives, so the logits must agree bit for bit: a read of stale
    # scratch would show as a difference.
    _no_alloc(*_inputs(8, 400, 400, 7))
    for n_heads, n_q, n_k, seed in ((6, 280, 280, 1), (3, 150, 97, 2)):
        args = _inputs(n_heads, n_q, n_k, seed)
        want = _with_workspace(*args)
        got = _no_alloc(*args)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    assert _lib.device_status(reset=True) == 0


def test_no_alloc_rejects_problems_beyond_its_scratch():
    limit = 8388608  # VEDA_PREDICT_NOALLOC_MAX_FLOATS
    n_heads, n_q = 2, 1
    n_k = limit // (n_heads * 128)  # one float too many
    fq = torch.zeros(1, dtype=torch.float32, device=DEV)
    with pytest.raises(ValueError, match='scratch'):
        _lib.call('veda_predict_logits_noalloc', fq.data_ptr(),
                  fq.data_ptr(), fq.data_ptr(), fq.data_ptr(), fq.data_ptr(),
                  n_heads, n_q, n_k, fq.data_ptr(), _lib.stream_ptr())
