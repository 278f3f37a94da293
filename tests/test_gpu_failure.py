"""Failure detection on the GPU without a fault: a bounded wait that nothing
completes expires, the kernel records VEDA_ERR_TIMEOUT in the device status
word and returns, the host reads the word and raises, and the CUDA context
keeps working afterwards. Every kernel of the library waits through the same
bounded helper."""

import time

import pytest
import torch

from miowtion_b200 import _lib

DEV = torch.device('cuda:0')


@pytest.mark.gpu
def test_expired_wait_is_reported_and_the_context_survives():
    _lib.device_status(reset=True)
    completed = torch.full((2,), -1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.call('veda_expire_wait', 200_000_000, completed.data_ptr(),
              _lib.stream_ptr())
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    # Neither wait completed; warp 1 left on warp 0's abort flag, well
    # before its own 4 s limit.
    assert completed.tolist() == [0, 0]
    assert 0.2 <= elapsed < 3.0, elapsed
    with pytest.raises(RuntimeError, match='timed out'):
        _lib.raise_on_device_status()
    assert _lib.device_status(reset=True) == 0
    # The context is intact: a tcgen05 kernel still runs and is right.
    gen = torch.Generator().manual_seed(5)
    a = torch.randn(128, 128, generator=gen).to(DEV, torch.bfloat16)
    b = torch.randn(128, 128, generator=gen).to(DEV, torch.bfloat16)
    d = torch.empty(128, 128, dtype=torch.float32, device=DEV)
    _lib.call('veda_probe_umma', a.data_ptr(), b.data_ptr(), d.data_ptr(), 0,
              _lib.stream_ptr())
    torch.testing.assert_close(d, a.float() @ b.float().T, rtol=1e-4,
                               atol=1e-3)
    _lib.raise_on_device_status()


@pytest.mark.gpu
def test_expire_wait_rejects_limits_outside_its_range():
    completed = torch.zeros(2, dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError, match='limit_ns'):
        _lib.call('veda_expire_wait', 10, completed.data_ptr(),
                  _lib.stream_ptr())
    with pytest.raises(ValueError, match='limit_ns'):
        _lib.call('veda_expire_wait', 5_000_000_000, completed.data_ptr(),
                  _lib.stream_ptr())
