"""The head-parallel layer across two GPUs (both exchange transports and
the backward through the exchange), when the machine shows at least two:
tests/multi_gpu_check.py under torchrun, rendezvous on 127.0.0.1."""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2,
                    reason='needs two GPUs')
def test_two_ranks_equal_one_process():
    cmd = [sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           '--nproc-per-node', '2', '--master-addr', '127.0.0.1',
           '--master-port', str(_free_port()),
           os.path.join(HERE, 'multi_gpu_check.py')]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert res.stdout.count('equal the one-process layer') == 2
