"""Tensor parallelism on 2 GPUs (NCCL): parity of every rank with the reference.

Runs tests/tp_ranks.py under torchrun with two ranks; skipped on fewer GPUs.
NVLS is switched off for the test's NCCL communicator.
"""

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_tp2_parity():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    here = Path(__file__).resolve().parent
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), str(here / "tp_ranks.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert res.stdout.count("ok, worst") == 2, res.stdout[-2000:]
