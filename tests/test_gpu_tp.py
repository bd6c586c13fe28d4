"""Tensor-parallel projections on 2, 4 and 8 GPUs (column-parallel QKV+gate, row-parallel output projection),
through the NCCL and the peer-store
transports; each size is skipped with fewer GPUs.

Runs tests/tp_worker.py under torchrun (rendezvous on 127.0.0.1, NVLS off), bounded by a timeout."""
import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("nproc", [2, 4, 8])
def test_tp(nproc):
    if not torch.cuda.is_available() or torch.cuda.device_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "420", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           os.path.join(ROOT, "tests", "tp_worker.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=480)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "TP check ok" in res.stdout
