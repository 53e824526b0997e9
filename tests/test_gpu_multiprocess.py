"""GPU: parity of the one-process-per-GPU mode (the mode bench.py measures at N > 1): IPC-mapped peers,
symmetric-heap buffers and NVLS across processes, against the oracle (tests/mp_parity_worker.py)."""

import os
import socket
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_multiprocess_collectives_match_oracle():
    ngpu = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if ngpu < 2:
        pytest.skip("needs >= 2 GPUs")
    n = min(ngpu, 8)
    env = dict(os.environ, DTORCH_COMM_TIMEOUT_SECOND="30")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "tests", "mp_parity_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    assert "MP PARITY OK" in r.stdout
