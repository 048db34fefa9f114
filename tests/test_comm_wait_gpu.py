"""Host-side deadline on NCCL (heph_comm_wait) with two real ranks: a rank
that never joins an exchange makes the other's wait abort the communicator
with DispatchFailed at its deadline instead of hanging, and the device stays
usable.  Child processes on two GPUs, NVLS off; skipped with fewer GPUs."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_wait_deadline_aborts_on_absent_rank(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    report = tmp_path / "rank0.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29547",
           os.path.join(ROOT, "tests", "comm_wait_worker.py"), str(report)]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-3000:]
    found = json.loads(report.read_text())
    x0 = np.arange(1000, dtype=np.int64)
    assert found["joined_sum"] == int(x0.sum() + (x0 + 1000).sum())
    assert "deadline of 2000 ms expired" in found["wait"], found["wait"]
    assert 1.5 < found["wait_s"] < 30
    assert found["local_sum"] == int(x0.sum())
