"""Partitioned 1-D scan and reduce over 2+ GPUs (NCCL all-gather of per-rank
totals), checked bit-exactly against the oracle on the whole buffer.  Runs the
ranks as child processes (tests/dist_worker.py); skipped with fewer than two
GPUs."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("exchange", ["default", "nccl"])
def test_partitioned_scan_and_reduce(tmp_path, oracle, exchange):
    """exchange = default: the fused scan + reduce exchanges over peer memory
    (B200s on NVLink map each other's mailboxes); nccl: forced onto the NCCL
    all-gather (HEPH_DIST_EXCHANGE=nccl)."""
    import torch
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    world = min(world, 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    if exchange == "nccl":
        env["HEPH_DIST_EXCHANGE"] = "nccl"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", "29533" if exchange == "default" else "29535",
           os.path.join(ROOT, "tests", "dist_worker.py"), str(tmp_path)]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    used = {(tmp_path / f"exchange_{r}.txt").read_text() for r in range(world)}
    assert used == ({"nccl"} if exchange == "nccl" else {"peer"}), used
    cat = lambda name: np.concatenate([np.load(tmp_path / f"{name}_{r}.npy") for r in range(world)])  # noqa: E731
    xi, xu = cat("in_i32"), cat("in_u32")
    np.testing.assert_array_equal(xi, oracle.generate(oracle.GEN_I32_PM1000, 4, xi.size))
    np.testing.assert_array_equal(xu, oracle.generate(oracle.GEN_U32_LOW4, 1, xu.size))
    np.testing.assert_array_equal(cat("scan_i32"), oracle.scan_axis(xi, [xi.size], 0))
    np.testing.assert_array_equal(cat("scan_u32"), oracle.scan_axis(xu, [xu.size], 0, exclusive=True))
    np.testing.assert_array_equal(cat("fscan_i32"), oracle.scan_axis(xi, [xi.size], 0))
    np.testing.assert_array_equal(cat("fscan_u32"), oracle.scan_axis(xu, [xu.size], 0, exclusive=True))
    for r in range(world):
        assert np.load(tmp_path / f"sum_{r}.npy")[0] == int(xi.astype(np.int64).sum())
        assert np.load(tmp_path / f"max_{r}.npy")[0] == xu.max()
        assert np.load(tmp_path / f"fsum_{r}.npy")[0] == int(xi.astype(np.int64).sum())
        assert np.load(tmp_path / f"fmax_{r}.npy")[0] == xu.max()


def test_partitioned_scan_and_reduce_large(tmp_path):
    """2^28 + 5 elements over the ranks (every slice takes the chunked scan),
    each rank's slice compared in process with the oracle (see dist_worker)."""
    import torch
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    world = min(world, 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", "29534",
           os.path.join(ROOT, "tests", "dist_worker.py"), str(tmp_path), "large"]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stderr[-3000:]
    for r in range(world):
        assert (tmp_path / f"ok_{r}.txt").exists(), r
