"""Host-side logic of the partitioned 1-D path with world_size 2-4 gloo ranks
on CPU: each rank owns a contiguous slice, exchanges its slice total, derives its
carry = fold of the lower ranks' totals (hephaestus_b200.dist.carries, the rule
dist.cu applies on the device) and scans its slice seeded with it; the
concatenation must equal the global scan.  A rank that fails before the
exchange must surface as an error on the other rank, not a hang."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=120):
    # Generous: spawned ranks import torch at very different speeds on a
    # loaded machine, and the rendezvous waits for the slowest.
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _scan_worker(rank, world, port, exclusive, result_dir):
    import torch
    from oracle import host_ref as oracle
    from hephaestus_b200.dist import carries
    _init(rank, world, port)
    n = 100_003
    full = oracle.generate(oracle.GEN_I32_PM1000, 4, n)
    per = (n + world - 1) // world
    lo, hi = rank * per, min(n, (rank + 1) * per)
    mine = full[lo:hi]
    total = np.array([oracle.reduce_full(mine, [mine.size])], dtype=np.int32)
    gathered = [torch.zeros(1, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(gathered, torch.from_numpy(total))
    totals = np.array([int(g[0]) for g in gathered], dtype=np.int32)
    carry = carries(totals, dtype=np.int32)[rank]
    local = oracle.scan_axis(mine, [mine.size], 0, exclusive=exclusive)
    with np.errstate(over="ignore"):
        local = (local.astype(np.int64) + int(carry)).astype(np.int64)
    local = ((local + 2**31) % 2**32 - 2**31).astype(np.int32)  # i32 wrap
    np.save(os.path.join(result_dir, f"r{rank}.npy"), local)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("exclusive,world", [(False, 2), (True, 2), (True, 3), (False, 4)])
def test_partitioned_scan_rank_logic(tmp_path, exclusive, world):
    from oracle import host_ref as oracle
    mp.spawn(_scan_worker, args=(world, _free_port(), exclusive, str(tmp_path)), nprocs=world, join=True)
    got = np.concatenate([np.load(tmp_path / f"r{r}.npy") for r in range(world)])
    full = oracle.generate(oracle.GEN_I32_PM1000, 4, 100_003)
    np.testing.assert_array_equal(got, oracle.scan_axis(full, [full.size], 0, exclusive=exclusive))


def _failing_worker(rank, world, port, result_dir):
    import torch
    _init(rank, world, port)
    # The exchange runs in a group with a short deadline; the rendezvous
    # above does not, so a slow start is not mistaken for the lost rank.
    group = dist.new_group(list(range(world)), timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise SystemExit(3)  # this rank drops out before the exchange
    try:
        out = [torch.zeros(1) for _ in range(world)]
        dist.all_gather(out, torch.ones(1), group=group)
        status = "completed"
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        status = "error: " + type(e).__name__
    with open(os.path.join(result_dir, "r0.txt"), "w") as fh:
        fh.write(status)


def test_lost_rank_surfaces_as_error(tmp_path):
    world = 2
    ctx = mp.start_processes(_failing_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                             join=False, start_method="spawn")
    try:
        ctx.join(timeout=60)
    except Exception:
        pass  # rank 1 exits non-zero by design
    for p in ctx.processes:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    status = (tmp_path / "r0.txt").read_text()
    assert status.startswith("error"), status


def test_carries_rule():
    from hephaestus_b200.dist import carries
    from hephaestus_b200 import _native as N
    np.testing.assert_array_equal(carries([3, 4, 5], dtype=np.int64), [0, 3, 7])
    np.testing.assert_array_equal(carries([2, 3, 4], N.PROD, dtype=np.int64), [1, 2, 6])
    np.testing.assert_array_equal(carries([2**31 - 1, 1, 1], dtype=np.int32), [0, 2**31 - 1, -2**31])


@pytest.mark.parametrize("scenario,ok,aborted,words", [
    (0, True, 0, ""),
    (1, False, 1, "asynchronous error"),
    (2, False, 1, "deadline of 50 ms expired"),
    (3, False, 0, "stream of the partitioned call failed"),
])
def test_comm_wait_policy(scenario, ok, aborted, words):
    """The host-side deadline of heph_comm_wait, run against scripted fakes of
    the stream and of NCCL (no GPU): it returns when the stream completes,
    aborts the communicator on an NCCL error or an expired deadline, and only
    reports a failed stream."""
    import ctypes
    from hephaestus_b200 import _native as N
    n = ctypes.c_int(-1)
    st = N.lib.heph_selftest_comm_wait_policy(scenario, 50, ctypes.byref(n))
    assert (st == 0) == ok
    assert n.value == aborted
    if not ok:
        assert st == N.DISPATCH_FAILED
        assert words in N.lib.heph_last_error().decode()
