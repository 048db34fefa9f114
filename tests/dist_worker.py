"""Worker of tests/test_multigpu_gpu.py, launched with torch.distributed.run:
every rank owns one contiguous slice of a global buffer generated on its GPU,
runs the partitioned scan / reduce through hephaestus_b200.dist, and writes its
slice of the results to the directory in argv[1].

With argv[2] == "large" the buffer is 2^28 + 5 i32 elements, and every rank
checks its own slice in process instead: it downloads its input, the ranks
exchange the oracle's totals of their slices over gloo, and the oracle scans
the slice seeded with the lower ranks' carry; the fused and the separate
calls must both match it bit for bit, and the i64 sum must equal the oracle's
widening sum of the whole buffer.  Each rank writes ok_<rank>.txt when its
slice matches."""
import os
import sys

import numpy as np
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import hephaestus_b200 as H  # noqa: E402
import hephaestus_b200.seams as S  # noqa: E402
from hephaestus_b200.core import CumSumOp, Layout, MaxOp, StridedView, SumOp  # noqa: E402
from hephaestus_b200.dist import Communicator  # noqa: E402

TOTAL = 25_000_003
LARGE_TOTAL = (1 << 28) + 5


def check_large(out_dir, dev, comm, rank, world):
    from oracle import host_ref as oracle
    oracle.build()
    per = (LARGE_TOTAL + world - 1) // world
    lo, hi = rank * per, min(LARGE_TOTAL, (rank + 1) * per)
    n = hi - lo
    lay, one = Layout.c_contiguous([n]), Layout.c_contiguous([1])
    x = dev.alloc_uninitialized(np.int32, n)
    S.synth_fill(dev, x, S.SYNTH_I32_PM1000, seed=4, index_base=lo)
    yf, ys = dev.alloc_zeroed(np.int32, n), dev.alloc_zeroed(np.int32, n)
    sf, ss = dev.alloc_zeroed(np.int64, 1), dev.alloc_zeroed(np.int64, 1)
    for _ in range(2):
        comm.scan_reduce_into(CumSumOp, StridedView(x, lay), StridedView(yf, lay), SumOp, StridedView(sf, one))
        comm.scan_into(CumSumOp, StridedView(x, lay), StridedView(ys, lay))
        comm.reduce_full_into(SumOp, StridedView(x, lay), StridedView(ss, one))
    hx = dev.download_owned(x)
    np.testing.assert_array_equal(hx, oracle.generate(oracle.GEN_I32_PM1000, 4, n, index_base=lo))
    sums = [None] * world
    dist.all_gather_object(sums, oracle.sum_i32_to_i64_mt(hx))
    carry = sum(sums[:rank])
    carry = (carry + (1 << 31)) % (1 << 32) - (1 << 31)
    want = np.empty_like(hx)
    oracle.inclusive_scan_i32_mt(hx, want, carry)
    np.testing.assert_array_equal(dev.download_owned(yf), want)
    np.testing.assert_array_equal(dev.download_owned(ys), want)
    assert int(dev.download_owned(sf)[0]) == sum(sums)
    assert int(dev.download_owned(ss)[0]) == sum(sums)
    with open(os.path.join(out_dir, f"ok_{rank}.txt"), "w") as fh:
        fh.write(f"{n} elements from {lo}\n")


def main():
    out_dir = sys.argv[1]
    dist.init_process_group("gloo")  # only ships the NCCL id
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = H.CudaDevice(int(os.environ["LOCAL_RANK"]))
    comm = Communicator.from_torch(dev)
    with open(os.path.join(out_dir, f"exchange_{rank}.txt"), "w") as fh:
        fh.write("peer" if comm.peer_exchange else "nccl")
    if len(sys.argv) > 2 and sys.argv[2] == "large":
        check_large(out_dir, dev, comm, rank, world)
        dev.synchronize()
        dist.barrier()
        comm.destroy()
        dist.destroy_process_group()
        return
    per = (TOTAL + world - 1) // world
    lo, hi = rank * per, min(TOTAL, (rank + 1) * per)
    n = hi - lo
    lay, one = Layout.c_contiguous([n]), Layout.c_contiguous([1])

    xi = dev.alloc_uninitialized(np.int32, n)
    S.synth_fill(dev, xi, S.SYNTH_I32_PM1000, seed=4, index_base=lo)
    xu = dev.alloc_uninitialized(np.uint32, n)
    S.synth_fill(dev, xu, S.SYNTH_U32_LOW4, seed=1, index_base=lo)
    yi, yu = dev.alloc_zeroed(np.int32, n), dev.alloc_zeroed(np.uint32, n)
    s64, mx = dev.alloc_zeroed(np.int64, 1), dev.alloc_zeroed(np.uint32, 1)
    yf, s64f = dev.alloc_zeroed(np.int32, n), dev.alloc_zeroed(np.int64, 1)
    yp, mxp = dev.alloc_zeroed(np.uint32, n), dev.alloc_zeroed(np.uint32, 1)
    dev.synchronize()
    for _ in range(2):  # twice: the second call reuses the workspaces
        comm.scan_into(CumSumOp, StridedView(xi, lay), StridedView(yi, lay))
        comm.scan_into(CumSumOp, StridedView(xu, lay), StridedView(yu, lay), exclusive=True)
        comm.reduce_full_into(SumOp, StridedView(xi, lay), StridedView(s64, one))
        comm.reduce_full_into(MaxOp, StridedView(xu, lay), StridedView(mx, one))
        # The fused pair: one pass over the slice for both exchanges.
        comm.scan_reduce_into(CumSumOp, StridedView(xi, lay), StridedView(yf, lay), SumOp, StridedView(s64f, one))
        comm.scan_reduce_into(CumSumOp, StridedView(xu, lay), StridedView(yp, lay), MaxOp, StridedView(mxp, one),
                              exclusive=True)
    np.save(os.path.join(out_dir, f"in_i32_{rank}.npy"), dev.download_owned(xi))
    np.save(os.path.join(out_dir, f"in_u32_{rank}.npy"), dev.download_owned(xu))
    np.save(os.path.join(out_dir, f"scan_i32_{rank}.npy"), dev.download_owned(yi))
    np.save(os.path.join(out_dir, f"scan_u32_{rank}.npy"), dev.download_owned(yu))
    np.save(os.path.join(out_dir, f"sum_{rank}.npy"), dev.download_owned(s64))
    np.save(os.path.join(out_dir, f"max_{rank}.npy"), dev.download_owned(mx))
    np.save(os.path.join(out_dir, f"fscan_i32_{rank}.npy"), dev.download_owned(yf))
    np.save(os.path.join(out_dir, f"fsum_{rank}.npy"), dev.download_owned(s64f))
    np.save(os.path.join(out_dir, f"fscan_u32_{rank}.npy"), dev.download_owned(yp))
    np.save(os.path.join(out_dir, f"fmax_{rank}.npy"), dev.download_owned(mxp))
    dev.synchronize()
    dist.barrier()
    comm.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
