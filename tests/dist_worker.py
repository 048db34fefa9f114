"""Worker of tests/test_multigpu_gpu.py, launched with torch.distributed.run:
every rank owns one contiguous slice of a global buffer generated on its GPU,
runs the partitioned scan / reduce through hephaestus_b200.dist, and writes its
slice of the results to the directory in argv[1]."""
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


def main():
    out_dir = sys.argv[1]
    dist.init_process_group("gloo")  # only ships the NCCL id
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = H.CudaDevice(int(os.environ["LOCAL_RANK"]))
    comm = Communicator.from_torch(dev)
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
