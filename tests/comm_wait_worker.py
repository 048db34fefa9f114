"""Worker of tests/test_comm_wait_gpu.py (two ranks, torch.distributed.run):
one partitioned reduction that both ranks join and wait on with a deadline,
then one that rank 1 never joins (it stays alive and idle, so no peer memory
goes away): rank 0's wait must abort the communicator at its deadline and the
device must still compute afterwards.  Rank 0 writes its findings to the JSON
file named in argv[1]."""
import json
import os
import sys
import time

import numpy as np
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import hephaestus_b200 as H  # noqa: E402
from hephaestus_b200.core import HephaestusError, Layout, StridedView, SumOp  # noqa: E402
from hephaestus_b200.dist import Communicator  # noqa: E402


def main():
    dist.init_process_group("gloo")  # ships the NCCL id; host-side barriers
    rank = dist.get_rank()
    dev = H.CudaDevice(int(os.environ["LOCAL_RANK"]))
    comm = Communicator.from_torch(dev)
    x = np.arange(1000, dtype=np.int32) + 1000 * rank
    xb, out = dev.upload(x), dev.alloc_zeroed(np.int32, 1)
    lay, one = Layout.c_contiguous([x.size]), Layout.c_contiguous([1])
    found = {}

    comm.reduce_full_into(SumOp, StridedView(xb, lay), StridedView(out, one))
    comm.wait(30.0)
    found["joined_sum"] = int(dev.download_owned(out)[0])
    dist.barrier()

    if rank == 0:
        comm.reduce_full_into(SumOp, StridedView(xb, lay), StridedView(out, one))
        t0 = time.perf_counter()
        try:
            comm.wait(2.0)
            found["wait"] = "completed"
        except HephaestusError as e:
            found["wait"] = str(e)
        found["wait_s"] = time.perf_counter() - t0
        # The context is intact: a local reduction still runs and is right.
        local = dev.alloc_zeroed(np.int32, 1)
        H.CudaFullReductionOps().reduce_full_into(SumOp, dev, StridedView(xb, lay), StridedView(local, one))
        found["local_sum"] = int(dev.download_owned(local)[0])
        with open(sys.argv[1], "w") as fh:
            json.dump(found, fh)
    dist.barrier()  # rank 1 idles here until rank 0 is done
    if rank == 1:
        comm.abort()
    comm.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
