"""Partitioned 1-D reduce and scan across GPUs (one process per GPU).

Each rank owns one contiguous slice of a global 1-D buffer, slices in rank
order.  The exchange is a single NCCL all-gather of one element per rank,
issued by ``libheph_b200.so`` on the compute stream (see
``hephaestus_b200/csrc/dist.cu``); ``torch.distributed`` is only used here to
ship the NCCL id from rank 0 to the others.  [EXT] — the reference has no
multi-device path.
"""
from __future__ import annotations

import ctypes

from . import _native as N
from .core import CudaDevice, StridedView, check


def unique_id() -> bytes:
    buf = ctypes.create_string_buffer(N.COMM_ID_BYTES)
    check(N.lib.heph_comm_unique_id(buf))
    return buf.raw


class Communicator:
    def __init__(self, device: CudaDevice, comm_id: bytes, nranks: int, rank: int):
        if len(comm_id) != N.COMM_ID_BYTES:
            raise ValueError("communicator id must be 128 bytes")
        h = ctypes.c_void_p()
        check(N.lib.heph_comm_init(device.handle, comm_id, int(nranks), int(rank), ctypes.byref(h)))
        self._h = h
        self.device = device
        self.nranks = nranks
        self.rank = rank

    @staticmethod
    def from_torch(device: CudaDevice, group=None) -> "Communicator":
        """Create the communicator of the current torch.distributed job."""
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        box = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0, group=group)
        return Communicator(device, box[0], world, rank)

    def reduce_full_into(self, op, input: StridedView, output: StridedView, stream=None):
        il, ol = input.layout.native(), output.layout.native()
        check(N.lib.heph_partitioned_reduce_full(self._h, op.code, input.buffer.handle,
                                                 ctypes.byref(il), output.buffer.handle,
                                                 ctypes.byref(ol),
                                                 ctypes.c_void_p(stream) if stream else None))

    def scan_into(self, op, input: StridedView, output: StridedView, exclusive: bool = False,
                  stream=None):
        il, ol = input.layout.native(), output.layout.native()
        check(N.lib.heph_partitioned_scan(self._h, op.code, int(bool(exclusive)),
                                          input.buffer.handle, ctypes.byref(il),
                                          output.buffer.handle, ctypes.byref(ol),
                                          ctypes.c_void_p(stream) if stream else None))

    def scan_reduce_into(self, scan_op, input: StridedView, scan_output: StridedView, reduce_op,
                         reduce_output: StridedView, exclusive: bool = False, stream=None):
        """scan_into and reduce_full_into of the same global buffer in one pass
        over the slice for both exchanges (heph_partitioned_scan_reduce)."""
        il, sl, rl = input.layout.native(), scan_output.layout.native(), reduce_output.layout.native()
        check(N.lib.heph_partitioned_scan_reduce(self._h, scan_op.code, int(bool(exclusive)),
                                                 input.buffer.handle, ctypes.byref(il),
                                                 scan_output.buffer.handle, ctypes.byref(sl), reduce_op.code,
                                                 reduce_output.buffer.handle, ctypes.byref(rl),
                                                 ctypes.c_void_p(stream) if stream else None))

    @property
    def peer_exchange(self) -> bool:
        """True when scan_reduce_into exchanges over peer memory (one kernel)
        instead of an NCCL all-gather; the same on every rank."""
        v = ctypes.c_int(0)
        check(N.lib.heph_comm_peer_exchange(self._h, ctypes.byref(v)))
        return bool(v.value)

    def wait(self, timeout_s: float, stream=None):
        """Host-side deadline on the calls queued on `stream` (heph_comm_wait):
        returns once they finished; raises HephaestusError (DispatchFailed)
        after aborting the communicator when NCCL reports an error or the
        deadline passes first (a peer rank died or never arrived)."""
        check(N.lib.heph_comm_wait(self._h, ctypes.c_void_p(stream) if stream else None,
                                   max(1, int(timeout_s * 1000))))

    def abort(self):
        if self._h:
            N.lib.heph_comm_abort(self._h)

    def destroy(self):
        if self._h:
            N.lib.heph_comm_destroy(self._h)
            self._h = ctypes.c_void_p(0)


def carries(totals, op_code: int = N.SUM, dtype=None):
    """Host restatement of the carry rule used by the partitioned scan:
    carry[r] = fold of totals[0..r-1] (identity for rank 0).  Used by the CPU
    tests of the rank logic; the device computes the same fold."""
    import numpy as np

    t = np.asarray(totals, dtype=dtype)
    out = np.empty_like(t)
    acc = t.dtype.type(1 if op_code == N.PROD else 0)
    with np.errstate(over="ignore"):
        for r in range(len(t)):
            out[r] = acc
            acc = acc * t[r] if op_code == N.PROD else acc + t[r]
    return out
