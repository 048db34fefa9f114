"""hephaestus_b200 — B200-native (sm_100a) reduce/scan path of hephaestus.

Drop-in for the ``FullReductionOps`` / ``AxisReductionOps`` / ``ScanOps``
seams of hephaestus-core over a CUDA ``ComputeDevice``; the kernels and the
C ABI live in ``libheph_b200.so`` (built by ``python -m hephaestus_b200.build``).
Importing this package fails if the library is missing: there is no CPU path.
"""
from .core import (AdapterUnavailable, AllocationFailed, CudaBuffer, CudaDevice, CumProdOp,
                   CumSumOp, DeviceUnavailable, DispatchFailed, HephaestusError,
                   InvalidConfiguration, Layout, LengthMismatch, MaxOp, MinOp, ProdOp,
                   ScanDirection, StridedView, SumOp, TransferFailed)
from .seams import CudaAxisReductionOps, CudaFullReductionOps, CudaScanOps

__all__ = [
    "AdapterUnavailable", "AllocationFailed", "CudaBuffer", "CudaDevice", "CumProdOp", "CumSumOp",
    "DeviceUnavailable", "DispatchFailed", "HephaestusError", "InvalidConfiguration", "Layout",
    "LengthMismatch", "MaxOp", "MinOp", "ProdOp", "ScanDirection", "StridedView", "SumOp",
    "TransferFailed", "CudaAxisReductionOps", "CudaFullReductionOps", "CudaScanOps",
]
