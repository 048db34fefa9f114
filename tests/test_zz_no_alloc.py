"""The allocation-free full reduction (heph_reduce_full_noalloc), for callers
that cannot allocate device memory at call time, e.g. an embedder working
inside a fixed memory budget that only hands the library buffers it already
owns.  Called through the C ABI with raw device pointers and checked against
heph_reduce_full on the same input, twice in a row (the static scratch keeps
the previous call's contents, and the second call must not be disturbed by
them).  This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest

from hephaestus_b200 import _native as N
from hephaestus_b200 import CudaFullReductionOps, Layout, StridedView, SumOp, MaxOp
from hephaestus_b200.core import check

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,op,out_dtype", [
    (np.float32, SumOp, np.float32),
    (np.uint32, SumOp, np.uint32),
    (np.int32, SumOp, np.int64),
    (np.float64, MaxOp, np.float64),
])
def test_noalloc_matches_reduce_full(device, dtype, op, out_dtype):
    rng = np.random.default_rng(2024)
    for n in (1, 1000, (1 << 22) + 3):
        x = (rng.uniform(-1, 1, n) if np.dtype(dtype).kind == "f" else rng.integers(-1000, 1000, n)).astype(dtype)
        buf = device.upload(x)
        ref = device.alloc_zeroed(out_dtype, 1)
        CudaFullReductionOps().reduce_full_into(op, device, StridedView(buf, Layout.c_contiguous([n])),
                                                StridedView(ref, Layout.c_contiguous([1])))
        want = device.download_owned(ref)[0]
        out = device.alloc_zeroed(out_dtype, 1)
        from hephaestus_b200.core import dtype_code
        for _ in range(2):
            check(N.lib.heph_reduce_full_noalloc(op.code, dtype_code(dtype), dtype_code(out_dtype),
                                                 ctypes.c_void_p(buf.device_ptr()), n,
                                                 ctypes.c_void_p(out.device_ptr()),
                                                 ctypes.c_void_p(device.stream())))
            got = device.download_owned(out)[0]  # ordered after the kernel on the device's stream
            if np.dtype(out_dtype).kind == "f":
                tol = (1e-5 if np.dtype(dtype) == np.float32 else 1e-12) * max(1.0, float(np.abs(x).sum()))
                assert abs(float(got) - float(want)) <= tol
            else:
                assert got == want
    device.synchronize()


def test_noalloc_rejects_bad_arguments():
    assert N.lib.heph_reduce_full_noalloc(N.SUM, N.F32, N.U32, ctypes.c_void_p(16), 4,
                                          ctypes.c_void_p(16), None) == N.INVALID_CONFIGURATION
    assert N.lib.heph_reduce_full_noalloc(N.SUM, N.F32, N.F32, None, 4, ctypes.c_void_p(16),
                                          None) == N.INVALID_CONFIGURATION
