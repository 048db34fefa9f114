"""Failure detection without a GPU fault: every device-side wait of the scan
kernels is bounded.  heph_selftest_wait_timeout runs the production look-back
wait and the staged-part mbarrier wait against partners that never arrive;
each wait must give up within its bound, the host must read the failure as
DispatchFailed on its next synchronisation, and the device must stay usable."""
import ctypes
import time

import numpy as np
import pytest

from hephaestus_b200 import CudaFullReductionOps, Layout, StridedView, SumOp
from hephaestus_b200 import _native as N
from hephaestus_b200.core import DispatchFailed, check

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("which,message", [(0, "look-back timeout"), (1, "bulk copy timeout")])
def test_bounded_wait_gives_up_and_device_stays_usable(device, which, message):
    device.synchronize()
    t0 = time.monotonic()
    check(N.lib.heph_selftest_wait_timeout(device.handle, which, None))
    with pytest.raises(DispatchFailed) as e:
        device.synchronize()
    elapsed = time.monotonic() - t0
    assert message in e.value.message
    assert elapsed < 20, f"bounded wait took {elapsed:.1f} s"
    # The error bit was consumed and the context is intact.
    device.synchronize()
    x = np.arange(1, 100_001, dtype=np.uint32)
    buf, out = device.upload(x), device.alloc_zeroed(np.uint32, 1)
    CudaFullReductionOps().reduce_full_into(SumOp, device, StridedView(buf, Layout.c_contiguous([x.size])),
                                            StridedView(out, Layout.c_contiguous([1])))
    assert int(device.download_owned(out)[0]) == int(x.astype(np.uint64).sum()) % (1 << 32)
    device.synchronize()


def test_selftest_rejects_unknown_wait(device):
    from hephaestus_b200 import InvalidConfiguration
    with pytest.raises(InvalidConfiguration):
        check(N.lib.heph_selftest_wait_timeout(device.handle, 7, None))
