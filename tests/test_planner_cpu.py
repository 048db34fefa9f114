"""Host-side planning and validation of libheph_b200.so against the
reference's planner rules and error messages.  No GPU: these entry points
make no CUDA calls."""
import ctypes

import pytest

from hephaestus_b200 import _native as N
from hephaestus_b200.core import DispatchFailed, Layout, check
from tests.golden_util import load_cases


def lay(shape, strides=None, offset=0):
    l = Layout.c_contiguous(shape) if strides is None else Layout.try_new(shape, strides, offset)
    return l.native()


def plan_axis(in_l, in_len, out_l, out_len, axis, alias=False):
    noop = ctypes.c_int(-1)
    st = N.lib.heph_plan_axis_reduction(ctypes.byref(in_l), in_len, ctypes.byref(out_l), out_len,
                                        axis, int(alias), ctypes.byref(noop))
    return st, N.last_error(), noop.value


def plan_scan(in_l, in_len, out_l, out_len, axis, alias=False):
    noop = ctypes.c_int(-1)
    st = N.lib.heph_plan_axis_scan(ctypes.byref(in_l), in_len, ctypes.byref(out_l), out_len, axis,
                                   int(alias), ctypes.byref(noop))
    return st, N.last_error(), noop.value


def test_width_messages_match_reference():
    for c in load_cases():
        if c["kind"] == "width":
            with pytest.raises(DispatchFailed) as e:
                check(N.lib.heph_validate_reduction_width(c["width"]))
            assert e.value.message == c["error"], c["source"]
    check(N.lib.heph_validate_reduction_width(128))
    check(N.lib.heph_validate_reduction_width(256))
    assert N.lib.heph_validate_scan_width(3) == N.DISPATCH_FAILED
    assert N.last_error() == "scan block width 3 must be a power of two"


def test_pass_count_matches_reference():
    for c in load_cases():
        if c["kind"] == "pass_count":
            for length, width, passes in c["cases"]:
                assert N.lib.heph_reduction_pass_count(length, width) == passes


def test_axis_reduction_planner_rules():
    # core reduction.rs:410-500 (+ tests :502-570)
    st, msg, _ = plan_axis(lay([3, 4]), 12, lay([1, 4]), 4, 2)
    assert st == N.DISPATCH_FAILED and msg == "axis 2 is out of bounds for rank-2 reduction"
    st, msg, _ = plan_axis(lay([3, 4]), 12, lay([1, 3]), 3, 0)
    assert st == N.DISPATCH_FAILED
    assert msg == "axis reduction output shape mismatch: input [3, 4], axis 0, out [1, 3]"
    st, msg, _ = plan_axis(lay([3, 4]), 12, lay([3, 1]), 3, 1, alias=True)
    assert msg == "axis reduction output buffer must not alias input buffer"
    st, msg, _ = plan_axis(lay([3, 4]), 12, lay([3, 1], [0, 1]), 3, 1)
    assert msg == "axis reduction output layout must not contain zero-stride aliasing"
    st, msg, _ = plan_axis(lay([3, 4]), 11, lay([3, 1]), 3, 1)
    assert st == N.DISPATCH_FAILED and msg.startswith("layout rejected:")
    st, msg, noop = plan_axis(lay([0, 4]), 0, lay([0, 1]), 0, 1)
    assert st == N.OK and noop == 1
    st, msg, noop = plan_axis(lay([3, 0]), 0, lay([3, 1]), 3, 1)
    assert st == N.OK and noop == 0  # empty reduced axis still writes identities
    st, msg, noop = plan_axis(lay([4, 3], [1, 4]), 12, lay([4, 1]), 4, 1)
    assert st == N.OK and noop == 0


def test_axis_scan_planner_rules():
    # core scan.rs:87-178 (+ tests :266-344)
    st, msg, _ = plan_scan(lay([3, 4]), 12, lay([3, 4]), 12, 2)
    assert msg == "scan axis 2 is out of bounds for rank-2 scan"
    st, msg, _ = plan_scan(lay([3, 4]), 12, lay([4, 3]), 12, 1)
    assert msg == "scan output shape mismatch: input [3, 4], out [4, 3]"
    st, msg, _ = plan_scan(lay([2, 2]), 4, lay([2, 2]), 4, 0, alias=True)
    assert msg == "scan output buffer must not alias input buffer"
    st, msg, noop = plan_scan(lay([0, 4]), 0, lay([0, 4]), 0, 1)
    assert st == N.OK and noop == 1
    st, msg, _ = plan_scan(lay([2, 3], [1, 2], 1), 6, lay([2, 3]), 6, 1)
    assert st == N.DISPATCH_FAILED and msg.startswith("layout rejected:")
    st, msg, _ = plan_scan(lay([2, 2, 2]), 8, lay([2, 2, 2]), 8, 0)
    assert msg == "cuda-sm100a scan supports rank 2 only, got rank 3"
    st, msg, noop = plan_scan(lay([1 << 32]), 1 << 32, lay([1 << 32]), 1 << 32, 0)
    assert st == N.OK and noop == 0  # 64-bit extents [EXT]


def test_full_reduction_planner_rules():
    # hephaestus-cuda application/full_reduction_seam.rs:59-72
    st = N.lib.heph_plan_full_reduction(ctypes.byref(lay([3, 4])), 12, ctypes.byref(lay([2])), 2)
    assert st == N.DISPATCH_FAILED
    assert N.last_error() == "full reduction output must have exactly 1 element"
    st = N.lib.heph_plan_full_reduction(ctypes.byref(lay([3], [4])), 9, ctypes.byref(lay([1])), 1)
    assert st == N.OK  # diagonal of a 3x3 matrix
    st = N.lib.heph_plan_full_reduction(ctypes.byref(lay([3], [4])), 8, ctypes.byref(lay([1])), 1)
    assert st == N.DISPATCH_FAILED and N.last_error().startswith("layout rejected:")
    st = N.lib.heph_plan_full_reduction(ctypes.byref(lay([0])), 0, ctypes.byref(lay([1])), 1)
    assert st == N.OK


def test_layout_validation_negative_strides():
    assert N.lib.heph_layout_validate(ctypes.byref(lay([4], [-1], 3)), 4) == N.OK
    assert N.lib.heph_layout_validate(ctypes.byref(lay([4], [-1], 2)), 4) == N.DISPATCH_FAILED
    assert "below storage index 0" in N.last_error()


def test_dense_block_detection_through_views():
    """Transposed / reversed dense views are recognised (they then stream
    contiguously); gapped or overlapping views are not.  Exercised on the
    GPU by the parity tests; here through heph_layout_validate only for
    well-formedness of the layouts used there."""
    for shape, strides, off, n in [([300, 333], [1, 300], 0, 99900), ([1000], [-1], 999, 1000),
                                   ([10, 10, 10, 10], [1, 10, 100, 1000], 0, 10000)]:
        assert N.lib.heph_layout_validate(ctypes.byref(lay(shape, strides, off)), n) == N.OK
