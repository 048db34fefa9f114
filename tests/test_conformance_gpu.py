"""The reference's conformance clauses and CUDA contract cases, run through
the seams on the GPU and compared exactly with the values the reference
asserts (tests/golden/reference_fixtures.json, each case citing its source
file:line in hephaestus)."""
import numpy as np
import pytest

import hephaestus_b200.seams as S
from hephaestus_b200 import (CudaAxisReductionOps, CudaFullReductionOps, CudaScanOps, DispatchFailed,
                             Layout, MaxOp, MinOp, ProdOp, StridedView, SumOp)
from hephaestus_b200.core import CumProdOp, CumSumOp
from tests.golden_util import DT, cases_of_kind, load_cases

pytestmark = pytest.mark.gpu

OPS = {"sum": SumOp, "prod": ProdOp, "min": MinOp, "max": MaxOp}
SCAN_OPS = {"sum": CumSumOp, "prod": CumProdOp}
CASES = {c["id"]: c for c in load_cases()}


def L(d):
    return Layout.try_new(d["shape"], d["strides"], d["offset"])


def upload_input(device, c):
    a = np.array(c["input"], dtype=DT[c["dtype"]])
    if a.size == 0:
        return device.alloc_zeroed(a.dtype, 0), a
    return device.upload(a), a


@pytest.mark.parametrize("cid", cases_of_kind("reduce_full", "reduce_full_prepared"))
def test_full_reduction_clause(device, cid):
    c = CASES[cid]
    buf, a = upload_input(device, c)
    ops = CudaFullReductionOps()
    ol = L(c["out_layout"]) if "out_layout" in c else Layout.c_contiguous([1])
    init = np.array(c.get("out_init", [0] * ol.size()), dtype=a.dtype)
    out = device.upload(init)
    if "error" in c:
        with pytest.raises(DispatchFailed) as e:
            ops.reduce_full_into(OPS[c["op"]], device, StridedView(buf, L(c["layout"])), StridedView(out, ol))
        assert e.value.message == c["error"], c["source"]
        np.testing.assert_array_equal(device.download_owned(out), init)  # untouched
        return
    if c["kind"] == "reduce_full_prepared":
        prep = ops.prepare_reduce_full(OPS[c["op"]], device, StridedView(buf, L(c["layout"])), StridedView(out, ol))
        ops.dispatch_full(device, prep)
        np.testing.assert_array_equal(device.download_owned(out), c["expected"])
        ops.dispatch_full(device, prep)
        np.testing.assert_array_equal(device.download_owned(out), c["expected"])
        device.write_buffer(buf, np.array(c["rewrite"], dtype=a.dtype))
        ops.dispatch_full(device, prep)
        np.testing.assert_array_equal(device.download_owned(out), c["expected_after_rewrite"])
        return
    ops.reduce_full_into(OPS[c["op"]], device, StridedView(buf, L(c["layout"])), StridedView(out, ol))
    np.testing.assert_array_equal(device.download_owned(out), np.array(c["expected"], dtype=a.dtype),
                                  err_msg=c["source"])


@pytest.mark.parametrize("cid", cases_of_kind("reduce_axis", "reduce_axis_prepared"))
def test_axis_reduction_clause(device, cid):
    c = CASES[cid]
    buf, a = upload_input(device, c)
    lay = L(c["layout"])
    axis = c["axis"]
    if "out_layout" in c:
        ol = L(c["out_layout"])
    else:
        shape = list(lay.shape)
        shape[axis] = 1
        ol = Layout.c_contiguous(shape)
    init = np.array(c.get("out_init", [0] * max(ol.size(), 1)), dtype=a.dtype)
    out = device.upload(init)
    ops = CudaAxisReductionOps()
    op = c["op"]

    def call():
        if op == "mean":
            ops.mean_axis_into(device, StridedView(buf, lay), axis, StridedView(out, ol))
        elif op == "prod":
            ops.prod_axis_into(device, StridedView(buf, lay), axis, StridedView(out, ol))
        else:
            ops.reduce_axis_into(OPS[op], device, StridedView(buf, lay), axis, StridedView(out, ol))

    if "error" in c or "error_prefix" in c:
        with pytest.raises(DispatchFailed) as e:
            call()
        if "error" in c:
            assert e.value.message == c["error"], c["source"]
        else:
            assert e.value.message.startswith(c["error_prefix"]), c["source"]
        np.testing.assert_array_equal(device.download_owned(out), init)
        return
    if c["kind"] == "reduce_axis_prepared":
        prep = ops.prepare_reduce_axis_into(OPS[op], device, StridedView(buf, lay), axis, StridedView(out, ol))
        for _ in range(2):
            ops.dispatch_prepared(device, prep)
            np.testing.assert_array_equal(device.download_owned(out), c["expected"])
        device.write_buffer(buf, np.array(c["rewrite"], dtype=a.dtype))
        ops.dispatch_prepared(device, prep)
        np.testing.assert_array_equal(device.download_owned(out), c["expected_after_rewrite"])
        return
    call()
    np.testing.assert_array_equal(device.download_owned(out), np.array(c["expected"], dtype=a.dtype),
                                  err_msg=c["source"])


@pytest.mark.parametrize("cid", cases_of_kind("scan", "scan_prepared"))
def test_scan_clause(device, cid):
    c = CASES[cid]
    buf, a = upload_input(device, c)
    lay = L(c["layout"])
    ol = L(c["out_layout"]) if "out_layout" in c else lay
    n = max(ol.size(), 1)
    init = np.array(c.get("out_init", [0] * n), dtype=a.dtype)
    out = device.upload(init) if init.size else device.alloc_zeroed(a.dtype, 0)
    ops = CudaScanOps()
    direction = 1 if c["reverse"] else 0
    if "error" in c or "error_prefix" in c:
        with pytest.raises(DispatchFailed) as e:
            ops.scan_axis_into(SCAN_OPS[c["op"]], device, StridedView(buf, lay), c["axis"], direction,
                               StridedView(out, ol))
        if "error" in c:
            assert e.value.message == c["error"], c["source"]
        else:
            assert e.value.message.startswith(c["error_prefix"]), c["source"]
        np.testing.assert_array_equal(device.download_owned(out), init)
        return
    if c["kind"] == "scan_prepared":
        prep = ops.prepare_scan_axis(SCAN_OPS[c["op"]], device, StridedView(buf, lay), c["axis"], direction,
                                     StridedView(out, ol))
        for _ in range(2):
            ops.dispatch_scan(device, prep)
            np.testing.assert_array_equal(device.download_owned(out), c["expected"])
        device.write_buffer(buf, np.array(c["rewrite"], dtype=a.dtype))
        ops.dispatch_scan(device, prep)
        np.testing.assert_array_equal(device.download_owned(out), c["expected_after_rewrite"])
        return
    ops.scan_axis_into(SCAN_OPS[c["op"]], device, StridedView(buf, lay), c["axis"], direction,
                       StridedView(out, ol))
    got = device.download_owned(out)
    np.testing.assert_array_equal(got[:len(c["expected"])], np.array(c["expected"], dtype=a.dtype),
                                  err_msg=c["source"])


def test_free_function_widths(device):
    # contract.rs:670-690: width 128 works, 192 is rejected with the reference message.
    host = np.arange(1027, dtype=np.uint32)
    buf = device.upload(host)
    out = S.reduction_with_width(SumOp, device, buf, 128)
    assert device.download_owned(out)[0] == host.sum()
    with pytest.raises(DispatchFailed) as e:
        S.reduction_with_width(SumOp, device, buf, 192)
    assert e.value.message == "reduction block width 192 must be a power of two"


def test_allocating_scan_conveniences(device):
    # contract.rs:1807-1911 through the allocating forms.
    buf = device.upload(np.arange(1, 7, dtype=np.int32))
    t = Layout.try_new([2, 3], [1, 2], 0)
    got = device.download_owned(S.cumprod(device, StridedView(buf, t), 0))
    np.testing.assert_array_equal(got, [1, 3, 5, 2, 12, 30])
    got = device.download_owned(S.suffix_prod(device, StridedView(buf, t), 1))
    np.testing.assert_array_equal(got, [15, 15, 5, 48, 24, 6])
    empty = device.alloc_zeroed(np.int32, 0)
    assert len(S.cumprod(device, StridedView(empty, Layout.c_contiguous([2, 0])), 1)) == 0


def test_prepared_batch_submission(device):
    """contract.rs:693-735: prepared min/max over u32 (i % 17) submitted as a
    batch; the batch replays its bound operands (rebind contract); prepared
    scans are not batchable."""
    host = (np.arange(1027) % 17).astype(np.uint32)
    buf = device.upload(host)
    lay, one = Layout.c_contiguous([1027]), Layout.c_contiguous([1])
    mn, mx = device.alloc_zeroed(np.uint32, 1), device.alloc_zeroed(np.uint32, 1)
    ops = CudaFullReductionOps()
    pmin = ops.prepare_reduce_full(MinOp, device, StridedView(buf, lay), StridedView(mn, one))
    pmax = ops.prepare_reduce_full(MaxOp, device, StridedView(buf, lay), StridedView(mx, one))
    m2 = device.upload(np.arange(1, 13, dtype=np.uint32))
    col = device.alloc_zeroed(np.uint32, 4)
    pcol = CudaAxisReductionOps().prepare_reduce_axis_into(SumOp, device, StridedView(m2, Layout.c_contiguous([3, 4])),
                                                           0, StridedView(col, Layout.c_contiguous([1, 4])))
    batch = S.submit_prepared_batch(device, [pmin, pmax, pcol])
    assert device.download_owned(mn)[0] == 0 and device.download_owned(mx)[0] == 16
    np.testing.assert_array_equal(device.download_owned(col), [15, 18, 21, 24])
    device.write_buffer(buf, host + 5)
    device.write_buffer(m2, np.full(12, 2, np.uint32))
    batch.launch()
    assert device.download_owned(mn)[0] == 5 and device.download_owned(mx)[0] == 21
    np.testing.assert_array_equal(device.download_owned(col), [6, 6, 6, 6])
    out = device.alloc_zeroed(np.uint32, 1027)
    pscan = CudaScanOps().prepare_scan_axis(CumSumOp, device, StridedView(buf, lay), 0, 0, StridedView(out, lay))
    from hephaestus_b200 import InvalidConfiguration
    with pytest.raises(InvalidConfiguration):
        S.Batch(device, [pscan])


MAPS = {"dot": 0, "trace": 1, "norm_l1": 2, "norm_l2": 3, "norm_max": 4}


@pytest.mark.parametrize("cid", cases_of_kind("map"))
def test_map_reduction_clause(device, cid):
    from hephaestus_b200 import _native as N
    import ctypes
    from hephaestus_b200.core import check
    c = CASES[cid]
    a, _ = upload_input(device, c)
    b = None
    if "input_b" in c:
        b, _ = upload_input(device, dict(c, input=c["input_b"]))
    out = device.upload(np.array([9.0], np.float32))
    ol = Layout.c_contiguous([1])
    av = StridedView(a, L(c["layout"]))
    bv = StridedView(b, L(c["layout_b"])) if b is not None else None
    if "error_prefix" in c:
        with pytest.raises(DispatchFailed) as e:
            S._map_call(device, MAPS[c["map"]], av, bv, StridedView(out, ol))
        assert e.value.message.startswith(c["error_prefix"]), c["source"]
        assert device.download_owned(out)[0] == 9.0
        return
    S._map_call(device, MAPS[c["map"]], av, bv, StridedView(out, ol))
    got = float(device.download_owned(out)[0])
    assert abs(got - c["expected"][0]) <= c.get("tolerance", 0.0), (c["source"], got)


def test_dense_vector_ops_prepared(device):
    """contract.rs:955-1029: prepared dot / norm_l2 reuse their output and observe rewrites."""
    ops = S.CudaDenseVectorOps()
    lhs = device.upload(np.array([1, 2, 3, 4], np.float32))
    rhs = device.upload(np.array([5, 6, 7, 8], np.float32))
    pd = ops.prepare_dot(device, lhs, rhs)
    out_ptr = pd.output().device_ptr()
    assert ops.dot_prepared(device, pd) == 70.0
    device.write_buffer(lhs, np.full(4, 2, np.float32))
    assert ops.dot_prepared(device, pd) == 52.0 and pd.output().device_ptr() == out_ptr
    pn = ops.prepare_norm_l2(device, lhs)
    assert ops.norm_l2_prepared(device, pn) == 4.0
    assert ops.norm_l1(device, rhs) == 26.0 and ops.norm_max(device, rhs) == 8.0
    t = S.trace(device, StridedView(device.upload(np.arange(1, 10, dtype=np.float32)), Layout.c_contiguous([3, 3])))
    assert device.download_owned(t)[0] == 15.0
    with pytest.raises(DispatchFailed):
        S.trace(device, StridedView(lhs, Layout.c_contiguous([1, 4])))
