"""The BASELINE configurations at their full sizes.

Configs 2-4 fit the multithreaded oracle: the device-generated inputs are
downloaded and the oracle runs on exactly those, element by element
(integers and argmax indices bit-exact, f64 within 1e-12 * sum|x| per
column).  Config 5 (2^32 elements, 16 GiB in + 16 GiB out) is compared
element by element too, in 1 GiB pieces: the oracle scans each downloaded
piece seeded with its own running carry, and the i64 total is checked against
the oracle's widening sum."""
import numpy as np
import pytest

import hephaestus_b200 as H
import hephaestus_b200.seams as S
from hephaestus_b200.core import CumSumOp, Layout, MaxOp, StridedView, SumOp

pytestmark = pytest.mark.gpu


def test_config2_u32_exclusive_scan_2p28(device, oracle):
    n = 1 << 28
    x = device.alloc_uninitialized(np.uint32, n)
    S.synth_fill(device, x, S.SYNTH_U32_LOW4, seed=1)
    y = device.alloc_uninitialized(np.uint32, n)
    lay = Layout.c_contiguous([n])
    H.CudaScanOps().scan_axis_into(CumSumOp, device, StridedView(x, lay), 0, 0, StridedView(y, lay), exclusive=True)
    hx = device.download_owned(x)
    # The device generator is the host one (integer SplitMix64 stream).
    np.testing.assert_array_equal(hx[:1 << 20], oracle.generate(oracle.GEN_U32_LOW4, 1, 1 << 20))
    want = np.empty_like(hx)
    oracle.exclusive_scan_u32_mt(hx, want)
    got = device.download_owned(y)
    np.testing.assert_array_equal(got, want)


def test_config3_f32_row_max_argmax_65536x4096(device, oracle):
    rows, cols = 65536, 4096
    x = device.alloc_uninitialized(np.float32, rows * cols)
    S.synth_fill(device, x, S.SYNTH_F32_NORMAL, seed=2)
    S.synth_inject_row_ties(device, x, rows, cols, seed=2)
    vals = device.alloc_zeroed(np.float32, rows)
    idx = device.alloc_zeroed(np.uint32, rows)
    il, ol = Layout.c_contiguous([rows, cols]), Layout.c_contiguous([rows, 1])
    H.CudaAxisReductionOps().argmax_axis_into(device, StridedView(x, il), 1, StridedView(vals, ol),
                                              StridedView(idx, ol))
    hx = device.download_owned(x)
    want_v, want_i = oracle.row_argmax_f32_mt(hx, rows, cols)
    np.testing.assert_array_equal(device.download_owned(vals), want_v)
    np.testing.assert_array_equal(device.download_owned(idx), want_i)
    # About 1 % of the rows carry an injected exact tie of their maximum.
    m = hx.reshape(rows, cols)
    ties = int(((m == want_v[:, None]).sum(axis=1) > 1).sum())
    assert 300 < ties < 1000, ties


def test_config4_f64_column_sum_4096x65536(device, oracle):
    rows, cols = 4096, 65536
    x = device.alloc_uninitialized(np.float64, rows * cols)
    S.synth_fill(device, x, S.SYNTH_F64_UNIT, seed=3)
    out = device.alloc_zeroed(np.float64, cols)
    H.CudaAxisReductionOps().reduce_axis_into(SumOp, device, StridedView(x, Layout.c_contiguous([rows, cols])), 0,
                                              StridedView(out, Layout.c_contiguous([1, cols])))
    hx = device.download_owned(x)
    want = oracle.col_sum_f64_mt(hx, rows, cols)
    got = device.download_owned(out)
    absum = np.abs(hx.reshape(rows, cols)).sum(axis=0)  # inputs are in [0, 1)
    assert np.all(np.abs(got - want) <= 1e-12 * np.maximum(absum, 1.0))


def test_config5_i32_scan_and_widening_sum_2p32(device, oracle):
    n = 1 << 32
    x = device.alloc_uninitialized(np.int32, n)
    S.synth_fill(device, x, S.SYNTH_I32_PM1000, seed=4)
    y = device.alloc_uninitialized(np.int32, n)
    s64 = device.alloc_zeroed(np.int64, 1)
    lay, one = Layout.c_contiguous([n]), Layout.c_contiguous([1])
    H.CudaScanOps().scan_axis_into(CumSumOp, device, StridedView(x, lay), 0, 0, StridedView(y, lay))
    H.CudaFullReductionOps().reduce_full_into(SumOp, device, StridedView(x, lay), StridedView(s64, one))
    total = int(device.download_owned(s64)[0])

    # Every one of the 2^32 outputs against the oracle's scan of the downloaded
    # input, 1 GiB at a time, each piece seeded with the oracle's running
    # (wrapping) carry; the i64 total against the oracle's widening sum.
    chunk = 1 << 28
    xs, ys, want = (np.empty(chunk, np.int32) for _ in range(3))
    carry, want_total = 0, 0
    for off in range(0, n, chunk):
        device.download_sub_buffer(x, off, xs)
        device.download_sub_buffer(y, off, ys)
        if off == 0:
            np.testing.assert_array_equal(xs[:1 << 20], oracle.generate(oracle.GEN_I32_PM1000, 4, 1 << 20))
        oracle.inclusive_scan_i32_mt(xs, want, carry)
        np.testing.assert_array_equal(ys, want, err_msg=f"scan piece at {off}")
        carry = int(want[-1])
        want_total += oracle.sum_i32_to_i64_mt(xs)
    assert total == want_total
    assert carry == (total + (1 << 31)) % (1 << 32) - (1 << 31)


def test_config1_f32_sum_2p20_batch_and_single(device, oracle):
    n, nbuf = 1 << 20, 64
    bufs = []
    for b in range(nbuf):
        xb = device.alloc_uninitialized(np.float32, n)
        S.synth_fill(device, xb, S.SYNTH_F32_UNIFORM_PM1, seed=b)
        bufs.append(xb)
    out = device.alloc_zeroed(np.float32, nbuf)
    single = device.alloc_zeroed(np.float32, 1)
    lay = Layout.c_contiguous([n])
    ops = H.CudaFullReductionOps()
    prepared = [ops.prepare_reduce_full(SumOp, device, StridedView(bufs[b], lay),
                                        StridedView(out, Layout.try_new([1], [1], b))) for b in range(nbuf)]
    S.Batch(device, prepared).launch()
    got = device.download_owned(out)
    for b in range(0, nbuf, 9):
        hx = device.download_owned(bufs[b])
        want = oracle.reduce_full(hx, [n])
        assert abs(float(got[b]) - float(want)) <= 1e-5 * float(np.abs(hx).sum())
        ops.reduce_full_into(SumOp, device, StridedView(bufs[b], lay), StridedView(single, Layout.c_contiguous([1])))
        assert abs(float(device.download_owned(single)[0]) - float(want)) <= 1e-5 * float(np.abs(hx).sum())
        ops.reduce_full_into(MaxOp, device, StridedView(bufs[b], lay), StridedView(single, Layout.c_contiguous([1])))
        assert float(device.download_owned(single)[0]) == float(hx.max())
