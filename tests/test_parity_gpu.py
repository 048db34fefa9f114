"""CUDA path vs the CPU oracle on seeded inputs: every element type and
operator, sizes around every tile edge, unaligned offsets, strided and
transposed views, reverse and exclusive scans, arg-reductions with ties.
Integers and argmax indices bit-exact; f32 within 1e-5*sum|x|, f64 within
1e-12*sum|x| (the tolerances the north star states)."""
import numpy as np
import pytest

from hephaestus_b200 import (CudaAxisReductionOps, CudaFullReductionOps, CudaScanOps, Layout,
                             MaxOp, MinOp, ProdOp, StridedView, SumOp)
from hephaestus_b200.core import CumProdOp, CumSumOp

pytestmark = pytest.mark.gpu

DTYPES = [np.float32, np.float64, np.uint32, np.int32, np.int64]
OPS = {0: SumOp, 1: ProdOp, 2: MinOp, 3: MaxOp}
SCAN_TILE = {4: 4096, 8: 2048}
EDGE_SIZES = [0, 1, 2, 3, 31, 32, 33, 255, 256, 257, 1023, 1025, 2047, 2049, 4095, 4096, 4097,
              8191, 8193, 65537, 1 << 20, (1 << 20) + 3]


def rand(dt, n, rng, prod=False):
    if np.dtype(dt).kind == "f":
        if prod:  # bounded products: rare factors of 2 and 1/2 among +-1
            return rng.choice([0.5, 1.0, 2.0, -1.0], p=[0.01, 0.49, 0.01, 0.49], size=n).astype(dt)
        return rng.uniform(-1, 1, size=n).astype(dt)
    if prod:
        return rng.choice([1, 3, 5, 7], size=n).astype(dt)  # odd: products never collapse to 0
    lo = 0 if np.dtype(dt).kind == "u" else -1000
    return rng.integers(lo, 1000, size=n).astype(dt)


def tol(dt, x):
    s = float(np.abs(x.astype(np.float64)).sum()) if x.size else 0.0
    return {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}.get(np.dtype(dt), 0) * max(s, 1.0)


def assert_close(got, want, dt, x):
    if np.dtype(dt).kind == "f":
        np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=0,
                                   atol=tol(dt, x))
    else:
        np.testing.assert_array_equal(got, want)


# ----------------------------------------------------------- full reductions


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_full_reduction_edges(device, oracle, dt, op):
    rng = np.random.default_rng(op * 10 + DTYPES.index(dt))
    ops = CudaFullReductionOps()
    for n in EDGE_SIZES:
        if op == 1 and n > 4096:
            continue
        x = rand(dt, n, rng, prod=op == 1)
        buf = device.upload(x) if n else device.alloc_zeroed(dt, 0)
        out = device.alloc_zeroed(dt, 1)
        ops.reduce_full_into(OPS[op], device, StridedView(buf, Layout.c_contiguous([n])),
                             StridedView(out, Layout.c_contiguous([1])))
        want = oracle.reduce_full(x, [n], op=op)
        assert_close(device.download_owned(out), np.array([want], dtype=dt), dt, x)


@pytest.mark.parametrize("dt", [np.float32, np.uint32, np.int64])
def test_full_reduction_unaligned_and_strided(device, oracle, dt):
    rng = np.random.default_rng(3)
    x = rand(dt, 100003, rng)
    buf = device.upload(x)
    ops = CudaFullReductionOps()
    out = device.alloc_zeroed(dt, 4)
    views = [
        Layout.try_new([99990], [1], 5),          # unaligned dense
        Layout.try_new([333, 300], [300, 1], 3),  # dense rank-2 with offset
        Layout.try_new([300, 333], [1, 300], 1),  # transposed
        Layout.try_new([50000], [2], 1),          # stride 2
        Layout.try_new([1000], [-7], 7000),       # negative stride
        Layout.try_new([10, 10, 10, 10], [10000, 1000, 10, 1], 17),
    ]
    for v in views:
        ops.reduce_full_into(SumOp, device, StridedView(buf, v), StridedView(out, Layout.try_new([1], [1], 2)))
        want = oracle.reduce_full(x, v.shape, v.strides, v.offset)
        got = device.download_owned(out)[2:3]
        assert_close(got, np.array([want], dtype=dt), dt, x)


def test_widening_sums(device, oracle):
    rng = np.random.default_rng(11)
    x = rng.integers(-2**31, 2**31 - 1, size=300007, dtype=np.int64).astype(np.int32)
    buf = device.upload(x)
    out = device.alloc_zeroed(np.int64, 1)
    CudaFullReductionOps().reduce_full_into(SumOp, device, StridedView(buf, Layout.c_contiguous([x.size])),
                                            StridedView(out, Layout.c_contiguous([1])))
    assert device.download_owned(out)[0] == int(x.astype(np.int64).sum())
    assert oracle.reduce_full(x, [x.size], out_dtype=np.int64) == int(x.astype(np.int64).sum())
    f = rng.uniform(-1, 1, size=300007).astype(np.float32)
    fb = device.upload(f)
    fo = device.alloc_zeroed(np.float64, 1)
    CudaFullReductionOps().reduce_full_into(SumOp, device, StridedView(fb, Layout.c_contiguous([f.size])),
                                            StridedView(fo, Layout.c_contiguous([1])))
    assert abs(device.download_owned(fo)[0] - f.astype(np.float64).sum()) <= 1e-12 * np.abs(f).sum()


# ------------------------------------------------------------ axis reductions

AXIS_SHAPES = [(1, 1), (3, 4), (7, 33), (33, 7), (5, 4097), (4097, 5), (2, 70000), (70000, 2),
               (129, 1024), (1024, 129), (1, 300000), (300000, 1)]


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("op", [0, 2, 3, 4])
def test_axis_reduction_shapes(device, oracle, dt, op):
    rng = np.random.default_rng(op + 7 * DTYPES.index(dt))
    ops = CudaAxisReductionOps()
    for shape in AXIS_SHAPES:
        x = rand(dt, shape[0] * shape[1], rng)
        buf = device.upload(x)
        for axis in (0, 1):
            oshape = list(shape)
            oshape[axis] = 1
            out = device.alloc_zeroed(dt, oshape[0] * oshape[1])
            ol = Layout.c_contiguous(oshape)
            if op == 4:
                ops.mean_axis_into(device, StridedView(buf, Layout.c_contiguous(shape)), axis, StridedView(out, ol))
            else:
                ops.reduce_axis_into(OPS[op], device, StridedView(buf, Layout.c_contiguous(shape)), axis,
                                     StridedView(out, ol))
            want = oracle.reduce_axis(x, shape, axis, op=op)
            got = device.download_owned(out)
            if op == 4 and np.dtype(dt).kind == "f":
                np.testing.assert_allclose(got, want, rtol=1e-5 if dt == np.float32 else 1e-12, atol=1e-6)
            else:
                assert_close(got, want, dt, x)


@pytest.mark.parametrize("dt", [np.float32, np.int32])
def test_axis_prod_and_strided_views(device, oracle, dt):
    rng = np.random.default_rng(5)
    x = rand(dt, 64 * 130 + 3, rng, prod=True)
    buf = device.upload(x)
    ops = CudaAxisReductionOps()
    for lay in [Layout.try_new([64, 130], [130, 1], 3), Layout.try_new([130, 64], [1, 130], 0),
                Layout.try_new([32, 130], [260, 1], 1), Layout.try_new([64, 65], [130, 2], 0)]:
        for axis in (0, 1):
            for op in (1, 0, 3):
                oshape = list(lay.shape)
                oshape[axis] = 1
                out = device.alloc_zeroed(dt, oshape[0] * oshape[1])
                ops.reduce_axis_into(OPS[op], device, StridedView(buf, lay), axis,
                                     StridedView(out, Layout.c_contiguous(oshape)))
                want = oracle.reduce_axis(x, lay.shape, axis, op=op, in_strides=lay.strides,
                                          in_offset=lay.offset)
                got = device.download_owned(out)
                if op == 1 and np.dtype(dt).kind == "f":
                    np.testing.assert_allclose(got, want, rtol=1e-5)
                else:
                    assert_close(got, want, dt, x)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("op", [3, 2])
def test_arg_reduction_ties(device, oracle, dt, op):
    rng = np.random.default_rng(17 + op)
    ops = CudaAxisReductionOps()
    for shape in [(3, 4), (33, 129), (5, 5000), (5000, 5), (1, 100000), (257, 4096)]:
        # few distinct values: many exact ties
        x = rng.integers(0, 7, size=shape[0] * shape[1]).astype(dt)
        buf = device.upload(x)
        for axis in (0, 1):
            oshape = list(shape)
            oshape[axis] = 1
            n = oshape[0] * oshape[1]
            vals, idx = device.alloc_zeroed(dt, n), device.alloc_zeroed(np.uint32, n)
            ol = Layout.c_contiguous(oshape)
            fn = ops.argmax_axis_into if op == 3 else ops.argmin_axis_into
            fn(device, StridedView(buf, Layout.c_contiguous(shape)), axis, StridedView(vals, ol), StridedView(idx, ol))
            wv, wi = oracle.arg_reduce_axis(x, shape, axis, op=op)
            np.testing.assert_array_equal(device.download_owned(idx), wi)
            np.testing.assert_array_equal(device.download_owned(vals), wv)


def test_argmax_infinities(device, oracle):
    x = np.full(64 * 40, -np.inf, dtype=np.float32)
    x[5 * 40 + 7] = -1.0
    buf = device.upload(x)
    ops = CudaAxisReductionOps()
    vals, idx = device.alloc_zeroed(np.float32, 64), device.alloc_zeroed(np.uint32, 64)
    ol = Layout.c_contiguous([64, 1])
    ops.argmax_axis_into(device, StridedView(buf, Layout.c_contiguous([64, 40])), 1, StridedView(vals, ol),
                         StridedView(idx, ol))
    wv, wi = oracle.arg_reduce_axis(x, [64, 40], 1)
    np.testing.assert_array_equal(device.download_owned(idx), wi)
    np.testing.assert_array_equal(device.download_owned(vals), wv)


# --------------------------------------------------------------------- scans


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("exclusive", [False, True])
@pytest.mark.parametrize("reverse", [False, True])
def test_scan_1d_edges(device, oracle, dt, exclusive, reverse):
    rng = np.random.default_rng(DTYPES.index(dt) * 4 + 2 * exclusive + reverse)
    tile = SCAN_TILE[np.dtype(dt).itemsize]
    sizes = sorted(set(EDGE_SIZES + [tile - 1, tile, tile + 1, 2 * tile - 1, 2 * tile + 1,
                                     33 * tile + 5, 1000 * tile]))
    ops = CudaScanOps()
    for n in sizes:
        x = rand(dt, n, rng)
        buf = device.upload(x) if n else device.alloc_zeroed(dt, 0)
        out = device.alloc_zeroed(dt, n)
        ops.scan_axis_into(CumSumOp, device, StridedView(buf, Layout.c_contiguous([n])), 0, int(reverse),
                           StridedView(out, Layout.c_contiguous([n])), exclusive=exclusive)
        want = oracle.scan_axis(x, [n], 0, reverse=reverse, exclusive=exclusive)
        got = device.download_owned(out)
        if np.dtype(dt).kind == "f":
            # float scans: |err| <= tol * sum|x| per element (ADR 0009 bound)
            np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=0,
                                       atol=tol(dt, x))
        else:
            np.testing.assert_array_equal(got, want, err_msg=f"n={n}")


@pytest.mark.parametrize("dt", [np.uint32, np.int64, np.float32])
def test_scan_prod_and_unaligned(device, oracle, dt):
    rng = np.random.default_rng(99)
    x = rand(dt, 50001, rng, prod=True)
    buf = device.upload(x)
    out = device.alloc_zeroed(dt, 50001)
    ops = CudaScanOps()
    for off_in, off_out, n in [(0, 0, 50001), (1, 0, 50000), (3, 5, 49990), (2, 2, 40000)]:
        for rev in (False, True):
            ops.scan_axis_into(CumProdOp, device, StridedView(buf, Layout.try_new([n], [1], off_in)), 0, int(rev),
                               StridedView(out, Layout.try_new([n], [1], off_out)))
            want = oracle.scan_axis(x, [n], 0, op=1, reverse=rev, in_offset=off_in)
            got = device.download_owned(out)[off_out:off_out + n]
            if np.dtype(dt).kind == "f":
                np.testing.assert_allclose(got, want[:n], rtol=1e-5)
            else:
                np.testing.assert_array_equal(got, want[:n])


@pytest.mark.parametrize("dt", [np.uint32, np.int32, np.float64])
def test_scan_2d_both_axes(device, oracle, dt):
    rng = np.random.default_rng(5)
    ops = CudaScanOps()
    # (5, 70001), (4, 65540): lines of 9 look-back tiles (position-major numbering), unaligned and aligned
    # rows; (300, 4096): rows of exactly one 16 KiB tile.
    for shape in [(3, 4), (7, 5000), (5000, 7), (3, 20000), (64, 4097), (2, 513), (5, 70001), (4, 65540),
                  (24, 40960), (300, 4096)]:
        x = rand(dt, shape[0] * shape[1], rng)
        buf = device.upload(x)
        for axis in (0, 1):
            for rev in (False, True):
                for exc in (False, True):
                    out = device.alloc_zeroed(dt, x.size)
                    ops.scan_axis_into(CumSumOp, device, StridedView(buf, Layout.c_contiguous(shape)), axis, int(rev),
                                       StridedView(out, Layout.c_contiguous(shape)), exclusive=exc)
                    want = oracle.scan_axis(x, shape, axis, reverse=rev, exclusive=exc)
                    got = device.download_owned(out)
                    if np.dtype(dt).kind == "f":
                        np.testing.assert_allclose(got, want, rtol=0, atol=1e-12 * max(1, np.abs(x).sum()))
                    else:
                        np.testing.assert_array_equal(got, want, err_msg=f"{shape} axis={axis} rev={rev} exc={exc}")


def test_scan_transposed_output(device, oracle):
    rng = np.random.default_rng(8)
    x = rand(np.int32, 300 * 500, rng)
    buf = device.upload(x)
    out = device.alloc_zeroed(np.int32, x.size)
    lin = Layout.c_contiguous([300, 500])
    lout = Layout.try_new([300, 500], [1, 300], 0)
    CudaScanOps().scan_axis_into(CumSumOp, device, StridedView(buf, lin), 1, 0, StridedView(out, lout))
    want = oracle.scan_axis(x, [300, 500], 1, out_strides=[1, 300])
    np.testing.assert_array_equal(device.download_owned(out), want)


def test_repeated_scans_reuse_workspace(device, oracle):
    """Many scans in a row on one stream: the epoch-tagged status and the
    tile counter stay consistent (no clearing between calls)."""
    rng = np.random.default_rng(1)
    ops = CudaScanOps()
    for k in range(40):
        n = int(rng.integers(1, 300000))
        dt = [np.uint32, np.int64][k % 2]
        x = rand(dt, n, rng)
        buf, out = device.upload(x), device.alloc_zeroed(dt, n)
        ops.scan_axis_into(CumSumOp, device, StridedView(buf, Layout.c_contiguous([n])), 0, k % 3 == 0,
                           StridedView(out, Layout.c_contiguous([n])), exclusive=k % 5 == 0)
        want = oracle.scan_axis(x, [n], 0, reverse=k % 3 == 0, exclusive=k % 5 == 0)
        np.testing.assert_array_equal(device.download_owned(out), want)
    device.synchronize()  # no device-side error (look-back timeout) was raised


@pytest.mark.parametrize("dt", DTYPES)
def test_scan_two_pass_lines(device, oracle, dt):
    """Single lines of 640+ look-back tiles below the chunked kernel's minimum
    take the two-pass scan (tile totals, then each tile scanned with the fold
    of the totals before it): 6 M 4-byte elements, 2.8-2.9 M 8-byte ones;
    aligned and misaligned views, both directions, inclusive and exclusive."""
    rng = np.random.default_rng(91 + DTYPES.index(dt))
    ops = CudaScanOps()
    for n, off in [(6_000_001, 0), (2_800_003, 0), (2_900_001, 1), (5_500_000, 3)]:
        x = rand(dt, n + off, rng)
        buf = device.upload(x)
        for rev in (False, True):
            for exc in (False, True):
                out = device.alloc_zeroed(dt, n)
                ops.scan_axis_into(CumSumOp, device, StridedView(buf, Layout.try_new([n], [1], off)), 0, int(rev),
                                   StridedView(out, Layout.c_contiguous([n])), exclusive=exc)
                want = oracle.scan_axis(x, [n], 0, reverse=rev, exclusive=exc, in_offset=off)
                assert_close(device.download_owned(out), want[:n], dt, x[off:])


def _check_rows_scan(device, oracle, dt, shape, ld=None, op=CumSumOp, seed=77):
    """Row scans (axis 1) of a [rows x cols] view with row stride `ld` into a
    dense output, every direction / inclusive-exclusive pair, against the
    oracle."""
    rows, cols = shape
    ld = ld or cols
    rng = np.random.default_rng(seed)
    x = rand(dt, rows * ld, rng, prod=op is CumProdOp)
    buf, out = device.upload(x), device.alloc_zeroed(dt, rows * cols)
    il, ol = Layout.try_new([rows, cols], [ld, 1], 0), Layout.c_contiguous([rows, cols])
    for rev in (False, True):
        for exc in (False, True):
            CudaScanOps().scan_axis_into(op, device, StridedView(buf, il), 1, int(rev), StridedView(out, ol),
                                         exclusive=exc)
            want = oracle.scan_axis(x, [rows, cols], 1, op=1 if op is CumProdOp else 0, reverse=rev,
                                    exclusive=exc, in_strides=[ld, 1])
            got = device.download_owned(out)
            if np.dtype(dt).kind == "f":
                np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=0,
                                           atol=tol(dt, x), err_msg=f"rev={rev} exc={exc}")
            else:
                np.testing.assert_array_equal(got, want, err_msg=f"rev={rev} exc={exc}")
    device.synchronize()  # no device-side error (wait timeout) was raised


@pytest.mark.parametrize("dt,shape", [(np.uint32, (2, 33_554_444)), (np.int64, (2, 16_777_220)),
                                      (np.uint32, (3, 7_500_000)), (np.uint32, (16, 1 << 21)),
                                      (np.float32, (4, 3_000_020)), (np.int32, (64, 1 << 17))])
def test_chunked_scan_multiline(device, oracle, dt, shape, monkeypatch):
    """Several long lines take the chunked kernel in ONE launch: every line's
    parts carry their own running prefix and each line starts from the
    identity (nothing leaks from the line before).  Line lengths that the part
    does not divide give every line a ragged last part.  The threshold knob is
    lowered for the shorter shapes so that they take the kernel too."""
    monkeypatch.setenv("HEPH_SCAN_MULTI_CHUNKED_BYTES", str(1 << 19))
    _check_rows_scan(device, oracle, dt, shape)


@pytest.mark.parametrize("dt,shape,ld", [(np.uint32, (5, 1_000_004), 1_000_008),
                                         (np.int64, (40, 100_002), 100_004),
                                         (np.uint32, (300, 20_000), 20_000),
                                         (np.float64, (7, 700_002), 700_004)])
def test_chunked_scan_multiline_many_chunks(device, oracle, dt, shape, ld, monkeypatch):
    """One chunked CTA per SM (148 parts per chunk) and the threshold lowered:
    lines begin and end in the middle of chunks, a line spans several chunks
    or several lines share one, and the row stride differs from the row
    length (input lines padded, output dense).  Rows stay 16-byte aligned
    (the kernel's condition) while the part does not divide them."""
    monkeypatch.setenv("HEPH_SCAN_CHUNK_CTAS", "1")
    monkeypatch.setenv("HEPH_SCAN_MULTI_CHUNKED_BYTES", "1")
    _check_rows_scan(device, oracle, dt, shape, ld=ld, seed=78)


def test_chunked_scan_multiline_prod(device, oracle, monkeypatch):
    monkeypatch.setenv("HEPH_SCAN_CHUNK_CTAS", "1")
    monkeypatch.setenv("HEPH_SCAN_MULTI_CHUNKED_BYTES", "1")
    _check_rows_scan(device, oracle, np.uint32, (9, 700_004), op=CumProdOp, seed=79)


@pytest.fixture
def small_parts(monkeypatch):
    """One chunked-scan CTA per SM (148 parts of 16 KiB per chunk), so that a
    few million elements span many chunks and every size below takes the
    chunked kernel (the launcher reads the knob at every call)."""
    monkeypatch.setenv("HEPH_SCAN_CHUNK_CTAS", "1")
    yield


@pytest.mark.parametrize("dt", DTYPES)
def test_chunked_scan_many_chunks(device, oracle, dt, small_parts):
    rng = np.random.default_rng(123 + DTYPES.index(dt))
    ops = CudaScanOps()
    for n in [6_000_000, 6_062_080, 9_000_001]:
        x = rand(dt, n, rng)
        buf, out = device.upload(x), device.alloc_zeroed(dt, n)
        for rev in (False, True):
            for exc in (False, True):
                ops.scan_axis_into(CumSumOp, device, StridedView(buf, Layout.c_contiguous([n])), 0, int(rev),
                                   StridedView(out, Layout.c_contiguous([n])), exclusive=exc)
                want = oracle.scan_axis(x, [n], 0, reverse=rev, exclusive=exc)
                got = device.download_owned(out)
                if np.dtype(dt).kind == "f":
                    np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=0,
                                               atol=tol(dt, x))
                else:
                    np.testing.assert_array_equal(got, want, err_msg=f"n={n} rev={rev} exc={exc}")
    device.synchronize()


def test_chunked_scan_prod_u32(device, oracle, small_parts):
    rng = np.random.default_rng(5)
    n = 8_000_000
    x = rand(np.uint32, n, rng, prod=True)
    buf, out = device.upload(x), device.alloc_zeroed(np.uint32, n)
    CudaScanOps().scan_axis_into(CumProdOp, device, StridedView(buf, Layout.c_contiguous([n])), 0, 0,
                                 StridedView(out, Layout.c_contiguous([n])))
    np.testing.assert_array_equal(device.download_owned(out), oracle.scan_axis(x, [n], 0, op=1))


@pytest.mark.parametrize("dt", [np.uint32, np.int64])
def test_lookback_scan_long_line(device, oracle, dt, monkeypatch):
    """The look-back kernel on a long line (the chunked kernel switched off)."""
    monkeypatch.setenv("HEPH_SCAN_NO_CHUNKED", "1")
    rng = np.random.default_rng(77)
    n = 12_000_003
    x = rand(dt, n, rng)
    buf, out = device.upload(x), device.alloc_zeroed(dt, n)
    for rev, exc in [(False, True), (True, False)]:
        CudaScanOps().scan_axis_into(CumSumOp, device, StridedView(buf, Layout.c_contiguous([n])), 0, int(rev),
                                     StridedView(out, Layout.c_contiguous([n])), exclusive=exc)
        np.testing.assert_array_equal(device.download_owned(out),
                                      oracle.scan_axis(x, [n], 0, reverse=rev, exclusive=exc))
    device.synchronize()


@pytest.mark.parametrize("dt,exc", [(np.uint32, True), (np.int32, False), (np.float32, False), (np.int64, True)])
def test_scan_host_pipeline(device, oracle, dt, exc):
    """heph_scan_host: chunked, transfer-overlapped scan of host arrays."""
    rng = np.random.default_rng(31)
    ops = CudaScanOps()
    for n, chunk in [(1, 0), (1000, 7), (100_003, 4096), (3_000_001, 1 << 20), (5_000_000, 0)]:
        x = rand(dt, n, rng)
        y = np.empty_like(x)
        ops.scan_host(CumSumOp, device, x, y, exclusive=exc, chunk_elems=chunk)
        want = oracle.scan_axis(x, [n], 0, exclusive=exc)
        if np.dtype(dt).kind == "f":
            np.testing.assert_allclose(y.astype(np.float64), want.astype(np.float64), rtol=0, atol=tol(dt, x))
        else:
            np.testing.assert_array_equal(y, want, err_msg=f"n={n} chunk={chunk}")


@pytest.mark.parametrize("dt,acc,rop", [(np.int32, np.int64, "sum"), (np.uint32, np.uint32, "max"),
                                        (np.float32, np.float64, "sum"), (np.int64, np.int64, "min")])
def test_scan_reduce_host_pipeline(device, oracle, dt, acc, rop):
    """heph_scan_reduce_host: the host-buffer scan plus a full reduction of the
    same input, chunk by chunk (ragged chunks, the ramp pieces, one chunk)."""
    from hephaestus_b200.core import MaxOp, MinOp
    op = {"sum": SumOp, "max": MaxOp, "min": MinOp}[rop]
    rng = np.random.default_rng(32)
    ops = CudaScanOps()
    for n, chunk in [(0, 0), (1, 0), (1000, 7), (100_003, 4096), (5_000_000, 1 << 20), (3_000_001, 0)]:
        x = rand(dt, n, rng)
        y = np.empty_like(x)
        got = ops.scan_reduce_host(CumSumOp, device, x, y, op, acc_dtype=acc, chunk_elems=chunk)
        want_y = oracle.scan_axis(x, [n], 0) if n else y
        want = oracle.reduce_full(x, [n], op=op.code, out_dtype=acc) if n else None
        if np.dtype(dt).kind == "f":
            np.testing.assert_allclose(y.astype(np.float64), want_y.astype(np.float64), rtol=0, atol=tol(dt, x))
            if n:
                assert abs(float(got) - float(want)) <= tol(dt, x), (n, chunk)
        else:
            np.testing.assert_array_equal(y, want_y, err_msg=f"n={n} chunk={chunk}")
            if n:
                assert got == want, (n, chunk)
        if n == 0:
            ident = {"sum": 0, "max": 0, "min": np.iinfo(np.int64).max}[rop]
            assert got == ident


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("map_kind", [0, 1, 2, 3, 4])
def test_map_reduction_parity(device, oracle, dt, map_kind):
    import hephaestus_b200.seams as S
    if map_kind == 3 and np.dtype(dt).kind != "f":
        pytest.skip("norm_l2 is defined for floating-point types")
    rng = np.random.default_rng(40 + map_kind)
    for n in [0, 1, 33, 4097, 1_000_003]:
        x, y = rand(dt, n, rng), rand(dt, n, rng)
        xb = device.upload(x) if n else device.alloc_zeroed(dt, 0)
        yb = device.upload(y) if n else device.alloc_zeroed(dt, 0)
        out = device.alloc_zeroed(dt, 1)
        views = [(Layout.c_contiguous([n]), Layout.c_contiguous([n]))]
        if n > 8:
            views.append((Layout.try_new([n // 2], [2], 1), Layout.try_new([n // 2], [-2], n - 1)))
        for la, lb in views:
            S._map_call(device, map_kind, StridedView(xb, la), StridedView(yb, lb) if map_kind == 0 else None,
                        StridedView(out, Layout.c_contiguous([1])))
            # Floats: the oracle's fold in f64 (a sequential f32 fold of 10^6
            # positive terms is itself off by ~1e-5 relative).
            xr, yr = (x.astype(np.float64), y.astype(np.float64)) if np.dtype(dt).kind == "f" and map_kind != 4 else (x, y)
            want = oracle.map_reduce(map_kind, xr, la.shape, la.strides, la.offset,
                                     b=yr if map_kind == 0 else None, b_strides=lb.strides, b_offset=lb.offset)
            got = device.download_owned(out)[0]
            if np.dtype(dt).kind == "f":
                scale = float(np.abs(x.astype(np.float64) * (np.abs(y) if map_kind == 0 else 1)).sum()) \
                    if map_kind != 3 else float(np.sqrt((x.astype(np.float64) ** 2).sum()))
                t = {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}[np.dtype(dt)] * max(scale, 1.0)
                assert abs(float(got) - float(want)) <= t, (n, la, got, want)
            else:
                assert got == want, (n, la)


@pytest.mark.parametrize("dt", [np.float32, np.int32, np.float64])
def test_permuted_dense_views_full_reduction(device, oracle, dt):
    """Transposed, permuted and reversed views of a dense block reduce through
    the contiguous fast path and still match the oracle."""
    import hephaestus_b200.seams as S
    rng = np.random.default_rng(9)
    x = rand(dt, 2 * 3 * 5 * 7 * 64 + 5, rng)
    buf = device.upload(x)
    out = device.alloc_zeroed(dt, 1)
    views = [Layout.try_new([64, 210], [1, 64], 5), Layout.try_new([13440], [-1], 13444),
             Layout.try_new([7, 5, 3, 128], [1, 7, 35, 105], 5), Layout.try_new([210, 64], [-64, 1], 5 + 209 * 64)]
    for v in views:
        for op, code in [(SumOp, 0), (MaxOp, 3)]:
            CudaFullReductionOps().reduce_full_into(op, device, StridedView(buf, v),
                                                    StridedView(out, Layout.c_contiguous([1])))
            want = oracle.reduce_full(x, v.shape, v.strides, v.offset, op=code)
            assert_close(device.download_owned(out), np.array([want], dtype=dt), dt, x)
        S._map_call(device, 2, StridedView(buf, v), None, StridedView(out, Layout.c_contiguous([1])))
        want = oracle.map_reduce(2, x.astype(np.float64) if np.dtype(dt).kind == "f" else x, v.shape, v.strides, v.offset)
        got = device.download_owned(out)[0]
        if np.dtype(dt).kind == "f":
            assert abs(float(got) - float(want)) <= 1e-5 * float(np.abs(x).sum())
        else:
            assert got == want


# Gapped N-D views: sub-blocks with row gaps (16-byte aligned inner runs and
# not), rank 3 and 4 with mixed-sign strides, a broadcast (stride-0) dim, a
# diagonal.  They take the division-free walk kernels.
def gapped_views(n_storage):
    views = [
        Layout.try_new([300, 256], [260, 1], 4),                 # aligned rows with gaps
        Layout.try_new([300, 255], [257, 1], 3),                 # unaligned rows
        Layout.try_new([7, 33, 64], [4000, 100, 1], 8),          # rank 3, aligned runs
        Layout.try_new([3, 5, 7, 11], [3000, -500, 60, 2], 2100),  # rank 4, negative and non-unit
        Layout.try_new([100, 64], [0, 1], 16),                   # broadcast rows
        Layout.try_new([64, 100], [1, 0], 16),                   # broadcast inner dim
        Layout.try_new([300], [301], 0),                         # diagonal
        Layout.try_new([2, 9, 1, 130], [40000, 4096, 7, 3], 12),  # unit dim dropped, stride-3 rows
        # Unaligned unit-stride runs (the row-run kernels):
        Layout.try_new([90, 1001], [1003, 1], 5),
        Layout.try_new([77, 130], [131, 1], 2),
        Layout.try_new([1000, 15], [16, 1], 3),                  # one-element gaps, rows straddle vectors
        Layout.try_new([200, 250], [-251, 1], 199 * 251 + 9),    # reversed rows
        Layout.try_new([10, 9000], [9001, 1], 3),                # runs of several segments
        Layout.try_new([3, 4, 300], [20011, 1003, 1], 7),        # rank 3, unaligned runs
    ]
    for v in views:
        lo = v.offset + sum(min(0, (s - 1) * st) for s, st in zip(v.shape, v.strides))
        hi = v.offset + sum(max(0, (s - 1) * st) for s, st in zip(v.shape, v.strides))
        assert 0 <= lo and hi < n_storage, v
    return views


@pytest.mark.parametrize("dt", DTYPES)
def test_gapped_views_full_reduction(device, oracle, dt):
    rng = np.random.default_rng(77)
    n = 100_000
    ops = CudaFullReductionOps()
    out = device.alloc_zeroed(dt, 1)
    for code, op in OPS.items():
        x = rand(dt, n, rng, prod=code == 1)
        buf = device.upload(x)
        for v in gapped_views(n):
            ops.reduce_full_into(op, device, StridedView(buf, v), StridedView(out, Layout.c_contiguous([1])))
            want = oracle.reduce_full(x, v.shape, v.strides, v.offset, op=code)
            assert_close(device.download_owned(out), np.array([want], dtype=dt), dt, x)


def test_gapped_views_widening(device, oracle):
    rng = np.random.default_rng(78)
    ops = CudaFullReductionOps()
    for src, dst in [(np.int32, np.int64), (np.float32, np.float64)]:
        x = (rng.integers(-2**31, 2**31 - 1, size=100_000, dtype=np.int64).astype(np.int32) if src == np.int32
             else rng.uniform(-1, 1, size=100_000).astype(np.float32))
        buf = device.upload(x)
        out = device.alloc_zeroed(dst, 1)
        for v in gapped_views(x.size):
            ops.reduce_full_into(SumOp, device, StridedView(buf, v), StridedView(out, Layout.c_contiguous([1])))
            want = oracle.reduce_full(x, v.shape, v.strides, v.offset, out_dtype=dst)
            got = device.download_owned(out)[0]
            if src == np.int32:
                assert got == want, v
            else:
                assert abs(float(got) - float(want)) <= 1e-12 * float(np.abs(x).sum()), v


def test_gapped_view_large_and_wide_inner_dim(device):
    """A broadcast inner dim beyond 32-bit coordinates (2 x (2^31 + 5) logical
    elements over 2 stored ones) and a large gapped sub-block, checked by closed
    forms."""
    x = np.array([3, 4], dtype=np.uint32)
    buf = device.upload(x)
    out = device.alloc_zeroed(np.uint32, 1)
    inner = (1 << 31) + 5
    v = Layout.try_new([2, inner], [1, 0], 0)
    CudaFullReductionOps().reduce_full_into(SumOp, device, StridedView(buf, v), StridedView(out, Layout.c_contiguous([1])))
    assert int(device.download_owned(out)[0]) == (7 * inner) % (1 << 32)
    CudaFullReductionOps().reduce_full_into(MaxOp, device, StridedView(buf, v), StridedView(out, Layout.c_contiguous([1])))
    assert int(device.download_owned(out)[0]) == 4
    # 8192 x 8000 of an 8192 x 8192 u32 matrix: every element i*8192+j, j<8000.
    rows, cols, ld = 8192, 8000, 8192
    big = np.arange(rows * ld, dtype=np.uint64).astype(np.uint32)
    bb = device.upload(big)
    CudaFullReductionOps().reduce_full_into(SumOp, device, StridedView(bb, Layout.try_new([rows, cols], [ld, 1], 0)),
                                            StridedView(out, Layout.c_contiguous([1])))
    i = np.arange(rows, dtype=np.uint64)
    want = (cols * i * ld).sum() + rows * (cols * (cols - 1) // 2)
    assert int(device.download_owned(out)[0]) == int(want) % (1 << 32)


@pytest.mark.parametrize("dt,acc,rop", [(np.int32, np.int64, "sum"), (np.uint32, np.uint32, "max"),
                                        (np.float32, np.float64, "sum"), (np.int64, np.int64, "min")])
def test_scan_reduce_host_pipeline(device, oracle, dt, acc, rop):
    """heph_scan_reduce_host: the host-buffer scan plus a full reduction of the
    same input, chunk by chunk (ragged chunks, the ramp pieces, one chunk)."""
    from hephaestus_b200.core import MaxOp, MinOp
    op = {"sum": SumOp, "max": MaxOp, "min": MinOp}[rop]
    rng = np.random.default_rng(32)
    ops = CudaScanOps()
    for n, chunk in [(0, 0), (1, 0), (1000, 7), (100_003, 4096), (5_000_000, 1 << 20), (3_000_001, 0)]:
        x = rand(dt, n, rng)
        y = np.empty_like(x)
        got = ops.scan_reduce_host(CumSumOp, device, x, y, op, acc_dtype=acc, chunk_elems=chunk)
        want_y = oracle.scan_axis(x, [n], 0) if n else y
        want = oracle.reduce_full(x, [n], op=op.code, out_dtype=acc) if n else None
        if np.dtype(dt).kind == "f":
            np.testing.assert_allclose(y.astype(np.float64), want_y.astype(np.float64), rtol=0, atol=tol(dt, x))
            if n:
                assert abs(float(got) - float(want)) <= tol(dt, x), (n, chunk)
        else:
            np.testing.assert_array_equal(y, want_y, err_msg=f"n={n} chunk={chunk}")
            if n:
                assert got == want, (n, chunk)
        if n == 0:
            ident = {"sum": 0, "max": 0, "min": np.iinfo(np.int64).max}[rop]
            assert got == ident


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("map_kind", [0, 1, 2, 3, 4])
def test_gapped_views_map_reduction(device, oracle, dt, map_kind):
    import hephaestus_b200.seams as S
    if map_kind == 3 and np.dtype(dt).kind != "f":
        pytest.skip("norm_l2 is defined for floating-point types")
    rng = np.random.default_rng(80 + map_kind)
    n = 100_000
    x, y = rand(dt, n, rng), rand(dt, n, rng)
    xb, yb = device.upload(x), device.upload(y)
    out = device.alloc_zeroed(dt, 1)
    views = gapped_views(n)
    pairs = [(v, v) for v in views]
    # Dot products of differently laid out operands: a sub-block against the
    # transpose of another, a broadcast against a reversed run, both transposed.
    pairs += [(Layout.try_new([300, 256], [260, 1], 4), Layout.try_new([300, 256], [1, 300], 7)),
              (Layout.try_new([100, 64], [0, 1], 16), Layout.try_new([100, 64], [-64, -1], 6399 + 20)),
              (Layout.try_new([64, 210], [1, 64], 8), Layout.try_new([64, 210], [1, 64], 12))]
    for la, lb in pairs:
        S._map_call(device, map_kind, StridedView(xb, la), StridedView(yb, lb) if map_kind == 0 else None,
                    StridedView(out, Layout.c_contiguous([1])))
        xr, yr = (x.astype(np.float64), y.astype(np.float64)) if np.dtype(dt).kind == "f" and map_kind != 4 else (x, y)
        want = oracle.map_reduce(map_kind, xr, la.shape, la.strides, la.offset,
                                 b=yr if map_kind == 0 else None, b_strides=lb.strides, b_offset=lb.offset)
        got = device.download_owned(out)[0]
        if np.dtype(dt).kind == "f":
            t = {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}[np.dtype(dt)]
            # Bounds the view's terms: no view here repeats an element more
            # than 100 times, and the buffers hold 10^5 terms of magnitude <= 1.
            scale = float(np.abs(x.astype(np.float64) * (np.abs(y) if map_kind == 0 else 1)).sum()) \
                if map_kind != 3 else float(np.sqrt((x.astype(np.float64) ** 2).sum()) * 10)
            assert abs(float(got) - float(want)) <= t * max(scale, 1.0), (la, lb, got, want)
        else:
            assert got == want, (la, lb)


# Batches: runs of dense full reductions of one operator and type are fused
# into one kernel; the results must equal running the items in order.
@pytest.mark.parametrize("dt", [np.float32, np.int32, np.uint32, np.float64, np.int64])
def test_fused_batch_of_full_reductions(device, oracle, dt):
    import hephaestus_b200.seams as S
    rng = np.random.default_rng(90)
    sizes = [1, 3, 31, 4096, 4099, 100_003, 1 << 20, 2_000_001, 7, 65536]
    xs = [rand(dt, n, rng) for n in sizes]
    bufs = [device.upload(x) for x in xs]
    out = device.alloc_zeroed(dt, 3 * len(sizes))
    ops = CudaFullReductionOps()
    items, want = [], []
    # run 1: sums over every buffer (unaligned offsets on some), run 2: max,
    # run 3: a permuted dense view and a reversed one (dense blocks).
    for k, (x, b) in enumerate(zip(xs, bufs)):
        off = k % 3 if x.size > 3 else 0
        lay = Layout.try_new([x.size - off], [1], off)
        items.append(ops.prepare_reduce_full(SumOp, device, StridedView(b, lay),
                                             StridedView(out, Layout.try_new([1], [1], k))))
        want.append((k, oracle.reduce_full(x, lay.shape, lay.strides, lay.offset, op=0), x))
    for k, (x, b) in enumerate(zip(xs, bufs)):
        lay = Layout.c_contiguous([x.size])
        items.append(ops.prepare_reduce_full(MaxOp, device, StridedView(b, lay),
                                             StridedView(out, Layout.try_new([1], [1], len(sizes) + k))))
        want.append((len(sizes) + k, oracle.reduce_full(x, [x.size], op=3), x))
    x = xs[6]
    for j, lay in enumerate([Layout.try_new([1024, 1024], [1, 1024], 0), Layout.try_new([1 << 20], [-1], (1 << 20) - 1)]):
        items.append(ops.prepare_reduce_full(MaxOp, device, StridedView(bufs[6], lay),
                                             StridedView(out, Layout.try_new([1], [1], 2 * len(sizes) + j))))
        want.append((2 * len(sizes) + j, oracle.reduce_full(x, lay.shape, lay.strides, lay.offset, op=3), x))
    batch = S.Batch(device, items)
    for rep in range(3):  # replays reuse the tickets: they must come back to rest
        device.write_buffer(out, np.zeros(3 * len(sizes), dtype=dt))
        batch.launch()
        got = device.download_owned(out)
        for slot, w, xx in want:
            assert_close(got[slot:slot + 1], np.array([w], dtype=dt), dt, xx)


def test_fused_batch_widening_and_hazards(device, oracle):
    import hephaestus_b200.seams as S
    rng = np.random.default_rng(91)
    ops = CudaFullReductionOps()
    x = rng.integers(-2**31, 2**31 - 1, size=1_000_003, dtype=np.int64).astype(np.int32)
    xb = device.upload(x)
    o64 = device.alloc_zeroed(np.int64, 4)
    one = lambda k: Layout.try_new([1], [1], k)  # noqa: E731
    items = [ops.prepare_reduce_full(SumOp, device, StridedView(xb, Layout.try_new([n], [1], 0)),
                                     StridedView(o64, one(k))) for k, n in enumerate([1_000_003, 5, 999_999, 64])]
    S.Batch(device, items).launch()
    got = device.download_owned(o64)
    for k, n in enumerate([1_000_003, 5, 999_999, 64]):
        assert got[k] == int(x[:n].astype(np.int64).sum())
    # Read-after-write inside a run: item 2 sums the buffer item 1 writes
    # into, item 3 writes the same element as item 1.  In order: s = sum(a);
    # t = s + b[1]; u = max(b[0..1]) overwrites the element item 1 wrote.
    a = device.upload(np.arange(1, 101, dtype=np.uint32))
    b = device.upload(np.array([0, 7], dtype=np.uint32))
    t = device.alloc_zeroed(np.uint32, 1)
    it1 = ops.prepare_reduce_full(SumOp, device, StridedView(a, Layout.c_contiguous([100])), StridedView(b, one(0)))
    it2 = ops.prepare_reduce_full(SumOp, device, StridedView(b, Layout.c_contiguous([2])), StridedView(t, one(0)))
    it3 = ops.prepare_reduce_full(SumOp, device, StridedView(b, Layout.try_new([1], [1], 1)), StridedView(b, one(0)))
    S.Batch(device, [it1, it2, it3]).launch()
    assert device.download_owned(t)[0] == 5050 + 7
    assert list(device.download_owned(b)) == [7, 7]


# Axis reductions over views whose rows do not start on a 16-byte boundary
# (odd column offsets, odd leading dimensions): rows align themselves per
# (row, segment), column reductions run a scalar head before the vector body.
MISALIGNED_AXIS_VIEWS = [
    Layout.try_new([17, 8000], [8003, 1], 1),     # odd leading dimension
    Layout.try_new([5, 20000], [20001, 1], 3),    # few long rows: split into segments
    Layout.try_new([300, 257], [260, 1], 1),      # row stride 16-byte multiple, odd offset
    Layout.try_new([100, 1000], [1004, 1], 2),
    Layout.try_new([64, 131], [131, 1], 5),       # dense rows of odd length at an odd offset
]


@pytest.mark.parametrize("dt", DTYPES)
def test_misaligned_axis_reductions(device, oracle, dt):
    rng = np.random.default_rng(23)
    ops = CudaAxisReductionOps()
    x = rand(dt, 150_000, rng)
    buf = device.upload(x)
    for lay in MISALIGNED_AXIS_VIEWS:
        for axis in (0, 1):
            for op in (0, 2, 3):
                oshape = list(lay.shape)
                oshape[axis] = 1
                out = device.alloc_zeroed(dt, oshape[0] * oshape[1])
                ops.reduce_axis_into(OPS[op], device, StridedView(buf, lay), axis,
                                     StridedView(out, Layout.c_contiguous(oshape)))
                want = oracle.reduce_axis(x, lay.shape, axis, op=op, in_strides=lay.strides, in_offset=lay.offset)
                assert_close(device.download_owned(out), want, dt, x)


@pytest.mark.parametrize("dt", [np.float32, np.int32, np.float64])
@pytest.mark.parametrize("op", [3, 2])
def test_misaligned_arg_reductions_with_ties(device, oracle, dt, op):
    rng = np.random.default_rng(29 + op)
    ops = CudaAxisReductionOps()
    x = rng.integers(0, 7, size=150_000).astype(dt)  # few distinct values: many exact ties
    buf = device.upload(x)
    fn = ops.argmax_axis_into if op == 3 else ops.argmin_axis_into
    for lay in MISALIGNED_AXIS_VIEWS:
        for axis in (0, 1):
            oshape = list(lay.shape)
            oshape[axis] = 1
            n = oshape[0] * oshape[1]
            vals, idx = device.alloc_zeroed(dt, n), device.alloc_zeroed(np.uint32, n)
            ol = Layout.c_contiguous(oshape)
            fn(device, StridedView(buf, lay), axis, StridedView(vals, ol), StridedView(idx, ol))
            wv, wi = oracle.arg_reduce_axis(x, lay.shape, axis, op=op, in_strides=lay.strides, in_offset=lay.offset)
            np.testing.assert_array_equal(device.download_owned(idx), wi, err_msg=str(lay))
            np.testing.assert_array_equal(device.download_owned(vals), wv)


@pytest.mark.parametrize("dt,op,acc,n,off", [(np.float32, SumOp, np.float32, (1 << 26) + 5, 1),
                                            (np.int32, SumOp, np.int64, (1 << 26) + 1029, 3),
                                            (np.uint32, MaxOp, np.uint32, (1 << 26) + 4096, 0),
                                            (np.float64, MinOp, np.float64, (1 << 25) + 7, 1)])
def test_full_reduction_bulk_staged(device, oracle, dt, op, acc, n, off):
    """Dense runs of 256 MiB and more stream through shared-memory stages
    filled by bulk copies: a 16-byte-misaligned head, whole 16 KiB blocks
    spread over the grid, a ragged tail."""
    import hephaestus_b200.seams as S
    kind = {np.dtype(np.float32): S.SYNTH_F32_UNIFORM_PM1, np.dtype(np.int32): S.SYNTH_I32_PM1000,
            np.dtype(np.uint32): S.SYNTH_U32_LOW4, np.dtype(np.float64): S.SYNTH_F64_UNIT}[np.dtype(dt)]
    x = device.alloc_uninitialized(dt, n + off)
    S.synth_fill(device, x, kind, seed=11)
    out = device.alloc_zeroed(acc, 1)
    for _ in range(2):
        CudaFullReductionOps().reduce_full_into(op, device, StridedView(x, Layout.try_new([n], [1], off)),
                                                StridedView(out, Layout.c_contiguous([1])))
        got = device.download_owned(out)[0]
        hx = device.download_owned(x)[off:]
        want = oracle.reduce_full(np.ascontiguousarray(hx), [n], op=op.code, out_dtype=acc)
        if np.dtype(acc).kind == "f" and op is SumOp:
            assert abs(float(got) - float(want)) <= tol(dt, hx)
        else:
            assert got == want


@pytest.mark.parametrize("dt,acc", [(np.float32, np.float32), (np.int32, np.int64), (np.uint32, np.uint32)])
def test_fused_batch_large(device, oracle, dt, acc):
    """A fused batch of more than 256 MiB: problems of very different sizes
    (many CTAs each, or one), misaligned starts, ragged tails, replayed three
    times."""
    import hephaestus_b200.seams as S
    kind = {np.dtype(np.float32): S.SYNTH_F32_UNIFORM_PM1, np.dtype(np.int32): S.SYNTH_I32_PM1000,
            np.dtype(np.uint32): S.SYNTH_U32_LOW4}[np.dtype(dt)]
    sizes, offs = [(1 << 24) + 3, (1 << 25) + 7, 5, 1 << 24, 30_000_001, 70_001], [1, 0, 2, 0, 3, 1]
    bufs = []
    for k, (n, off) in enumerate(zip(sizes, offs)):
        b = device.alloc_uninitialized(dt, n + off)
        S.synth_fill(device, b, kind, seed=20 + k)
        bufs.append(b)
    out = device.alloc_zeroed(acc, len(sizes))
    ops = CudaFullReductionOps()
    items = [ops.prepare_reduce_full(SumOp, device, StridedView(b, Layout.try_new([n], [1], off)),
                                     StridedView(out, Layout.try_new([1], [1], k)))
             for k, (b, n, off) in enumerate(zip(bufs, sizes, offs))]
    hx = [device.download_owned(b)[off:] for b, off in zip(bufs, offs)]
    want = [oracle.reduce_full(np.ascontiguousarray(x), [x.size], out_dtype=acc) for x in hx]
    batch = S.Batch(device, items)
    for _ in range(3):
        device.write_buffer(out, np.zeros(len(sizes), dtype=acc))
        batch.launch()
        got = device.download_owned(out)
        for k, x in enumerate(hx):
            if np.dtype(acc).kind == "f":
                assert abs(float(got[k]) - float(want[k])) <= tol(dt, x), k
            else:
                assert got[k] == want[k], k
    device.synchronize()
