"""The allocation-free full reduction (heph_reduce_full_noalloc).

It exists for callers that cannot allocate device memory at call time: an
embedder working inside a fixed memory budget that only hands the library
buffers it already owns, or code that must not re-enter an allocator from the
call site.  Each case calls it through the C ABI with raw device pointers and
checks the result against the CPU oracle (the host reference's sequential
fold) on the same input, twice in a row: the static scratch keeps the previous
call's contents, and the second call must not be disturbed by them.  The cases
cover a 16-byte-aligned base, a base aligned only to the element size (the
scalar head of the vector loop), the empty input (the operator's identity) and
SUM / PROD / MIN / MAX.

The file name sorts last so that a run stopping at the first failure has run
every other GPU test before this one; it also passes on its own in a fresh
process (nothing here depends on earlier tests).
"""
import ctypes

import numpy as np
import pytest

from hephaestus_b200 import _native as N
from hephaestus_b200.core import check, dtype_code

pytestmark = pytest.mark.gpu

# Tolerances of the parity suite: integers bit-exact, f32 |d| <= 1e-5 * sum|x|,
# f64 |d| <= 1e-12 * sum|x| (min / max are exact for every type).
_TOL = {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}


def _input(rng, dtype, n, op):
    if op == N.PROD and np.dtype(dtype).kind == "f":
        # ones with a few powers of two: every partial product is exact
        x = np.ones(n, dtype)
        k = min(n, 24)
        x[rng.choice(n, k, replace=False)] = rng.choice([0.5, 2.0], k)
        return x
    if op == N.PROD:
        return rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(dtype) | 1  # odd: the product never hits 0
    if np.dtype(dtype).kind == "f":
        return rng.uniform(-1, 1, n).astype(dtype)
    if np.dtype(dtype) == np.uint32:
        return rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    return rng.integers(-1000, 1000, n).astype(dtype)


def _noalloc(op, dtype, out_dtype, in_ptr, n, out_buf, device):
    check(N.lib.heph_reduce_full_noalloc(op, dtype_code(dtype), dtype_code(out_dtype), ctypes.c_void_p(in_ptr),
                                         n, ctypes.c_void_p(out_buf.device_ptr()),
                                         ctypes.c_void_p(device.stream())))
    return device.download_owned(out_buf)[0]  # ordered after the kernel on the device's stream


def _assert_close(got, want, x, out_dtype, op):
    od = np.dtype(out_dtype)
    if od.kind != "f" or op in (N.MIN, N.MAX):
        assert got == want, (got, want)
        return
    scale = float(np.abs(x.astype(np.float64)).sum()) if op == N.SUM else float(abs(want))
    assert abs(float(got) - float(want)) <= _TOL[od] * max(1.0, scale), (got, want)


@pytest.mark.parametrize("dtype,op,out_dtype", [
    (np.float32, N.SUM, np.float32),
    (np.float32, N.SUM, np.float64),
    (np.uint32, N.SUM, np.uint32),
    (np.int32, N.SUM, np.int64),
    (np.int64, N.SUM, np.int64),
    (np.float64, N.MAX, np.float64),
    (np.float32, N.MIN, np.float32),
    (np.int32, N.MIN, np.int32),
    (np.uint32, N.PROD, np.uint32),
    (np.float32, N.PROD, np.float32),
])
@pytest.mark.parametrize("head", [0, 1])
def test_noalloc_matches_oracle(device, oracle, dtype, op, out_dtype, head):
    """head = 0: the view starts at the buffer's 16-byte-aligned base; head = 1:
    it starts one element in, so only the element size aligns it."""
    rng = np.random.default_rng(2024 + op)
    item = np.dtype(dtype).itemsize
    for n in (1, 7, 1000, (1 << 22) + 3):
        x = _input(rng, dtype, n + head, op)
        buf = device.upload(x)
        view = x[head:]
        want = oracle.reduce_full(np.ascontiguousarray(view), [n], op=op, out_dtype=out_dtype)
        out = device.alloc_zeroed(out_dtype, 1)
        for _ in range(2):
            got = _noalloc(op, dtype, out_dtype, buf.device_ptr() + head * item, n, out, device)
            _assert_close(got, want, view, out_dtype, op)
    device.synchronize()


@pytest.mark.parametrize("dtype,op,identity", [
    (np.float32, N.SUM, 0.0),
    (np.uint32, N.PROD, 1),
    (np.int32, N.MIN, np.iinfo(np.int32).max),
    (np.float32, N.MAX, np.float32(-3.402823466e38)),
])
def test_noalloc_empty_input_gives_identity(device, dtype, op, identity):
    out = device.upload(np.array([7], dtype=dtype))
    buf = device.upload(np.array([5], dtype=dtype))
    for _ in range(2):
        assert _noalloc(op, dtype, dtype, buf.device_ptr(), 0, out, device) == np.array(identity, dtype=dtype)
    device.synchronize()


def test_noalloc_rejects_bad_arguments():
    assert N.lib.heph_reduce_full_noalloc(N.SUM, N.F32, N.U32, ctypes.c_void_p(16), 4,
                                          ctypes.c_void_p(16), None) == N.INVALID_CONFIGURATION
    assert N.lib.heph_reduce_full_noalloc(N.SUM, N.F32, N.F32, None, 4, ctypes.c_void_p(16),
                                          None) == N.INVALID_CONFIGURATION
    assert N.lib.heph_reduce_full_noalloc(N.SUM, N.F32, N.F32, ctypes.c_void_p(18), 4, ctypes.c_void_p(16),
                                          None) == N.INVALID_CONFIGURATION
