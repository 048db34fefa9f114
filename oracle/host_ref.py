"""ctypes wrapper over the C oracle ``oracle/_build/libhost_ref.so``.

TEST INFRASTRUCTURE ONLY.  Imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference arm as the checker; the product
package ``hephaestus_b200`` never imports it.  What the C code restates, and
from which reference file:line, is documented in ``oracle/host_ref.h``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libhost_ref.so")

F32, F64, U32, I32, I64 = 0, 1, 2, 3, 4
SUM, PROD, MIN, MAX, MEAN = 0, 1, 2, 3, 4
GEN_F32_UNIFORM_PM1, GEN_U32_LOW4, GEN_F32_NORMAL, GEN_F64_UNIT, GEN_I32_PM1000 = range(5)

_NP = {F32: np.float32, F64: np.float64, U32: np.uint32, I32: np.int32, I64: np.int64}


def dtype_code(np_dtype) -> int:
    dt = np.dtype(np_dtype)
    for code, t in _NP.items():
        if np.dtype(t) == dt:
            return code
    raise TypeError(f"unsupported dtype {dt}")


class _Layout(ctypes.Structure):
    _fields_ = [
        ("rank", ctypes.c_uint32),
        ("_pad", ctypes.c_uint32),
        ("shape", ctypes.c_uint64 * 4),
        ("strides", ctypes.c_int64 * 4),
        ("offset", ctypes.c_uint64),
    ]


def layout(shape, strides=None, offset=0) -> _Layout:
    shape = list(shape)
    if strides is None:
        strides, acc = [], 1
        for extent in reversed(shape):
            strides.insert(0, acc)
            acc *= max(int(extent), 1)
    l = _Layout()
    l.rank = len(shape)
    for d, (s, st) in enumerate(zip(shape, strides)):
        l.shape[d] = int(s)
        l.strides[d] = int(st)
    l.offset = int(offset)
    return l


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, lp = ctypes.c_void_p, ctypes.POINTER(_Layout)
        u64, i32 = ctypes.c_uint64, ctypes.c_int
        L.href_reduce_full.argtypes = [i32, i32, i32, vp, lp, vp]
        L.href_reduce_axis.argtypes = [i32, i32, vp, lp, ctypes.c_uint32, vp, lp]
        L.href_arg_reduce_axis.argtypes = [i32, i32, vp, lp, ctypes.c_uint32, vp, lp, vp, lp]
        L.href_scan_axis.argtypes = [i32, i32, i32, i32, vp, lp, ctypes.c_uint32, vp, lp]
        L.href_map_reduce.argtypes = [i32, i32, vp, lp, vp, lp, vp]
        L.href_hash.argtypes = [u64, u64]
        L.href_hash.restype = u64
        L.href_generate.argtypes = [i32, u64, u64, u64, vp]
        L.href_max_threads.restype = i32
        L.href_exclusive_scan_u32_mt.argtypes = [vp, vp, u64, ctypes.c_uint32, i32]
        L.href_inclusive_scan_i32_mt.argtypes = [vp, vp, u64, ctypes.c_int32, i32]
        L.href_sum_i32_to_i64_mt.argtypes = [vp, u64, i32]
        L.href_sum_i32_to_i64_mt.restype = ctypes.c_int64
        L.href_sum_f32_mt.argtypes = [vp, u64, i32]
        L.href_sum_f32_mt.restype = ctypes.c_float
        L.href_row_argmax_f32_mt.argtypes = [vp, u64, u64, vp, vp, i32]
        L.href_col_sum_f64_mt.argtypes = [vp, u64, u64, vp, i32]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def _check(rc: int, what: str):
    if rc != 0:
        raise ValueError(f"oracle rejected {what}")


# ------------------------------------------------------------------ folds

def reduce_full(storage: np.ndarray, shape, strides=None, offset=0, op=SUM, out_dtype=None):
    """Sequential left fold of the strided view of ``storage`` (1-D array)."""
    dt = dtype_code(storage.dtype)
    odt = dt if out_dtype is None else dtype_code(out_dtype)
    out = np.zeros(1, dtype=_NP[odt])
    l = layout(shape, strides, offset)
    _check(lib().href_reduce_full(dt, odt, op, _ptr(storage), ctypes.byref(l), _ptr(out)), "reduce_full")
    return out[0]


def reduce_axis(storage, in_shape, axis, op=SUM, in_strides=None, in_offset=0,
                out_storage=None, out_shape=None, out_strides=None, out_offset=0):
    dt = dtype_code(storage.dtype)
    il = layout(in_shape, in_strides, in_offset)
    if axis not in (0, 1) or len(in_shape) != 2:
        raise ValueError(f"oracle rejected axis {axis} of a rank-{len(in_shape)} reduction")
    if out_shape is None:
        out_shape = list(in_shape)
        out_shape[axis] = 1
    ol = layout(out_shape, out_strides, out_offset)
    if out_storage is None:
        out_storage = np.zeros(int(np.prod(out_shape)), dtype=storage.dtype)
    _check(lib().href_reduce_axis(dt, op, _ptr(storage), ctypes.byref(il), axis,
                                  _ptr(out_storage), ctypes.byref(ol)), "reduce_axis")
    return out_storage


def arg_reduce_axis(storage, in_shape, axis, op=MAX, in_strides=None, in_offset=0):
    dt = dtype_code(storage.dtype)
    il = layout(in_shape, in_strides, in_offset)
    out_shape = list(in_shape)
    out_shape[axis] = 1
    ol = layout(out_shape)
    vals = np.zeros(int(np.prod(out_shape)), dtype=storage.dtype)
    idx = np.zeros(int(np.prod(out_shape)), dtype=np.uint32)
    _check(lib().href_arg_reduce_axis(dt, op, _ptr(storage), ctypes.byref(il), axis,
                                      _ptr(vals), ctypes.byref(ol), _ptr(idx), ctypes.byref(ol)),
           "arg_reduce_axis")
    return vals, idx


def scan_axis(storage, in_shape, axis, op=SUM, reverse=False, exclusive=False,
              in_strides=None, in_offset=0, out_storage=None, out_strides=None, out_offset=0):
    dt = dtype_code(storage.dtype)
    if axis >= len(in_shape):
        raise ValueError(f"oracle rejected scan axis {axis} of a rank-{len(in_shape)} view")
    il = layout(in_shape, in_strides, in_offset)
    ol = layout(in_shape, out_strides, out_offset)
    if out_storage is None:
        out_storage = np.zeros(int(np.prod(in_shape)), dtype=storage.dtype)
    _check(lib().href_scan_axis(dt, op, int(reverse), int(exclusive), _ptr(storage),
                                ctypes.byref(il), axis, _ptr(out_storage), ctypes.byref(ol)),
           "scan_axis")
    return out_storage


MAP_DOT, MAP_SUM, MAP_NORM_L1, MAP_NORM_L2, MAP_NORM_MAX = range(5)


def map_reduce(map_kind, a, shape, strides=None, offset=0, b=None, b_strides=None, b_offset=0):
    dt = dtype_code(a.dtype)
    la = layout(shape, strides, offset)
    lb = layout(shape, b_strides, b_offset) if b is not None else la
    out = np.zeros(1, dtype=a.dtype)
    _check(lib().href_map_reduce(dt, map_kind, _ptr(a), ctypes.byref(la), _ptr(b if b is not None else a),
                                 ctypes.byref(lb), _ptr(out)), "map_reduce")
    return out[0]


# -------------------------------------------------------------- generators

def hash64(seed: int, index: int) -> int:
    return int(lib().href_hash(seed, index))


def generate(kind: int, seed: int, count: int, index_base: int = 0) -> np.ndarray:
    np_t = {GEN_F32_UNIFORM_PM1: np.float32, GEN_U32_LOW4: np.uint32, GEN_F32_NORMAL: np.float32,
            GEN_F64_UNIT: np.float64, GEN_I32_PM1000: np.int32}[kind]
    out = np.empty(count, dtype=np_t)
    lib().href_generate(kind, seed, index_base, count, _ptr(out))
    return out


# ----------------------------------------------------- CPU baseline variants

def max_threads() -> int:
    return int(lib().href_max_threads())


def exclusive_scan_u32_mt(a: np.ndarray, out: np.ndarray, carry: int = 0, threads: int = 0):
    lib().href_exclusive_scan_u32_mt(_ptr(a), _ptr(out), a.size, carry, threads)
    return out


def inclusive_scan_i32_mt(a: np.ndarray, out: np.ndarray, carry: int = 0, threads: int = 0):
    lib().href_inclusive_scan_i32_mt(_ptr(a), _ptr(out), a.size, carry, threads)
    return out


def sum_i32_to_i64_mt(a: np.ndarray, threads: int = 0) -> int:
    return int(lib().href_sum_i32_to_i64_mt(_ptr(a), a.size, threads))


def sum_f32_mt(a: np.ndarray, threads: int = 0) -> float:
    return float(lib().href_sum_f32_mt(_ptr(a), a.size, threads))


def row_argmax_f32_mt(a: np.ndarray, rows: int, cols: int, threads: int = 0):
    vals = np.empty(rows, np.float32)
    idx = np.empty(rows, np.uint32)
    lib().href_row_argmax_f32_mt(_ptr(a), rows, cols, _ptr(vals), _ptr(idx), threads)
    return vals, idx


def col_sum_f64_mt(a: np.ndarray, rows: int, cols: int, threads: int = 0):
    out = np.empty(cols, np.float64)
    lib().href_col_sum_f64_mt(_ptr(a), rows, cols, _ptr(out), threads)
    return out
