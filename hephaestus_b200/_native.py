"""ctypes binding of ``libheph_b200.so`` (the C ABI declared in include/heph/heph.h).

The library is loaded from this package directory.  There is no fallback: if
the shared library is missing or fails to load, importing this module raises,
so no call of this package can silently run anywhere but the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libheph_b200.so")

OK, ADAPTER_UNAVAILABLE, DEVICE_UNAVAILABLE, ALLOCATION_FAILED, LENGTH_MISMATCH, \
    DISPATCH_FAILED, INVALID_CONFIGURATION, TRANSFER_FAILED = range(8)
F32, F64, U32, I32, I64 = range(5)
SUM, PROD, MIN, MAX, MEAN = range(5)
FORWARD, REVERSE = 0, 1
MAP_DOT, MAP_SUM, MAP_NORM_L1, MAP_NORM_L2, MAP_NORM_MAX = range(5)
MAX_RANK = 4
COMM_ID_BYTES = 128


class Layout_t(ctypes.Structure):
    _fields_ = [
        ("rank", ctypes.c_uint32),
        ("_pad", ctypes.c_uint32),
        ("shape", ctypes.c_uint64 * MAX_RANK),
        ("strides", ctypes.c_int64 * MAX_RANK),
        ("offset", ctypes.c_uint64),
    ]


if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `python hephaestus_b200/build.py` "
        "(nvcc, sm_100a); the reduce/scan path has no CPU fallback")

lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)

_vp = ctypes.c_void_p
_u64 = ctypes.c_uint64
_u32 = ctypes.c_uint32
_i = ctypes.c_int
_lp = ctypes.POINTER(Layout_t)
_pp = ctypes.POINTER(ctypes.c_void_p)
_st = ctypes.c_int  # heph_status

# (name, restype, argtypes) of every entry point in include/heph/heph.h and
# include/heph/heph_synth.h.
SIGNATURES = [
    ("heph_last_error", ctypes.c_char_p, []),
    ("heph_status_name", ctypes.c_char_p, [_i]),
    ("heph_dtype_size", ctypes.c_size_t, [_i]),
    ("heph_version", ctypes.c_char_p, []),
    ("heph_device_count", _st, [ctypes.POINTER(_i)]),
    ("heph_device_open", _st, [_i, _pp]),
    ("heph_device_close", _st, [_vp]),
    ("heph_device_backend_name", ctypes.c_char_p, [_vp]),
    ("heph_device_synchronize", _st, [_vp]),
    ("heph_selftest_wait_timeout", _st, [_vp, _i, _vp]),
    ("heph_stream_synchronize", _st, [_vp, _vp]),
    ("heph_device_stream", _st, [_vp, _pp]),
    ("heph_device_ordinal", _st, [_vp, ctypes.POINTER(_i)]),
    ("heph_device_sm_count", _st, [_vp, ctypes.POINTER(_i)]),
    ("heph_buffer_alloc", _st, [_vp, _i, _u64, _i, _pp]),
    ("heph_buffer_upload", _st, [_vp, _i, _vp, _u64, _pp]),
    ("heph_buffer_download", _st, [_vp, _vp, _vp, _u64]),
    ("heph_buffer_download_sub", _st, [_vp, _vp, _u64, _vp, _u64]),
    ("heph_buffer_write", _st, [_vp, _vp, _vp, _u64]),
    ("heph_buffer_write_sub", _st, [_vp, _vp, _u64, _vp, _u64]),
    ("heph_buffer_copy", _st, [_vp, _vp, _vp]),
    ("heph_buffer_free", _st, [_vp]),
    ("heph_buffer_len", _u64, [_vp]),
    ("heph_buffer_dtype", _i, [_vp]),
    ("heph_buffer_device_ptr", _vp, [_vp]),
    ("heph_buffer_wrap", _st, [_vp, _i, _vp, _u64, _pp]),
    ("heph_buffer_upload_async", _st, [_vp, _vp, _u64, _vp, _u64, _vp]),
    ("heph_buffer_download_async", _st, [_vp, _vp, _u64, _vp, _u64, _vp]),
    ("heph_host_alloc_pinned", _st, [_u64, _pp]),
    ("heph_host_free_pinned", _st, [_vp]),
    ("heph_validate_reduction_width", _st, [_u32]),
    ("heph_validate_scan_width", _st, [_u32]),
    ("heph_reduction_pass_count", _u64, [_u64, _u32]),
    ("heph_layout_validate", _st, [_lp, _u64]),
    ("heph_plan_axis_reduction", _st, [_lp, _u64, _lp, _u64, _u32, _i, ctypes.POINTER(_i)]),
    ("heph_plan_axis_scan", _st, [_lp, _u64, _lp, _u64, _u32, _i, ctypes.POINTER(_i)]),
    ("heph_plan_full_reduction", _st, [_lp, _u64, _lp, _u64]),
    ("heph_reduce_full", _st, [_vp, _i, _vp, _lp, _vp, _lp, _vp]),
    ("heph_reduce_axis", _st, [_vp, _i, _vp, _lp, _u32, _vp, _lp, _vp]),
    ("heph_arg_reduce_axis", _st, [_vp, _i, _vp, _lp, _u32, _vp, _lp, _vp, _lp, _vp]),
    ("heph_map_reduce_full", _st, [_vp, _i, _vp, _lp, _vp, _lp, _vp, _lp, _vp]),
    ("heph_prepare_map_reduce_full", _st, [_vp, _i, _vp, _lp, _vp, _lp, _vp, _lp, _pp]),
    ("heph_scan_axis", _st, [_vp, _i, _i, _i, _vp, _lp, _u32, _vp, _lp, _vp]),
    ("heph_prepare_reduce_full", _st, [_vp, _i, _vp, _lp, _vp, _lp, _pp]),
    ("heph_prepare_reduce_axis", _st, [_vp, _i, _vp, _lp, _u32, _vp, _lp, _pp]),
    ("heph_prepare_scan_axis", _st, [_vp, _i, _i, _i, _vp, _lp, _u32, _vp, _lp, _pp]),
    ("heph_dispatch_prepared", _st, [_vp, _vp, _vp]),
    ("heph_prepared_free", _st, [_vp]),
    ("heph_batch_create", _st, [_vp, ctypes.POINTER(ctypes.c_void_p), _u32, _pp]),
    ("heph_batch_launch", _st, [_vp, _vp]),
    ("heph_batch_free", _st, [_vp]),
    ("heph_comm_unique_id", _st, [ctypes.c_char_p]),
    ("heph_comm_init", _st, [_vp, ctypes.c_char_p, _i, _i, _pp]),
    ("heph_comm_destroy", _st, [_vp]),
    ("heph_comm_abort", _st, [_vp]),
    ("heph_comm_peer_exchange", _st, [_vp, ctypes.POINTER(ctypes.c_int)]),
    ("heph_comm_wait", _st, [_vp, _vp, _u32]),
    ("heph_selftest_comm_wait_policy", _st, [_i, _u32, ctypes.POINTER(_i)]),
    ("heph_partitioned_reduce_full", _st, [_vp, _i, _vp, _lp, _vp, _lp, _vp]),
    ("heph_partitioned_scan", _st, [_vp, _i, _i, _vp, _lp, _vp, _lp, _vp]),
    ("heph_partitioned_scan_reduce", _st, [_vp, _i, _i, _vp, _lp, _vp, _lp, _i, _vp, _lp, _vp]),
    ("heph_scan_seeded", _st, [_vp, _i, _i, _vp, _lp, _vp, _lp, _vp, _u64, _vp]),
    ("heph_scan_host", _st, [_vp, _i, _i, _i, _vp, _vp, _u64, _u64]),
    ("heph_scan_reduce_host", _st, [_vp, _i, _i, _i, _vp, _vp, _u64, _i, _i, _vp, _u64]),
    ("heph_reduce_full_noalloc", _st, [_i, _i, _i, _vp, _u64, _vp, _vp]),
    ("heph_synth_fill", _st, [_vp, _vp, _u64, _u64, _i, _u64, _u64, _vp]),
    ("heph_synth_inject_row_ties", _st, [_vp, _vp, _u64, _u64, _u64, _vp]),
]

for _name, _res, _args in SIGNATURES:
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def last_error() -> str:
    msg = lib.heph_last_error()
    return msg.decode() if msg else ""


def make_layout(shape, strides, offset) -> Layout_t:
    l = Layout_t()
    l.rank = len(shape)
    for d, (s, st) in enumerate(zip(shape, strides)):
        l.shape[d] = int(s)
        l.strides[d] = int(st)
    l.offset = int(offset)
    return l
