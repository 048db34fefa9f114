"""Host mirror of hephaestus-core's device/buffer/error vocabulary.

Names follow the reference so that ported tests read like its own:
``HephaestusError`` and its variants (crates/hephaestus-core/src/domain/error.rs:8-58),
``Layout`` (leto::Layout: shape, element strides, element offset),
``StridedView`` (core view.rs:27), ``CudaDevice`` / ``CudaBuffer``
(the ``ComputeDevice`` seam, core device.rs:90-224), the operator markers
(core ops.rs:736-804) and ``ScanDirection`` (core scan.rs:38).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

import numpy as np

from . import _native as N

# ----------------------------------------------------------------- errors


class HephaestusError(Exception):
    """Base of the seven error variants; ``message`` carries the detail."""

    status = -1
    prefix = "hephaestus error"

    def __init__(self, message: str):
        super().__init__(f"{self.prefix}: {message}")
        self.message = message


class AdapterUnavailable(HephaestusError):
    status, prefix = N.ADAPTER_UNAVAILABLE, "no compatible accelerator adapter available"


class DeviceUnavailable(HephaestusError):
    status, prefix = N.DEVICE_UNAVAILABLE, "accelerator device creation failed"


class AllocationFailed(HephaestusError):
    status, prefix = N.ALLOCATION_FAILED, "accelerator allocation failed"


class LengthMismatch(HephaestusError):
    status, prefix = N.LENGTH_MISMATCH, "length mismatch"


class DispatchFailed(HephaestusError):
    status, prefix = N.DISPATCH_FAILED, "kernel dispatch failed"


class InvalidConfiguration(HephaestusError):
    status, prefix = N.INVALID_CONFIGURATION, "invalid configuration"


class TransferFailed(HephaestusError):
    status, prefix = N.TRANSFER_FAILED, "device transfer failed"


_ERRORS = {c.status: c for c in (AdapterUnavailable, DeviceUnavailable, AllocationFailed,
                                 LengthMismatch, DispatchFailed, InvalidConfiguration,
                                 TransferFailed)}


def check(status: int) -> None:
    """Raise the HephaestusError variant of a non-OK status."""
    if status != N.OK:
        raise _ERRORS.get(status, HephaestusError)(N.last_error())


# -------------------------------------------------------------- operators


class _Op:
    code: int
    name: str


class SumOp(_Op):
    code, name = N.SUM, "sum"


class ProdOp(_Op):
    code, name = N.PROD, "prod"


class MinOp(_Op):
    code, name = N.MIN, "min"


class MaxOp(_Op):
    code, name = N.MAX, "max"


class CumSumOp(_Op):
    code, name = N.SUM, "cumsum"


class CumProdOp(_Op):
    code, name = N.PROD, "cumprod"


class ScanDirection:
    Forward = N.FORWARD
    Reverse = N.REVERSE


# ------------------------------------------------------------------ types

_DTYPES = {
    np.dtype(np.float32): N.F32,
    np.dtype(np.float64): N.F64,
    np.dtype(np.uint32): N.U32,
    np.dtype(np.int32): N.I32,
    np.dtype(np.int64): N.I64,
}
_NP = {v: k for k, v in _DTYPES.items()}


def dtype_code(dtype) -> int:
    try:
        return _DTYPES[np.dtype(dtype)]
    except KeyError:
        raise InvalidConfiguration(f"unsupported element type {np.dtype(dtype)}") from None


def np_dtype(code: int) -> np.dtype:
    return _NP[code]


# ----------------------------------------------------------------- layout


@dataclass(frozen=True)
class Layout:
    """Shape, element strides and element offset of a strided view."""

    shape: tuple
    strides: tuple
    offset: int = 0

    @staticmethod
    def c_contiguous(shape: Sequence[int]) -> "Layout":
        strides, acc = [], 1
        for extent in reversed(list(shape)):
            strides.insert(0, acc)
            acc *= max(int(extent), 1)
        return Layout(tuple(int(s) for s in shape), tuple(strides), 0)

    @staticmethod
    def try_new(shape: Sequence[int], strides: Sequence[int], offset: int = 0) -> "Layout":
        if len(shape) != len(strides):
            raise InvalidConfiguration("shape and strides have different ranks")
        return Layout(tuple(int(s) for s in shape), tuple(int(s) for s in strides), int(offset))

    @property
    def rank(self) -> int:
        return len(self.shape)

    def size(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    def native(self) -> N.Layout_t:
        return N.make_layout(self.shape, self.strides, self.offset)


# ----------------------------------------------------------------- device


class CudaBuffer:
    """A typed device buffer (``DeviceBuffer<T>``); freed when dropped."""

    def __init__(self, device: "CudaDevice", handle: int):
        self.device = device
        self._h = ctypes.c_void_p(handle)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def __len__(self) -> int:
        return int(N.lib.heph_buffer_len(self._h))

    @property
    def dtype(self) -> np.dtype:
        return np_dtype(N.lib.heph_buffer_dtype(self._h))

    def device_ptr(self) -> int:
        return int(N.lib.heph_buffer_device_ptr(self._h) or 0)

    def raw(self) -> int:
        return self.device_ptr()

    def free(self) -> None:
        if self._h:
            N.lib.heph_buffer_free(self._h)
            self._h = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


@dataclass
class StridedView:
    """A buffer viewed through a layout (``StridedView<'_, B, N>``)."""

    buffer: CudaBuffer
    layout: Layout


class CudaDevice:
    """The ``ComputeDevice`` implementor of this backend (one CUDA ordinal)."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        check(N.lib.heph_device_open(int(ordinal), ctypes.byref(h)))
        self._h = h
        self.ordinal = int(ordinal)

    @staticmethod
    def try_default() -> "CudaDevice":
        return CudaDevice(0)

    @staticmethod
    def try_with_ordinal(ordinal: int) -> "CudaDevice":
        return CudaDevice(ordinal)

    @staticmethod
    def device_count() -> int:
        n = ctypes.c_int()
        check(N.lib.heph_device_count(ctypes.byref(n)))
        return n.value

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def backend_name(self) -> str:
        return N.lib.heph_device_backend_name(self._h).decode()

    def sm_count(self) -> int:
        n = ctypes.c_int()
        check(N.lib.heph_device_sm_count(self._h, ctypes.byref(n)))
        return n.value

    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(N.lib.heph_device_stream(self._h, ctypes.byref(s)))
        return int(s.value or 0)

    # --- allocation and transfers (ComputeDevice) ---

    def alloc_zeroed(self, dtype, length: int) -> CudaBuffer:
        h = ctypes.c_void_p()
        check(N.lib.heph_buffer_alloc(self._h, dtype_code(dtype), int(length), 1, ctypes.byref(h)))
        return CudaBuffer(self, h.value)

    def alloc_uninitialized(self, dtype, length: int) -> CudaBuffer:
        h = ctypes.c_void_p()
        check(N.lib.heph_buffer_alloc(self._h, dtype_code(dtype), int(length), 0, ctypes.byref(h)))
        return CudaBuffer(self, h.value)

    def upload(self, host, dtype=None) -> CudaBuffer:
        a = np.ascontiguousarray(host, dtype=dtype)
        h = ctypes.c_void_p()
        check(N.lib.heph_buffer_upload(self._h, dtype_code(a.dtype), a.ctypes.data_as(ctypes.c_void_p),
                                       a.size, ctypes.byref(h)))
        return CudaBuffer(self, h.value)

    def download(self, buffer: CudaBuffer, out: np.ndarray) -> None:
        if not out.flags.c_contiguous:
            raise InvalidConfiguration("download target must be C-contiguous")
        if np.dtype(out.dtype) != buffer.dtype:
            raise InvalidConfiguration("download target element type differs from the buffer")
        check(N.lib.heph_buffer_download(self._h, buffer.handle, out.ctypes.data_as(ctypes.c_void_p),
                                         out.size))

    def download_owned(self, buffer: CudaBuffer) -> np.ndarray:
        out = np.empty(len(buffer), dtype=buffer.dtype)
        self.download(buffer, out)
        return out

    def download_sub_buffer(self, buffer: CudaBuffer, offset: int, out: np.ndarray) -> None:
        check(N.lib.heph_buffer_download_sub(self._h, buffer.handle, int(offset),
                                             out.ctypes.data_as(ctypes.c_void_p), out.size))

    def write_buffer(self, buffer: CudaBuffer, host) -> None:
        a = np.ascontiguousarray(host, dtype=buffer.dtype)
        check(N.lib.heph_buffer_write(self._h, buffer.handle, a.ctypes.data_as(ctypes.c_void_p), a.size))

    def write_sub_buffer(self, buffer: CudaBuffer, offset: int, host) -> None:
        a = np.ascontiguousarray(host, dtype=buffer.dtype)
        check(N.lib.heph_buffer_write_sub(self._h, buffer.handle, int(offset),
                                          a.ctypes.data_as(ctypes.c_void_p), a.size))

    def copy_buffer(self, src: CudaBuffer, dst: CudaBuffer) -> None:
        check(N.lib.heph_buffer_copy(self._h, src.handle, dst.handle))

    def synchronize(self) -> None:
        check(N.lib.heph_device_synchronize(self._h))

    def synchronize_stream(self, stream: int) -> None:
        check(N.lib.heph_stream_synchronize(self._h, ctypes.c_void_p(stream)))

    def close(self) -> None:
        if self._h:
            N.lib.heph_device_close(self._h)
            self._h = ctypes.c_void_p(0)
