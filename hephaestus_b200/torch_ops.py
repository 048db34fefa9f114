"""torch boundary: the module-level functions of the reference's Python
bindings (``sum``, ``min``, ``max``, ``mean``, ``sum_axis``, ``mean_axis``,
``min_axis``, ``max_axis``, ``norm_l1``, ``norm_l2``, ``norm_max``,
``cumsum`` — crates/hephaestus-python/src/reduction.rs:112-367, scan.rs:13)
over CUDA torch tensors, plus ``argmax_axis`` / ``argmin_axis`` / ``cumprod``
/ exclusive scans [EXT].

The tensors' memory is wrapped, not copied (``heph_buffer_wrap``); the work is
enqueued on torch's current stream and results are returned as new tensors
allocated by torch, so these calls compose with ordinary torch code.  Strided
(non-contiguous) tensors are passed as strided views.
"""
from __future__ import annotations

import builtins
import ctypes

import torch

from . import _native as N
from .core import CudaBuffer, CudaDevice, InvalidConfiguration, Layout, StridedView, check

_TORCH_DTYPES = {torch.float32: N.F32, torch.float64: N.F64, torch.int32: N.I32, torch.int64: N.I64}
if hasattr(torch, "uint32"):
    _TORCH_DTYPES[torch.uint32] = N.U32
_devices: dict[int, CudaDevice] = {}


def _device(t: torch.Tensor) -> CudaDevice:
    if not t.is_cuda:
        raise InvalidConfiguration("hephaestus_b200.torch_ops needs CUDA tensors")
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if idx not in _devices:
        _devices[idx] = CudaDevice(idx)
    return _devices[idx]


def _view(t: torch.Tensor) -> StridedView:
    """Wrap a tensor's memory as a buffer + layout (no copy)."""
    if t.dtype not in _TORCH_DTYPES:
        raise InvalidConfiguration(f"unsupported tensor dtype {t.dtype}")
    dev = _device(t)
    span = 1 + builtins.sum((s - 1) * st for s, st in zip(t.shape, t.stride())) if t.numel() else 0
    h = ctypes.c_void_p()
    check(N.lib.heph_buffer_wrap(dev.handle, _TORCH_DTYPES[t.dtype], ctypes.c_void_p(t.data_ptr()), span,
                                 ctypes.byref(h)))
    buf = CudaBuffer(dev, h.value)
    buf._keep = t  # the tensor outlives the wrapper
    shape = list(t.shape) or [1]
    strides = list(t.stride()) or [1]
    return StridedView(buf, Layout.try_new(shape, strides, 0))


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _full(op_code: int, t: torch.Tensor) -> torch.Tensor:
    out = torch.empty(1, dtype=t.dtype, device=t.device)
    iv, ov = _view(t), _view(out)
    check(N.lib.heph_reduce_full(iv.buffer.device.handle, op_code, iv.buffer.handle, ctypes.byref(iv.layout.native()),
                                 ov.buffer.handle, ctypes.byref(ov.layout.native()), ctypes.c_void_p(_stream())))
    return out.reshape(())


def sum(t: torch.Tensor) -> torch.Tensor:  # noqa: A001 - reference name
    return _full(N.SUM, t)


def prod(t: torch.Tensor) -> torch.Tensor:
    return _full(N.PROD, t)


def min(t: torch.Tensor) -> torch.Tensor:  # noqa: A001
    return _full(N.MIN, t)


def max(t: torch.Tensor) -> torch.Tensor:  # noqa: A001
    return _full(N.MAX, t)


def mean(t: torch.Tensor) -> torch.Tensor:
    s = sum(t)
    return s / t.numel() if t.dtype.is_floating_point else torch.div(s, t.numel(), rounding_mode="trunc")


def _axis(op_code: int, t: torch.Tensor, axis: int) -> torch.Tensor:
    if t.dim() != 2:
        raise InvalidConfiguration("axis reductions take rank-2 tensors")
    shape = list(t.shape)
    shape[axis] = 1
    out = torch.empty(shape, dtype=t.dtype, device=t.device)
    iv, ov = _view(t), _view(out)
    check(N.lib.heph_reduce_axis(iv.buffer.device.handle, op_code, iv.buffer.handle, ctypes.byref(iv.layout.native()),
                                 int(axis), ov.buffer.handle, ctypes.byref(ov.layout.native()),
                                 ctypes.c_void_p(_stream())))
    return out


def sum_axis(t, axis):
    return _axis(N.SUM, t, axis)


def mean_axis(t, axis):
    return _axis(N.MEAN, t, axis)


def min_axis(t, axis):
    return _axis(N.MIN, t, axis)


def max_axis(t, axis):
    return _axis(N.MAX, t, axis)


def prod_axis(t, axis):
    return _axis(N.PROD, t, axis)


def _arg(op_code: int, t: torch.Tensor, axis: int):
    if t.dim() != 2:
        raise InvalidConfiguration("arg-reductions take rank-2 tensors")
    shape = list(t.shape)
    shape[axis] = 1
    vals = torch.empty(shape, dtype=t.dtype, device=t.device)
    idx = torch.empty(shape, dtype=torch.int32, device=t.device)
    iv, vv = _view(t), _view(vals)
    h = ctypes.c_void_p()
    check(N.lib.heph_buffer_wrap(iv.buffer.device.handle, N.U32, ctypes.c_void_p(idx.data_ptr()), idx.numel(),
                                 ctypes.byref(h)))
    ib = CudaBuffer(iv.buffer.device, h.value)
    il = Layout.c_contiguous(shape)
    check(N.lib.heph_arg_reduce_axis(iv.buffer.device.handle, op_code, iv.buffer.handle,
                                     ctypes.byref(iv.layout.native()), int(axis), vv.buffer.handle,
                                     ctypes.byref(vv.layout.native()), ib.handle, ctypes.byref(il.native()),
                                     ctypes.c_void_p(_stream())))
    return vals, idx.to(torch.int64)


def argmax_axis(t, axis):
    """[EXT] (values, indices) of the maxima along `axis`; lowest index wins ties."""
    return _arg(N.MAX, t, axis)


def argmin_axis(t, axis):
    """[EXT] (values, indices) of the minima along `axis`; lowest index wins ties."""
    return _arg(N.MIN, t, axis)


def _scan(op_code: int, t: torch.Tensor, axis: int, reverse: bool, exclusive: bool) -> torch.Tensor:
    if t.dim() not in (1, 2):
        raise InvalidConfiguration("scans take rank-1 or rank-2 tensors")
    out = torch.empty(t.shape, dtype=t.dtype, device=t.device)
    iv, ov = _view(t), _view(out)
    check(N.lib.heph_scan_axis(iv.buffer.device.handle, op_code, N.REVERSE if reverse else N.FORWARD,
                               int(bool(exclusive)), iv.buffer.handle, ctypes.byref(iv.layout.native()), int(axis),
                               ov.buffer.handle, ctypes.byref(ov.layout.native()), ctypes.c_void_p(_stream())))
    return out


def cumsum(t, axis=0, reverse=False, exclusive=False):
    return _scan(N.SUM, t, axis, reverse, exclusive)


def cumprod(t, axis=0, reverse=False, exclusive=False):
    return _scan(N.PROD, t, axis, reverse, exclusive)


def _map(map_kind: int, a: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty(1, dtype=a.dtype, device=a.device)
    av, ov = _view(a), _view(out)
    bv = _view(b) if b is not None else None
    check(N.lib.heph_map_reduce_full(av.buffer.device.handle, map_kind, av.buffer.handle,
                                     ctypes.byref(av.layout.native()),
                                     bv.buffer.handle if bv is not None else None,
                                     ctypes.byref(bv.layout.native()) if bv is not None else None,
                                     ov.buffer.handle, ctypes.byref(ov.layout.native()),
                                     ctypes.c_void_p(_stream())))
    return out.reshape(())


def dot(a, b):
    return _map(N.MAP_DOT, a, b)


def norm_l1(t):
    return _map(N.MAP_NORM_L1, t)


def norm_l2(t):
    return _map(N.MAP_NORM_L2, t)


def norm_max(t):
    return _map(N.MAP_NORM_MAX, t)
