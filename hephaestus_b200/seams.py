"""The reduce/scan seams of hephaestus-core, implemented by the sm_100a kernels.

* ``CudaFullReductionOps``  — ``FullReductionOps`` (crates/hephaestus-core/src/domain/reduction.rs:243-309)
* ``CudaAxisReductionOps``  — ``AxisReductionOps`` (reduction.rs:74-223), plus ``argmax_axis_into`` /
  ``argmin_axis_into`` [EXT: no reference counterpart]
* ``CudaScanOps``           — ``ScanOps`` (crates/hephaestus-core/src/domain/scan.rs:197-264), plus the
  ``exclusive`` flag [EXT]

and the backend free functions the reference's CUDA crate exports
(``reduction``, ``reduce_axis``, ``prod_axis``, ``mean_axis``, ``scan_axis``,
``cumsum``/``suffix_sum``/``cumprod``/``suffix_prod`` and their ``_into`` forms,
crates/hephaestus-cuda/src/application/reduction.rs:67-575,
crates/hephaestus-core/src/domain/accelerator/scan.rs:376-435), which take a
``BlockWidth`` that is validated exactly as the reference validates it
(reduction.rs:339); the kernels size their own launches.

Every call goes through ``libheph_b200.so``; compute calls are stream-ordered
on the device's stream and become visible to ``download`` (which synchronises).
"""
from __future__ import annotations

import ctypes

from . import _native as N
from .core import (CudaBuffer, CudaDevice, CumProdOp, CumSumOp, DispatchFailed, Layout, MaxOp,
                   MinOp, ProdOp, ScanDirection, StridedView, SumOp, check)

BLOCK_WIDTH_DEFAULT = 256  # BlockWidth::DEFAULT (core launch.rs:26)


def _stream(stream):
    return ctypes.c_void_p(stream) if stream else None


class Prepared:
    """A prepared dispatch bound to its operand buffers (rebind contract)."""

    def __init__(self, handle: int, keep):
        self._h = ctypes.c_void_p(handle)
        self._keep = keep  # operands stay alive as long as the handle

    def free(self):
        if self._h:
            N.lib.heph_prepared_free(self._h)
            self._h = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _dispatch(device: CudaDevice, prepared: Prepared, stream=None):
    check(N.lib.heph_dispatch_prepared(device.handle, prepared._h, _stream(stream)))


class Batch:
    """Prepared reductions replayed as one CUDA graph (heph_batch_*)."""

    def __init__(self, device: CudaDevice, items):
        self.device = device
        self._items = list(items)  # keep the prepared handles (and their operands) alive
        arr = (ctypes.c_void_p * len(self._items))(*[it._h.value for it in self._items])
        h = ctypes.c_void_p()
        check(N.lib.heph_batch_create(device.handle, arr, len(self._items), ctypes.byref(h)))
        self._h = h

    def launch(self, stream=None):
        check(N.lib.heph_batch_launch(self._h, _stream(stream)))

    def free(self):
        if self._h:
            N.lib.heph_batch_free(self._h)
            self._h = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def submit_prepared_batch(device: CudaDevice, items, stream=None) -> "Batch":
    """Record `items` (prepared reductions) as a batch and launch it once."""
    b = Batch(device, items)
    b.launch(stream)
    return b


class CudaFullReductionOps:
    """``FullReductionOps<CudaDevice, T>``."""

    def reduce_full_into(self, op, device: CudaDevice, input: StridedView, output: StridedView,
                         stream=None):
        il, ol = input.layout.native(), output.layout.native()
        check(N.lib.heph_reduce_full(device.handle, op.code, input.buffer.handle, ctypes.byref(il),
                                     output.buffer.handle, ctypes.byref(ol), _stream(stream)))

    def prepare_reduce_full(self, op, device: CudaDevice, input: StridedView, output: StridedView):
        il, ol = input.layout.native(), output.layout.native()
        h = ctypes.c_void_p()
        check(N.lib.heph_prepare_reduce_full(device.handle, op.code, input.buffer.handle,
                                             ctypes.byref(il), output.buffer.handle, ctypes.byref(ol),
                                             ctypes.byref(h)))
        return Prepared(h.value, (input, output))

    def dispatch_full(self, device: CudaDevice, prepared: Prepared, stream=None):
        _dispatch(device, prepared, stream)


class CudaAxisReductionOps:
    """``AxisReductionOps<CudaDevice, T>`` (rank-2, keepdims)."""

    def reduce_axis_into(self, op, device, input: StridedView, axis: int, output: StridedView,
                         stream=None):
        self._reduce(op.code, device, input, axis, output, stream)

    def prod_axis_into(self, device, input, axis, output, stream=None):
        self._reduce(N.PROD, device, input, axis, output, stream)

    def mean_axis_into(self, device, input, axis, output, stream=None):
        self._reduce(N.MEAN, device, input, axis, output, stream)

    def min_axis_into(self, device, input, axis, output, stream=None):
        self._reduce(N.MIN, device, input, axis, output, stream)

    def max_axis_into(self, device, input, axis, output, stream=None):
        self._reduce(N.MAX, device, input, axis, output, stream)

    def sum_axis_into(self, device, input, axis, output, stream=None):
        self._reduce(N.SUM, device, input, axis, output, stream)

    def argmax_axis_into(self, device, input: StridedView, axis: int, values: StridedView,
                         indices: StridedView, stream=None):
        self._arg(N.MAX, device, input, axis, values, indices, stream)

    def argmin_axis_into(self, device, input: StridedView, axis: int, values: StridedView,
                         indices: StridedView, stream=None):
        self._arg(N.MIN, device, input, axis, values, indices, stream)

    def prepare_reduce_axis_into(self, op, device, input: StridedView, axis: int,
                                 output: StridedView):
        return _prepare_axis(op.code, device, input, axis, output)

    def dispatch_prepared(self, device, prepared: Prepared, stream=None):
        _dispatch(device, prepared, stream)

    @staticmethod
    def _reduce(code, device, input, axis, output, stream):
        il, ol = input.layout.native(), output.layout.native()
        check(N.lib.heph_reduce_axis(device.handle, code, input.buffer.handle, ctypes.byref(il),
                                     int(axis), output.buffer.handle, ctypes.byref(ol),
                                     _stream(stream)))

    @staticmethod
    def _arg(code, device, input, axis, values, indices, stream):
        il, vl, xl = input.layout.native(), values.layout.native(), indices.layout.native()
        check(N.lib.heph_arg_reduce_axis(device.handle, code, input.buffer.handle, ctypes.byref(il),
                                         int(axis), values.buffer.handle, ctypes.byref(vl),
                                         indices.buffer.handle, ctypes.byref(xl), _stream(stream)))


def _prepare_axis(code, device, input, axis, output):
    il, ol = input.layout.native(), output.layout.native()
    h = ctypes.c_void_p()
    check(N.lib.heph_prepare_reduce_axis(device.handle, code, input.buffer.handle, ctypes.byref(il),
                                         int(axis), output.buffer.handle, ctypes.byref(ol),
                                         ctypes.byref(h)))
    return Prepared(h.value, (input, output))


class CudaScanOps:
    """``ScanOps<CudaDevice, T>`` (``AxisScanOps<CudaDevice>`` in the reference)."""

    def scan_axis_into(self, op, device, input: StridedView, axis: int, direction: int,
                       output: StridedView, exclusive: bool = False, stream=None):
        il, ol = input.layout.native(), output.layout.native()
        check(N.lib.heph_scan_axis(device.handle, op.code, int(direction), int(bool(exclusive)),
                                   input.buffer.handle, ctypes.byref(il), int(axis),
                                   output.buffer.handle, ctypes.byref(ol), _stream(stream)))

    def prepare_scan_axis(self, op, device, input: StridedView, axis: int, direction: int,
                          output: StridedView, exclusive: bool = False):
        il, ol = input.layout.native(), output.layout.native()
        h = ctypes.c_void_p()
        check(N.lib.heph_prepare_scan_axis(device.handle, op.code, int(direction),
                                           int(bool(exclusive)), input.buffer.handle,
                                           ctypes.byref(il), int(axis), output.buffer.handle,
                                           ctypes.byref(ol), ctypes.byref(h)))
        return Prepared(h.value, (input, output))

    def scan_host(self, op, device, host_in, host_out, exclusive: bool = False, chunk_elems: int = 0):
        """[EXT] Scan a host array into a host array with the transfers
        overlapped (heph_scan_host); both arrays C-contiguous, same dtype."""
        from .core import InvalidConfiguration, dtype_code
        if host_in.dtype != host_out.dtype or host_in.size != host_out.size:
            raise InvalidConfiguration("host input and output must have the same type and length")
        if not (host_in.flags.c_contiguous and host_out.flags.c_contiguous):
            raise InvalidConfiguration("host arrays must be C-contiguous")
        check(N.lib.heph_scan_host(device.handle, op.code, int(bool(exclusive)), dtype_code(host_in.dtype),
                                   host_in.ctypes.data_as(ctypes.c_void_p),
                                   host_out.ctypes.data_as(ctypes.c_void_p), host_in.size, int(chunk_elems)))

    def scan_reduce_host(self, op, device, host_in, host_out, reduce_op, acc_dtype=None, exclusive: bool = False,
                         chunk_elems: int = 0):
        """[EXT] scan_host plus the full reduction `reduce_op` of the same host
        array (heph_scan_reduce_host), accumulated in `acc_dtype` (the input
        type, or i64 for i32 / f64 for f32).  Returns the reduction."""
        import numpy as np

        from .core import InvalidConfiguration, dtype_code
        if host_in.dtype != host_out.dtype or host_in.size != host_out.size:
            raise InvalidConfiguration("host input and output must have the same type and length")
        if not (host_in.flags.c_contiguous and host_out.flags.c_contiguous):
            raise InvalidConfiguration("host arrays must be C-contiguous")
        acc = np.zeros(1, dtype=host_in.dtype if acc_dtype is None else acc_dtype)
        check(N.lib.heph_scan_reduce_host(device.handle, op.code, int(bool(exclusive)), dtype_code(host_in.dtype),
                                          host_in.ctypes.data_as(ctypes.c_void_p),
                                          host_out.ctypes.data_as(ctypes.c_void_p), host_in.size, reduce_op.code,
                                          dtype_code(acc.dtype), acc.ctypes.data_as(ctypes.c_void_p),
                                          int(chunk_elems)))
        return acc[0]

    def dispatch_scan(self, device, prepared: Prepared, stream=None):
        _dispatch(device, prepared, stream)


# ------------------------------------------------ backend free functions


def validate_reduction_width(width: int) -> None:
    check(N.lib.heph_validate_reduction_width(int(width)))


def reduction_pass_count(length: int, width: int) -> int:
    return int(N.lib.heph_reduction_pass_count(int(length), int(width)))


def reduction_with_width(op, device: CudaDevice, input: CudaBuffer, width: int) -> CudaBuffer:
    """Reduce a whole contiguous buffer into a new 1-element buffer
    (hephaestus-cuda application/reduction.rs:76)."""
    validate_reduction_width(width)
    out = device.alloc_zeroed(input.dtype, 1)
    CudaFullReductionOps().reduce_full_into(
        op, device, StridedView(input, Layout.c_contiguous([len(input)])),
        StridedView(out, Layout.c_contiguous([1])))
    return out


def reduction(op, device: CudaDevice, input: CudaBuffer) -> CudaBuffer:
    return reduction_with_width(op, device, input, BLOCK_WIDTH_DEFAULT)


def _reduced_layout(layout: Layout, axis: int) -> Layout:
    if axis >= 2:
        raise DispatchFailed(f"axis {axis} is out of bounds for rank-2 reduction")
    shape = list(layout.shape)
    shape[axis] = 1
    return Layout.c_contiguous(shape)


def reduce_axis_into(op, device, input: StridedView, axis: int, output: StridedView,
                     width: int = BLOCK_WIDTH_DEFAULT):
    validate_reduction_width(width)
    CudaAxisReductionOps().reduce_axis_into(op, device, input, axis, output)


def reduce_axis(op, device, input: StridedView, axis: int, width: int = BLOCK_WIDTH_DEFAULT):
    validate_reduction_width(width)
    ol = _reduced_layout(input.layout, axis)
    out = device.alloc_uninitialized(input.buffer.dtype, ol.size())
    CudaAxisReductionOps().reduce_axis_into(op, device, input, axis, StridedView(out, ol))
    return out


def prod_axis(device, input, axis, width=BLOCK_WIDTH_DEFAULT):
    return reduce_axis(ProdOp, device, input, axis, width)


def prod_axis_into(device, input, axis, output, width=BLOCK_WIDTH_DEFAULT):
    reduce_axis_into(ProdOp, device, input, axis, output, width)


def sum_axis(device, input, axis, width=BLOCK_WIDTH_DEFAULT):
    return reduce_axis(SumOp, device, input, axis, width)


def min_axis(device, input, axis, width=BLOCK_WIDTH_DEFAULT):
    return reduce_axis(MinOp, device, input, axis, width)


def max_axis(device, input, axis, width=BLOCK_WIDTH_DEFAULT):
    return reduce_axis(MaxOp, device, input, axis, width)


def mean_axis_into(device, input, axis, output, width=BLOCK_WIDTH_DEFAULT):
    validate_reduction_width(width)
    CudaAxisReductionOps().mean_axis_into(device, input, axis, output)


def mean_axis(device, input, axis, width=BLOCK_WIDTH_DEFAULT):
    validate_reduction_width(width)
    ol = _reduced_layout(input.layout, axis)
    out = device.alloc_uninitialized(input.buffer.dtype, ol.size())
    CudaAxisReductionOps().mean_axis_into(device, input, axis, StridedView(out, ol))
    return out


def prepare_reduce_axis_into(op, device, input, axis, output, width=BLOCK_WIDTH_DEFAULT):
    validate_reduction_width(width)
    return _prepare_axis(op.code, device, input, axis, output)


def prepare_sum_axis_into(device, input, axis, output, width=BLOCK_WIDTH_DEFAULT):
    return prepare_reduce_axis_into(SumOp, device, input, axis, output, width)


def prepare_min_axis_into(device, input, axis, output, width=BLOCK_WIDTH_DEFAULT):
    return prepare_reduce_axis_into(MinOp, device, input, axis, output, width)


def prepare_max_axis_into(device, input, axis, output, width=BLOCK_WIDTH_DEFAULT):
    return prepare_reduce_axis_into(MaxOp, device, input, axis, output, width)


def prepare_mean_axis_into(device, input, axis, output, width=BLOCK_WIDTH_DEFAULT):
    validate_reduction_width(width)
    return _prepare_axis(N.MEAN, device, input, axis, output)


def scan_axis_into(op, device, input: StridedView, axis: int, direction: int, output: StridedView,
                   width: int = BLOCK_WIDTH_DEFAULT, exclusive: bool = False):
    check(N.lib.heph_validate_scan_width(int(width)))
    CudaScanOps().scan_axis_into(op, device, input, axis, direction, output, exclusive)


def scan_axis(op, device, input: StridedView, axis: int, direction: int,
              width: int = BLOCK_WIDTH_DEFAULT, exclusive: bool = False) -> CudaBuffer:
    check(N.lib.heph_validate_scan_width(int(width)))
    ol = Layout.c_contiguous(input.layout.shape)
    out = device.alloc_uninitialized(input.buffer.dtype, ol.size())
    CudaScanOps().scan_axis_into(op, device, input, axis, direction, StridedView(out, ol), exclusive)
    return out


def _conv(op, direction):
    def into(device, input, axis, output, width=BLOCK_WIDTH_DEFAULT):
        scan_axis_into(op, device, input, axis, direction, output, width)

    def alloc(device, input, axis, width=BLOCK_WIDTH_DEFAULT):
        return scan_axis(op, device, input, axis, direction, width)
    return into, alloc


cumsum_into, cumsum = _conv(CumSumOp, ScanDirection.Forward)
suffix_sum_into, suffix_sum = _conv(CumSumOp, ScanDirection.Reverse)
cumprod_into, cumprod = _conv(CumProdOp, ScanDirection.Forward)
suffix_prod_into, suffix_prod = _conv(CumProdOp, ScanDirection.Reverse)


def synth_fill(device: CudaDevice, buffer: CudaBuffer, kind: int, seed: int, index_base: int = 0,
               offset: int = 0, count=None, stream=None):
    """Seeded device-side generator (test/bench support, include/heph/heph_synth.h)."""
    n = len(buffer) - offset if count is None else count
    check(N.lib.heph_synth_fill(device.handle, buffer.handle, int(offset), int(n), int(kind),
                                int(seed), int(index_base), _stream(stream)))


def synth_inject_row_ties(device: CudaDevice, matrix: CudaBuffer, rows: int, cols: int, seed: int,
                          stream=None):
    check(N.lib.heph_synth_inject_row_ties(device.handle, matrix.handle, int(rows), int(cols),
                                           int(seed), _stream(stream)))


SYNTH_F32_UNIFORM_PM1, SYNTH_U32_LOW4, SYNTH_F32_NORMAL, SYNTH_F64_UNIT, SYNTH_I32_PM1000 = range(5)



# ------------------------------------------------ fused map-reductions


def _map_call(device, map_kind, a: StridedView, b, out: StridedView, stream=None):
    al, ol = a.layout.native(), out.layout.native()
    bl = b.layout.native() if b is not None else None
    check(N.lib.heph_map_reduce_full(device.handle, map_kind, a.buffer.handle, ctypes.byref(al),
                                     b.buffer.handle if b is not None else None,
                                     ctypes.byref(bl) if bl is not None else None,
                                     out.buffer.handle, ctypes.byref(ol), _stream(stream)))


def _map_alloc(device, map_kind, a: StridedView, b=None) -> CudaBuffer:
    out = device.alloc_uninitialized(a.buffer.dtype, 1)
    _map_call(device, map_kind, a, b, StridedView(out, Layout.c_contiguous([1])))
    return out


def dot(device, a: StridedView, b: StridedView) -> CudaBuffer:
    """Σ a[i]*b[i] into a new 1-element buffer (hephaestus-cuda linalg/norms.rs:357)."""
    return _map_alloc(device, N.MAP_DOT, a, b)


def trace(device, matrix: StridedView) -> CudaBuffer:
    """Σ a[i][i] of a square rank-2 view (norms.rs:379): the diagonal view
    (stride = row stride + column stride) reduced with the identity map."""
    lay = matrix.layout
    if lay.rank != 2 or lay.shape[0] != lay.shape[1]:
        raise DispatchFailed(f"trace requires a square matrix, got shape {list(lay.shape)}")
    diag = Layout.try_new([lay.shape[0]], [lay.strides[0] + lay.strides[1]], lay.offset)
    return _map_alloc(device, N.MAP_SUM, StridedView(matrix.buffer, diag))


def norm_l1(device, view: StridedView) -> CudaBuffer:
    return _map_alloc(device, N.MAP_NORM_L1, view)


def norm_l2(device, view: StridedView) -> CudaBuffer:
    return _map_alloc(device, N.MAP_NORM_L2, view)


def norm_max(device, view: StridedView) -> CudaBuffer:
    return _map_alloc(device, N.MAP_NORM_MAX, view)


class PreparedMap(Prepared):
    """A prepared map-reduction that owns its 1-element output (prepare_dot /
    prepare_norm_l2 of hephaestus-cuda application/prepared_map_reduction.rs)."""

    def __init__(self, device, map_kind, a: StridedView, b=None):
        out = device.alloc_zeroed(a.buffer.dtype, 1)
        ov = StridedView(out, Layout.c_contiguous([1]))
        al, ol = a.layout.native(), ov.layout.native()
        bl = b.layout.native() if b is not None else None
        h = ctypes.c_void_p()
        check(N.lib.heph_prepare_map_reduce_full(device.handle, map_kind, a.buffer.handle, ctypes.byref(al),
                                                 b.buffer.handle if b is not None else None,
                                                 ctypes.byref(bl) if bl is not None else None,
                                                 out.handle, ctypes.byref(ol), ctypes.byref(h)))
        super().__init__(h.value, (a, b, ov))
        self.device = device
        self._out = out

    def output(self) -> CudaBuffer:
        return self._out

    def dispatch(self, stream=None):
        _dispatch(self.device, self, stream)


def prepare_dot(device, a: StridedView, b: StridedView) -> PreparedMap:
    return PreparedMap(device, N.MAP_DOT, a, b)


def prepare_norm_l2(device, view: StridedView) -> PreparedMap:
    return PreparedMap(device, N.MAP_NORM_L2, view)


class CudaDenseVectorOps:
    """The reduction half of ``DenseVectorOps`` (crates/hephaestus-core/src/domain/vector.rs:57-229):
    one-shot and prepared dot / norms of whole contiguous buffers, read back to the host."""

    @staticmethod
    def _whole(buf):
        return StridedView(buf, Layout.c_contiguous([len(buf)]))

    def _read(self, device, map_kind, a, b=None):
        out = _map_alloc(device, map_kind, self._whole(a), self._whole(b) if b is not None else None)
        return device.download_owned(out)[0]

    def dot(self, device, left: CudaBuffer, right: CudaBuffer):
        if len(left) != len(right):
            raise DispatchFailed(f"dot product shape mismatch: lhs [{len(left)}], rhs [{len(right)}]")
        return self._read(device, N.MAP_DOT, left, right)

    def norm_l1(self, device, vector: CudaBuffer):
        return self._read(device, N.MAP_NORM_L1, vector)

    def norm_l2(self, device, vector: CudaBuffer):
        return self._read(device, N.MAP_NORM_L2, vector)

    def norm_max(self, device, vector: CudaBuffer):
        return self._read(device, N.MAP_NORM_MAX, vector)

    def prepare_dot(self, device, left: CudaBuffer, right: CudaBuffer) -> PreparedMap:
        return prepare_dot(device, self._whole(left), self._whole(right))

    def dot_prepared(self, device, prepared: PreparedMap):
        prepared.dispatch()
        return device.download_owned(prepared.output())[0]

    def prepare_norm_l2(self, device, vector: CudaBuffer) -> PreparedMap:
        return prepare_norm_l2(device, self._whole(vector))

    def norm_l2_prepared(self, device, prepared: PreparedMap):
        prepared.dispatch()
        return device.download_owned(prepared.output())[0]
