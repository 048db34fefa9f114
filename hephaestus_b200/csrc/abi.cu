// abi.cu — the C ABI: device acquisition, typed buffers over a stream-ordered
// pool, host transfers, and the FullReductionOps / AxisReductionOps / ScanOps
// entry points with their prepared (rebind) forms.
//
// Reference counterparts: ComputeDevice (crates/hephaestus-core/src/domain/device.rs:90-224),
// CudaDevice/CudaBuffer (crates/hephaestus-cuda/src/infrastructure/device.rs:91-914,
// buffer.rs:22-97), the seams of core reduction.rs:74-309 and scan.rs:197-264.
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "plan.h"

namespace heph {

// ------------------------------------------------------------------ errors

static thread_local std::string t_last_error;

void set_last_error(const std::string &msg) { t_last_error = msg; }

heph_status fail(heph_status status, const std::string &msg) {
    t_last_error = msg;
    return status;
}

heph_status cuda_fail(heph_status status, cudaError_t err, const char *what) {
    t_last_error = std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")";
    return status;
}

size_t dtype_size(heph_dtype dt) {
    switch (dt) {
        case HEPH_F32: case HEPH_U32: case HEPH_I32: return 4;
        case HEPH_F64: case HEPH_I64: return 8;
    }
    return 0;
}

bool dtype_valid(heph_dtype dt) { return dtype_size(dt) != 0; }

heph_status bind(Device *device) {
    HEPH_CUDA_TRY(cudaSetDevice(device->ordinal), HEPH_DEVICE_UNAVAILABLE, "cudaSetDevice");
    return HEPH_OK;
}

cudaStream_t resolve_stream(Device *device, heph_stream stream) {
    return stream ? static_cast<cudaStream_t>(stream) : device->stream;
}

static heph_status pool_alloc(Device *dev, size_t bytes, cudaStream_t stream, void **out) {
    *out = nullptr;
    if (bytes == 0) return HEPH_OK;
    HEPH_CUDA_TRY(cudaMallocFromPoolAsync(out, bytes, dev->pool, stream), HEPH_ALLOCATION_FAILED,
                  "device allocation");
    return HEPH_OK;
}

heph_status workspace_for(Device *dev, cudaStream_t stream, size_t partial_bytes,
                          size_t scan_status_bytes, Workspace **out) {
    Workspace *ws;
    auto it = dev->workspaces.find(stream);
    if (it == dev->workspaces.end()) {
        ws = new Workspace();
        ws->stream = stream;
        void *p = nullptr;
        heph_status st = pool_alloc(dev, Workspace::kTickets * sizeof(unsigned int) +
                                             sizeof(unsigned long long) + 256,
                                    stream, &p);
        if (st != HEPH_OK) {
            delete ws;
            return st;
        }
        HEPH_CUDA_TRY(cudaMemsetAsync(p, 0, Workspace::kTickets * sizeof(unsigned int) +
                                                 sizeof(unsigned long long) + 256,
                                      stream),
                      HEPH_ALLOCATION_FAILED, "workspace clear");
        ws->tickets = static_cast<unsigned int *>(p);
        ws->tile_counter = reinterpret_cast<unsigned long long *>(ws->tickets + Workspace::kTickets);
        ws->small = ws->tile_counter + 1;
        dev->workspaces[stream] = ws;
    } else {
        ws = it->second;
    }
    if (partial_bytes > ws->partials_bytes) {
        size_t want = std::max(partial_bytes, (size_t)64 << 10);
        if (ws->partials)
            HEPH_CUDA_TRY(cudaFreeAsync(ws->partials, stream), HEPH_ALLOCATION_FAILED, "workspace free");
        ws->partials = nullptr;
        ws->partials_bytes = 0;
        heph_status st = pool_alloc(dev, want, stream, &ws->partials);
        if (st != HEPH_OK) return st;
        ws->partials_bytes = want;
    }
    if (scan_status_bytes > ws->scan_status_bytes) {
        if (ws->scan_status)
            HEPH_CUDA_TRY(cudaFreeAsync(ws->scan_status, stream), HEPH_ALLOCATION_FAILED, "workspace free");
        ws->scan_status = nullptr;
        ws->scan_status_bytes = 0;
        heph_status st = pool_alloc(dev, scan_status_bytes, stream, &ws->scan_status);
        if (st != HEPH_OK) return st;
        HEPH_CUDA_TRY(cudaMemsetAsync(ws->scan_status, 0, scan_status_bytes, stream),
                      HEPH_ALLOCATION_FAILED, "scan status clear");
        ws->scan_status_bytes = scan_status_bytes;
        ws->epoch = 0;
    }
    *out = ws;
    return HEPH_OK;
}

static heph_status check_device_error(Device *dev) {
    unsigned int e = __atomic_exchange_n(dev->error_host, 0u, __ATOMIC_SEQ_CST);
    if (e & DEVERR_LOOKBACK_TIMEOUT)
        return fail(HEPH_DISPATCH_FAILED, "look-back timeout: a scan tile waited too long for its predecessor");
    if (e & DEVERR_BULK_TIMEOUT)
        return fail(HEPH_DISPATCH_FAILED, "bulk copy timeout: a scan part's input never arrived");
    if (e & DEVERR_EXCHANGE_TIMEOUT)
        return fail(HEPH_DISPATCH_FAILED, "exchange timeout: a peer rank's total never arrived");
    if (e) return fail(HEPH_DISPATCH_FAILED, "device reported error code " + std::to_string(e));
    return HEPH_OK;
}

static bool ranges_overlap(const Buffer *a, const Buffer *b) {
    if (!a || !b || a->len == 0 || b->len == 0) return false;
    const char *a0 = static_cast<const char *>(a->ptr), *a1 = a0 + a->len * dtype_size(a->dtype);
    const char *b0 = static_cast<const char *>(b->ptr), *b1 = b0 + b->len * dtype_size(b->dtype);
    return a0 < b1 && b0 < a1;
}

}  // namespace heph

using namespace heph;

// ------------------------------------------------------------------ C ABI

extern "C" const char *heph_last_error(void) { return t_last_error.c_str(); }

extern "C" const char *heph_status_name(heph_status status) {
    // Display prefixes of HephaestusError (core error.rs:10-52).
    switch (status) {
        case HEPH_OK: return "ok";
        case HEPH_ADAPTER_UNAVAILABLE: return "no compatible accelerator adapter available";
        case HEPH_DEVICE_UNAVAILABLE: return "accelerator device creation failed";
        case HEPH_ALLOCATION_FAILED: return "accelerator allocation failed";
        case HEPH_LENGTH_MISMATCH: return "host length does not match device buffer length";
        case HEPH_DISPATCH_FAILED: return "kernel dispatch failed";
        case HEPH_INVALID_CONFIGURATION: return "invalid configuration";
        case HEPH_TRANSFER_FAILED: return "device transfer failed";
    }
    return "unknown status";
}

extern "C" size_t heph_dtype_size(heph_dtype dtype) { return dtype_size(dtype); }

extern "C" const char *heph_version(void) { return "hephaestus-b200 0.1.0 (sm_100a)"; }

extern "C" heph_status heph_device_count(int *out_count) {
    if (!out_count) return fail(HEPH_INVALID_CONFIGURATION, "null output");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    *out_count = n;
    return HEPH_OK;
}

extern "C" heph_status heph_device_open(int ordinal, heph_device **out) {
    if (!out) return fail(HEPH_INVALID_CONFIGURATION, "null output");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(HEPH_ADAPTER_UNAVAILABLE, "no CUDA device is visible to this process");
    }
    if (ordinal < 0 || ordinal >= n)
        return fail(HEPH_DEVICE_UNAVAILABLE, "CUDA device ordinal " + std::to_string(ordinal) +
                                                 " is out of range (" + std::to_string(n) + " devices)");
    cudaDeviceProp prop;
    HEPH_CUDA_TRY(cudaGetDeviceProperties(&prop, ordinal), HEPH_DEVICE_UNAVAILABLE, "device query");
    if (prop.major != 10)
        return fail(HEPH_DEVICE_UNAVAILABLE, std::string("this library is built for sm_100a (B200); device ") +
                                                 prop.name + " is sm_" + std::to_string(prop.major) +
                                                 std::to_string(prop.minor));
    heph_device *dev = new (std::nothrow) heph_device();
    if (!dev) return fail(HEPH_ALLOCATION_FAILED, "host allocation of the device object failed");
    dev->ordinal = ordinal;
    dev->sm_count = prop.multiProcessorCount;
    auto cleanup = [&](heph_status st) {
        if (dev->stream) cudaStreamDestroy(dev->stream);
        if (dev->error_host) cudaFreeHost(dev->error_host);
        delete dev;
        return st;
    };
    if (cudaSetDevice(ordinal) != cudaSuccess)
        return cleanup(fail(HEPH_DEVICE_UNAVAILABLE, "cudaSetDevice failed"));
    if (cudaStreamCreateWithFlags(&dev->stream, cudaStreamNonBlocking) != cudaSuccess)
        return cleanup(fail(HEPH_DEVICE_UNAVAILABLE, "stream creation failed"));
    if (cudaDeviceGetDefaultMemPool(&dev->pool, ordinal) != cudaSuccess)
        return cleanup(fail(HEPH_DEVICE_UNAVAILABLE, "memory pool query failed"));
    // Keep freed pool memory for reuse instead of returning it at every sync.
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(dev->pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    if (cudaHostAlloc((void **)&dev->error_host, sizeof(unsigned int), cudaHostAllocMapped) != cudaSuccess)
        return cleanup(fail(HEPH_DEVICE_UNAVAILABLE, "mapped error word allocation failed"));
    *dev->error_host = 0;
    if (cudaHostGetDevicePointer((void **)&dev->error_dev, dev->error_host, 0) != cudaSuccess)
        return cleanup(fail(HEPH_DEVICE_UNAVAILABLE, "mapped error word lookup failed"));
    // Sanity round trip, as CudaDevice::try_with_ordinal does (device.rs:179-202).
    void *probe = nullptr;
    uint32_t sent = 0x9e3779b9u, got = 0;
    if (cudaMallocFromPoolAsync(&probe, 4, dev->pool, dev->stream) != cudaSuccess ||
        cudaMemcpyAsync(probe, &sent, 4, cudaMemcpyHostToDevice, dev->stream) != cudaSuccess ||
        cudaMemcpyAsync(&got, probe, 4, cudaMemcpyDeviceToHost, dev->stream) != cudaSuccess ||
        cudaFreeAsync(probe, dev->stream) != cudaSuccess ||
        cudaStreamSynchronize(dev->stream) != cudaSuccess || got != sent) {
        cudaGetLastError();
        return cleanup(fail(HEPH_DEVICE_UNAVAILABLE, "device sanity round trip failed"));
    }
    *out = dev;
    return HEPH_OK;
}

extern "C" heph_status heph_device_close(heph_device *device) {
    if (!device) return HEPH_OK;
    cudaSetDevice(device->ordinal);
    cudaDeviceSynchronize();
    for (auto &kv : device->workspaces) {
        Workspace *ws = kv.second;
        if (ws->partials) cudaFree(ws->partials);
        if (ws->scan_status) cudaFree(ws->scan_status);
        if (ws->tickets) cudaFree(ws->tickets);
        delete ws;
    }
    device->workspaces.clear();
    if (device->stream) cudaStreamDestroy(device->stream);
    if (device->error_host) cudaFreeHost(device->error_host);
    delete device;
    return HEPH_OK;
}

extern "C" const char *heph_device_backend_name(const heph_device *) { return "cuda-sm100a"; }

extern "C" heph_status heph_stream_synchronize(heph_device *device, heph_stream stream) {
    if (!device) return fail(HEPH_INVALID_CONFIGURATION, "null device");
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    HEPH_CUDA_TRY(cudaStreamSynchronize(resolve_stream(device, stream)), HEPH_DISPATCH_FAILED,
                  "stream synchronize");
    return check_device_error(device);
}

extern "C" heph_status heph_device_synchronize(heph_device *device) {
    return heph_stream_synchronize(device, nullptr);
}

extern "C" heph_status heph_selftest_wait_timeout(heph_device *device, int which, heph_stream stream) {
    if (!device) return fail(HEPH_INVALID_CONFIGURATION, "null device");
    if (which != 0 && which != 1) return fail(HEPH_INVALID_CONFIGURATION, "unknown wait self-test");
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    return launch_wait_selftest(device, resolve_stream(device, stream), which);
}

extern "C" heph_status heph_device_stream(heph_device *device, heph_stream *out) {
    if (!device || !out) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    *out = device->stream;
    return HEPH_OK;
}

extern "C" heph_status heph_device_ordinal(const heph_device *device, int *out) {
    if (!device || !out) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    *out = device->ordinal;
    return HEPH_OK;
}

extern "C" heph_status heph_device_sm_count(const heph_device *device, int *out) {
    if (!device || !out) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    *out = device->sm_count;
    return HEPH_OK;
}

// ----------------------------------------------------------------- buffers

extern "C" heph_status heph_buffer_alloc(heph_device *device, heph_dtype dtype, uint64_t len,
                                         int zeroed, heph_buffer **out) {
    if (!device || !out) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    *out = nullptr;
    if (!dtype_valid(dtype)) return fail(HEPH_ALLOCATION_FAILED, "unknown element type");
    const size_t es = dtype_size(dtype);
    if (len > UINT64_MAX / es) return fail(HEPH_ALLOCATION_FAILED, "buffer byte size overflows");
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    heph_buffer *b = new (std::nothrow) heph_buffer();
    if (!b) return fail(HEPH_ALLOCATION_FAILED, "host allocation of the buffer object failed");
    b->device = device;
    b->dtype = dtype;
    b->len = len;
    b->owned = true;
    const size_t bytes = (size_t)len * es;
    // Allocations are ordered on the device stream and complete before return.
    if (bytes) {
        if (cudaMallocFromPoolAsync(&b->ptr, bytes, device->pool, device->stream) != cudaSuccess) {
            cudaGetLastError();
            delete b;
            return fail(HEPH_ALLOCATION_FAILED, "device allocation of " + std::to_string(bytes) + " bytes failed");
        }
        if (zeroed) cudaMemsetAsync(b->ptr, 0, bytes, device->stream);
        if (cudaStreamSynchronize(device->stream) != cudaSuccess) {
            cudaGetLastError();
            delete b;
            return fail(HEPH_ALLOCATION_FAILED, "device allocation did not complete");
        }
    }
    *out = b;
    return HEPH_OK;
}

extern "C" heph_status heph_buffer_wrap(heph_device *device, heph_dtype dtype, void *device_ptr,
                                        uint64_t len, heph_buffer **out) {
    if (!device || !out) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    if (!dtype_valid(dtype)) return fail(HEPH_INVALID_CONFIGURATION, "unknown element type");
    if (len && !device_ptr) return fail(HEPH_INVALID_CONFIGURATION, "null device pointer");
    heph_buffer *b = new (std::nothrow) heph_buffer();
    if (!b) return fail(HEPH_ALLOCATION_FAILED, "host allocation of the buffer object failed");
    b->device = device;
    b->dtype = dtype;
    b->len = len;
    b->ptr = device_ptr;
    b->owned = false;
    *out = b;
    return HEPH_OK;
}

extern "C" heph_status heph_buffer_free(heph_buffer *buffer) {
    if (!buffer) return HEPH_OK;
    if (buffer->owned && buffer->ptr) {
        cudaSetDevice(buffer->device->ordinal);
        // Stream-ordered free: work already queued on the device stream that
        // reads the buffer completes first.
        cudaFreeAsync(buffer->ptr, buffer->device->stream);
    }
    delete buffer;
    return HEPH_OK;
}

extern "C" uint64_t heph_buffer_len(const heph_buffer *buffer) { return buffer ? buffer->len : 0; }
extern "C" heph_dtype heph_buffer_dtype(const heph_buffer *buffer) {
    return buffer ? buffer->dtype : HEPH_F32;
}
extern "C" void *heph_buffer_device_ptr(const heph_buffer *buffer) {
    return buffer ? buffer->ptr : nullptr;
}

extern "C" heph_status heph_buffer_upload(heph_device *device, heph_dtype dtype, const void *host,
                                          uint64_t len, heph_buffer **out) {
    heph_status st = heph_buffer_alloc(device, dtype, len, 0, out);
    if (st != HEPH_OK) return st;
    if (len == 0) return HEPH_OK;
    if (!host) {
        heph_buffer_free(*out);
        *out = nullptr;
        return fail(HEPH_TRANSFER_FAILED, "null host pointer");
    }
    if (cudaMemcpyAsync((*out)->ptr, host, len * dtype_size(dtype), cudaMemcpyHostToDevice,
                        device->stream) != cudaSuccess ||
        cudaStreamSynchronize(device->stream) != cudaSuccess) {
        cudaError_t e = cudaGetLastError();
        heph_buffer_free(*out);
        *out = nullptr;
        return cuda_fail(HEPH_TRANSFER_FAILED, e, "host-to-device copy");
    }
    return HEPH_OK;
}

static heph_status copy_sub(heph_device *device, const heph_buffer *buffer, uint64_t offset,
                            uint64_t count, void *host_dst, const void *host_src, bool to_host) {
    if (!device || !buffer) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    if (offset > buffer->len || count > buffer->len - offset)
        return fail(HEPH_LENGTH_MISMATCH, "host length " + std::to_string(count) + " at offset " +
                                              std::to_string(offset) +
                                              " does not fit device buffer length " +
                                              std::to_string(buffer->len));
    if (count == 0) return HEPH_OK;
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    const size_t es = dtype_size(buffer->dtype);
    char *dptr = static_cast<char *>(buffer->ptr) + offset * es;
    cudaError_t e = to_host
        ? cudaMemcpyAsync(host_dst, dptr, count * es, cudaMemcpyDeviceToHost, device->stream)
        : cudaMemcpyAsync(dptr, host_src, count * es, cudaMemcpyHostToDevice, device->stream);
    if (e != cudaSuccess) return cuda_fail(HEPH_TRANSFER_FAILED, e, "transfer");
    e = cudaStreamSynchronize(device->stream);
    if (e != cudaSuccess) return cuda_fail(HEPH_TRANSFER_FAILED, e, "transfer");
    return check_device_error(device);
}

extern "C" heph_status heph_buffer_download(heph_device *device, const heph_buffer *buffer,
                                            void *host, uint64_t host_len) {
    if (!buffer) return fail(HEPH_INVALID_CONFIGURATION, "null buffer");
    if (host_len != buffer->len)
        return fail(HEPH_LENGTH_MISMATCH, "host length " + std::to_string(host_len) +
                                              " does not match device buffer length " +
                                              std::to_string(buffer->len));
    return copy_sub(device, buffer, 0, host_len, host, nullptr, true);
}

extern "C" heph_status heph_buffer_download_sub(heph_device *device, const heph_buffer *buffer,
                                                uint64_t offset, void *host, uint64_t count) {
    return copy_sub(device, buffer, offset, count, host, nullptr, true);
}

extern "C" heph_status heph_buffer_write(heph_device *device, heph_buffer *buffer,
                                         const void *host, uint64_t host_len) {
    if (!buffer) return fail(HEPH_INVALID_CONFIGURATION, "null buffer");
    if (host_len != buffer->len)
        return fail(HEPH_LENGTH_MISMATCH, "host length " + std::to_string(host_len) +
                                              " does not match device buffer length " +
                                              std::to_string(buffer->len));
    return copy_sub(device, buffer, 0, host_len, nullptr, host, false);
}

extern "C" heph_status heph_buffer_write_sub(heph_device *device, heph_buffer *buffer,
                                             uint64_t offset, const void *host, uint64_t count) {
    return copy_sub(device, buffer, offset, count, nullptr, host, false);
}

extern "C" heph_status heph_buffer_copy(heph_device *device, const heph_buffer *src,
                                        heph_buffer *dst) {
    if (!device || !src || !dst) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    if (src->len != dst->len)
        return fail(HEPH_LENGTH_MISMATCH, "host length " + std::to_string(src->len) +
                                              " does not match device buffer length " +
                                              std::to_string(dst->len));
    if (src->dtype != dst->dtype) return fail(HEPH_INVALID_CONFIGURATION, "element types differ");
    if (src->len == 0) return HEPH_OK;
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    HEPH_CUDA_TRY(cudaMemcpyAsync(dst->ptr, src->ptr, src->len * dtype_size(src->dtype),
                                  cudaMemcpyDeviceToDevice, device->stream),
                  HEPH_TRANSFER_FAILED, "device copy");
    HEPH_CUDA_TRY(cudaStreamSynchronize(device->stream), HEPH_TRANSFER_FAILED, "device copy");
    return HEPH_OK;
}

extern "C" heph_status heph_buffer_upload_async(heph_device *device, heph_buffer *buffer,
                                                uint64_t offset, const void *host, uint64_t count,
                                                heph_stream stream) {
    if (!device || !buffer) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    if (offset > buffer->len || count > buffer->len - offset)
        return fail(HEPH_LENGTH_MISMATCH, "upload range exceeds the device buffer");
    if (count == 0) return HEPH_OK;
    const size_t es = dtype_size(buffer->dtype);
    HEPH_CUDA_TRY(cudaMemcpyAsync(static_cast<char *>(buffer->ptr) + offset * es, host, count * es,
                                  cudaMemcpyHostToDevice, resolve_stream(device, stream)),
                  HEPH_TRANSFER_FAILED, "host-to-device copy");
    return HEPH_OK;
}

extern "C" heph_status heph_buffer_download_async(heph_device *device, const heph_buffer *buffer,
                                                  uint64_t offset, void *host, uint64_t count,
                                                  heph_stream stream) {
    if (!device || !buffer) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    if (offset > buffer->len || count > buffer->len - offset)
        return fail(HEPH_LENGTH_MISMATCH, "download range exceeds the device buffer");
    if (count == 0) return HEPH_OK;
    const size_t es = dtype_size(buffer->dtype);
    HEPH_CUDA_TRY(cudaMemcpyAsync(host, static_cast<const char *>(buffer->ptr) + offset * es,
                                  count * es, cudaMemcpyDeviceToHost, resolve_stream(device, stream)),
                  HEPH_TRANSFER_FAILED, "device-to-host copy");
    return HEPH_OK;
}

extern "C" heph_status heph_host_alloc_pinned(uint64_t bytes, void **out) {
    if (!out) return fail(HEPH_INVALID_CONFIGURATION, "null output");
    HEPH_CUDA_TRY(cudaHostAlloc(out, bytes ? bytes : 1, cudaHostAllocPortable),
                  HEPH_ALLOCATION_FAILED, "pinned host allocation");
    return HEPH_OK;
}

extern "C" heph_status heph_host_free_pinned(void *ptr) {
    if (ptr) cudaFreeHost(ptr);
    return HEPH_OK;
}

// -------------------------------------------------------------- the seams

namespace {

enum class Kind { Full, Axis, Arg, Scan, Map };

struct Call {
    Kind kind;
    int op;
    heph_buffer *in;
    heph_layout in_l;
    heph_buffer *out;
    heph_layout out_l;
    heph_buffer *idx = nullptr;
    heph_layout idx_l{};
    uint32_t axis = 0;
    bool reverse = false, exclusive = false, mean = false;
    bool noop = false;
    uint64_t count = 0;  // full and map reductions
    AxisProblem p{};     // axis reductions and scans
    const heph_buffer *b = nullptr;  // second operand of a dot product
    heph_layout b_l{};
};

heph_status check_buffers(const heph_device *device, const heph_buffer *in, const heph_layout *il,
                          const heph_buffer *out, const heph_layout *ol) {
    if (!device || !in || !il || !out || !ol) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    if (in->device != device || out->device != device)
        return fail(HEPH_DISPATCH_FAILED, "operand buffers belong to another device");
    return HEPH_OK;
}

heph_status plan_full(heph_device *device, heph_op op, const heph_buffer *in, const heph_layout *il,
                      heph_buffer *out, const heph_layout *ol, Call *c) {
    heph_status st = check_buffers(device, in, il, out, ol);
    if (st != HEPH_OK) return st;
    if (op != HEPH_SUM && op != HEPH_PROD && op != HEPH_MIN && op != HEPH_MAX)
        return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
    const bool widen = (in->dtype == HEPH_I32 && out->dtype == HEPH_I64) ||
                       (in->dtype == HEPH_F32 && out->dtype == HEPH_F64);
    if (in->dtype != out->dtype && !widen)
        return fail(HEPH_DISPATCH_FAILED,
                    "full reduction output element type must match the input or widen it (i32->i64, f32->f64)");
    uint64_t count = 0;
    st = plan_full_reduction(*il, in->len, *ol, out->len, &count);
    if (st != HEPH_OK) return st;
    *c = Call{Kind::Full, (int)op, const_cast<heph_buffer *>(in), *il, out, *ol};
    c->count = count;
    return HEPH_OK;
}

heph_status plan_axis(heph_device *device, heph_op op, const heph_buffer *in, const heph_layout *il,
                      uint32_t axis, heph_buffer *out, const heph_layout *ol, Call *c) {
    heph_status st = check_buffers(device, in, il, out, ol);
    if (st != HEPH_OK) return st;
    if (op < HEPH_SUM || op > HEPH_MEAN) return fail(HEPH_INVALID_CONFIGURATION, "unknown axis reduction operator");
    if (in->dtype != out->dtype)
        return fail(HEPH_DISPATCH_FAILED, "axis reduction output element type must match the input");
    // reject_empty_axis precedes planning (hephaestus-cuda application/reduction.rs:180-187,
    // prepared_axis_reduction.rs:165,185,205).
    if (axis >= 2)
        return fail(HEPH_DISPATCH_FAILED, "axis " + std::to_string(axis) + " is out of bounds for rank-2 reduction");
    if ((op == HEPH_MIN || op == HEPH_MAX || op == HEPH_MEAN) && il->rank == 2 && il->shape[axis] == 0) {
        const char *name = op == HEPH_MIN ? "min_axis" : op == HEPH_MAX ? "max_axis" : "mean_axis";
        return fail(HEPH_DISPATCH_FAILED,
                    std::string(name) + " is undefined for empty axis " + std::to_string(axis));
    }
    *c = Call{Kind::Axis, op == HEPH_MEAN ? (int)HEPH_SUM : (int)op, const_cast<heph_buffer *>(in), *il, out, *ol};
    c->axis = axis;
    c->mean = op == HEPH_MEAN;
    return plan_axis_reduction(*il, in->len, *ol, out->len, axis, ranges_overlap(in, out), &c->noop, &c->p);
}

heph_status plan_scan(heph_device *device, heph_op op, heph_scan_direction dir, int exclusive,
                      const heph_buffer *in, const heph_layout *il, uint32_t axis, heph_buffer *out,
                      const heph_layout *ol, Call *c) {
    heph_status st = check_buffers(device, in, il, out, ol);
    if (st != HEPH_OK) return st;
    if (op != HEPH_SUM && op != HEPH_PROD)
        return fail(HEPH_INVALID_CONFIGURATION, "scans support the sum (cumsum) and product (cumprod) operators");
    if (dir != HEPH_FORWARD && dir != HEPH_REVERSE)
        return fail(HEPH_INVALID_CONFIGURATION, "unknown scan direction");
    if (in->dtype != out->dtype) return fail(HEPH_DISPATCH_FAILED, "scan output element type must match the input");
    *c = Call{Kind::Scan, (int)op, const_cast<heph_buffer *>(in), *il, out, *ol};
    c->axis = axis;
    c->reverse = dir == HEPH_REVERSE;
    c->exclusive = exclusive != 0;
    return plan_axis_scan(*il, in->len, *ol, out->len, axis, ranges_overlap(in, out), &c->noop, &c->p);
}

heph_status plan_map(heph_device *device, heph_map map, const heph_buffer *a, const heph_layout *al,
                     const heph_buffer *b, const heph_layout *bl, heph_buffer *out, const heph_layout *ol, Call *c) {
    heph_status st = check_buffers(device, a, al, out, ol);
    if (st != HEPH_OK) return st;
    if ((int)map < HEPH_MAP_DOT || (int)map > HEPH_MAP_NORM_MAX)
        return fail(HEPH_INVALID_CONFIGURATION, "unknown map reduction");
    if (out->dtype != a->dtype) return fail(HEPH_DISPATCH_FAILED, "map reduction output element type must match the input");
    if (map == HEPH_MAP_NORM_L2 && a->dtype != HEPH_F32 && a->dtype != HEPH_F64)
        return fail(HEPH_DISPATCH_FAILED, "norm_l2 requires a floating-point element type");
    if (map == HEPH_MAP_DOT) {
        if (!b || !bl) return fail(HEPH_INVALID_CONFIGURATION, "dot product needs two operands");
        if (b->device != device) return fail(HEPH_DISPATCH_FAILED, "operand buffers belong to another device");
        if (b->dtype != a->dtype) return fail(HEPH_DISPATCH_FAILED, "dot product operands must share an element type");
        bool same = al->rank == bl->rank;
        for (uint32_t d = 0; same && d < al->rank && d < HEPH_MAX_RANK; ++d) same = al->shape[d] == bl->shape[d];
        if (!same)
            return fail(HEPH_DISPATCH_FAILED, "dot product shape mismatch: lhs " + shape_debug(*al) + ", rhs " +
                                                  shape_debug(*bl));
        st = validate_layout(*bl, b->len);
        if (st != HEPH_OK) return st;
    }
    uint64_t count = 0;
    st = plan_full_reduction(*al, a->len, *ol, out->len, &count);
    if (st != HEPH_OK) return st;
    *c = Call{Kind::Map, (int)map, const_cast<heph_buffer *>(a), *al, out, *ol};
    c->count = count;
    c->b = map == HEPH_MAP_DOT ? b : a;
    c->b_l = map == HEPH_MAP_DOT ? *bl : *al;
    return HEPH_OK;
}

heph_status run(heph_device *device, const Call &c, heph_stream stream) {
    if (c.noop) return HEPH_OK;
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    cudaStream_t s = resolve_stream(device, stream);
    switch (c.kind) {
        case Kind::Full: {
            void *out = static_cast<char *>(c.out->ptr) + c.out_l.offset * dtype_size(c.out->dtype);
            return launch_reduce_full(device, s, c.op, c.in->dtype, c.out->dtype, c.in->ptr, c.in_l,
                                      c.count, out);
        }
        case Kind::Axis:
            return launch_reduce_axis(device, s, c.op, c.in->dtype, c.in->ptr, c.p, c.out->ptr, c.mean,
                                      nullptr, 0, 0);
        case Kind::Arg: {
            const uint32_t other = 1 - c.axis;
            return launch_reduce_axis(device, s, c.op, c.in->dtype, c.in->ptr, c.p, c.out->ptr, false,
                                      static_cast<uint32_t *>(c.idx->ptr), (int64_t)c.idx_l.offset,
                                      c.idx_l.strides[other]);
        }
        case Kind::Scan:
            return launch_scan(device, s, c.op, c.in->dtype, c.in->ptr, c.out->ptr, c.p, c.reverse,
                               c.exclusive, nullptr);
        case Kind::Map: {
            void *out = static_cast<char *>(c.out->ptr) + c.out_l.offset * dtype_size(c.out->dtype);
            return launch_map_reduce(device, s, c.op, c.in->dtype, c.in->ptr, c.in_l, c.b->ptr, c.b_l, c.count, out);
        }
    }
    return fail(HEPH_DISPATCH_FAILED, "unknown call kind");
}

}  // namespace

struct heph_prepared {
    Call call;
};

extern "C" heph_status heph_reduce_full(heph_device *device, heph_op op, const heph_buffer *in,
                                        const heph_layout *in_layout, heph_buffer *out,
                                        const heph_layout *out_layout, heph_stream stream) {
    Call c{};
    heph_status st = plan_full(device, op, in, in_layout, out, out_layout, &c);
    if (st != HEPH_OK) return st;
    return run(device, c, stream);
}

extern "C" heph_status heph_reduce_axis(heph_device *device, heph_op op, const heph_buffer *in,
                                        const heph_layout *in_layout, uint32_t axis,
                                        heph_buffer *out, const heph_layout *out_layout,
                                        heph_stream stream) {
    Call c{};
    heph_status st = plan_axis(device, op, in, in_layout, axis, out, out_layout, &c);
    if (st != HEPH_OK) return st;
    return run(device, c, stream);
}

extern "C" heph_status heph_arg_reduce_axis(heph_device *device, heph_op op, const heph_buffer *in,
                                            const heph_layout *in_layout, uint32_t axis,
                                            heph_buffer *values, const heph_layout *values_layout,
                                            heph_buffer *indices, const heph_layout *indices_layout,
                                            heph_stream stream) {
    if (op != HEPH_MIN && op != HEPH_MAX)
        return fail(HEPH_INVALID_CONFIGURATION, "arg-reduction supports min and max");
    if (!indices || !indices_layout) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    Call c{};
    heph_status st = plan_axis(device, op, in, in_layout, axis, values, values_layout, &c);
    if (st != HEPH_OK) return st;
    if (indices->device != device) return fail(HEPH_DISPATCH_FAILED, "operand buffers belong to another device");
    if (indices->dtype != HEPH_U32) return fail(HEPH_DISPATCH_FAILED, "arg-reduction indices must be a u32 buffer");
    if (indices_layout->rank != 2 || values_layout->rank != 2 ||
        indices_layout->shape[0] != values_layout->shape[0] ||
        indices_layout->shape[1] != values_layout->shape[1])
        return fail(HEPH_DISPATCH_FAILED, "arg-reduction index layout must match the value layout shape " +
                                              shape_debug(*values_layout));
    if (ranges_overlap(in, indices) || ranges_overlap(values, indices))
        return fail(HEPH_DISPATCH_FAILED, "arg-reduction index buffer must not alias another operand");
    if (has_zero_stride_aliasing(*indices_layout))
        return fail(HEPH_DISPATCH_FAILED, "arg-reduction index layout must not contain zero-stride aliasing");
    st = validate_layout(*indices_layout, indices->len);
    if (st != HEPH_OK) return st;
    if (in_layout->shape[axis] > 0xffffffffull)
        return fail(HEPH_DISPATCH_FAILED, "arg-reduction axis length exceeds the u32 index range");
    c.kind = Kind::Arg;
    c.idx = indices;
    c.idx_l = *indices_layout;
    return run(device, c, stream);
}

extern "C" heph_status heph_scan_axis(heph_device *device, heph_op op, heph_scan_direction direction,
                                      int exclusive, const heph_buffer *in,
                                      const heph_layout *in_layout, uint32_t axis, heph_buffer *out,
                                      const heph_layout *out_layout, heph_stream stream) {
    Call c{};
    heph_status st = plan_scan(device, op, direction, exclusive, in, in_layout, axis, out, out_layout, &c);
    if (st != HEPH_OK) return st;
    return run(device, c, stream);
}

extern "C" heph_status heph_scan_seeded(heph_device *device, heph_op op, int exclusive,
                                        const heph_buffer *in, const heph_layout *in_layout,
                                        heph_buffer *out, const heph_layout *out_layout,
                                        const heph_buffer *carry, uint64_t carry_offset,
                                        heph_stream stream) {
    Call c{};
    heph_status st = plan_scan(device, op, HEPH_FORWARD, exclusive, in, in_layout, 0, out, out_layout, &c);
    if (st != HEPH_OK) return st;
    if (in_layout->rank != 1) return fail(HEPH_DISPATCH_FAILED, "seeded scans take rank-1 views");
    if (!carry || carry->dtype != in->dtype || carry_offset >= carry->len)
        return fail(HEPH_DISPATCH_FAILED, "seeded scan carry must be an element of the input type");
    if (c.noop) return HEPH_OK;
    st = bind(device);
    if (st != HEPH_OK) return st;
    const void *cptr = static_cast<const char *>(carry->ptr) + carry_offset * dtype_size(carry->dtype);
    return launch_scan(device, resolve_stream(device, stream), c.op, in->dtype, in->ptr, out->ptr, c.p,
                       false, c.exclusive, cptr);
}

extern "C" heph_status heph_map_reduce_full(heph_device *device, heph_map map, const heph_buffer *a,
                                            const heph_layout *a_layout, const heph_buffer *b,
                                            const heph_layout *b_layout, heph_buffer *out,
                                            const heph_layout *out_layout, heph_stream stream) {
    Call c{};
    heph_status st = plan_map(device, map, a, a_layout, b, b_layout, out, out_layout, &c);
    if (st != HEPH_OK) return st;
    return run(device, c, stream);
}

extern "C" heph_status heph_prepare_map_reduce_full(heph_device *device, heph_map map, const heph_buffer *a,
                                                    const heph_layout *a_layout, const heph_buffer *b,
                                                    const heph_layout *b_layout, heph_buffer *out,
                                                    const heph_layout *out_layout, heph_prepared **out_prepared) {
    if (!out_prepared) return fail(HEPH_INVALID_CONFIGURATION, "null output");
    *out_prepared = nullptr;
    Call c{};
    heph_status st = plan_map(device, map, a, a_layout, b, b_layout, out, out_layout, &c);
    if (st != HEPH_OK) return st;
    *out_prepared = new heph_prepared{c};
    return HEPH_OK;
}

extern "C" heph_status heph_prepare_reduce_full(heph_device *device, heph_op op, const heph_buffer *in,
                                                const heph_layout *in_layout, heph_buffer *out,
                                                const heph_layout *out_layout, heph_prepared **out_prepared) {
    if (!out_prepared) return fail(HEPH_INVALID_CONFIGURATION, "null output");
    *out_prepared = nullptr;
    Call c{};
    heph_status st = plan_full(device, op, in, in_layout, out, out_layout, &c);
    if (st != HEPH_OK) return st;
    *out_prepared = new heph_prepared{c};
    return HEPH_OK;
}

extern "C" heph_status heph_prepare_reduce_axis(heph_device *device, heph_op op, const heph_buffer *in,
                                                const heph_layout *in_layout, uint32_t axis,
                                                heph_buffer *out, const heph_layout *out_layout,
                                                heph_prepared **out_prepared) {
    if (!out_prepared) return fail(HEPH_INVALID_CONFIGURATION, "null output");
    *out_prepared = nullptr;
    Call c{};
    heph_status st = plan_axis(device, op, in, in_layout, axis, out, out_layout, &c);
    if (st != HEPH_OK) return st;
    *out_prepared = new heph_prepared{c};
    return HEPH_OK;
}

extern "C" heph_status heph_prepare_scan_axis(heph_device *device, heph_op op,
                                              heph_scan_direction direction, int exclusive,
                                              const heph_buffer *in, const heph_layout *in_layout,
                                              uint32_t axis, heph_buffer *out,
                                              const heph_layout *out_layout, heph_prepared **out_prepared) {
    if (!out_prepared) return fail(HEPH_INVALID_CONFIGURATION, "null output");
    *out_prepared = nullptr;
    Call c{};
    heph_status st = plan_scan(device, op, direction, exclusive, in, in_layout, axis, out, out_layout, &c);
    if (st != HEPH_OK) return st;
    *out_prepared = new heph_prepared{c};
    return HEPH_OK;
}

extern "C" heph_status heph_dispatch_prepared(heph_device *device, const heph_prepared *prepared,
                                              heph_stream stream) {
    if (!device || !prepared) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    if (prepared->call.in->device != device)
        return fail(HEPH_DISPATCH_FAILED, "prepared operands belong to another device");
    return run(device, prepared->call, stream);
}

extern "C" heph_status heph_prepared_free(heph_prepared *prepared) {
    delete prepared;
    return HEPH_OK;
}

// ----------------------------------------------------- prepared batches

// A CUDA graph that replays a fixed list of prepared reductions with one
// launch (submit_prepared_reduction_batch, hephaestus-cuda
// application/prepared_reduction.rs:165; submit_prepared_axis_reduction_batch,
// prepared_axis_reduction.rs:84).  Scans are not batchable: each scan launch
// carries the epoch tag of its tile status, which a replayed graph would reuse.
//
// Consecutive dense full reductions of one operator and element type are
// fused into ONE kernel node (reduce_fused_kernel): the resident CTAs are
// shared out over the problems, so a batch of small reductions streams at
// HBM speed instead of paying a launch and a serial finalize per item.  A run
// is fused only while no output of it overlaps an input of it or another of
// its outputs, so the result equals running the items in order.
namespace {

struct Segment {
    uint32_t first = 0, count = 1;  // items [first, first + count)
    bool fused = false;
    uint32_t grid = 0;
    size_t table_off = 0, partials_off = 0, tickets_off = 0;  // into heph_batch::fused_mem
};

struct ByteRange {
    uintptr_t lo, hi;
    bool overlaps(const ByteRange &o) const { return lo < o.hi && o.lo < hi; }
};

// The dense run a full reduction reads, or false when its view is not one.
bool fusable_full(const Call &c, FusedFull *f, ByteRange *in, ByteRange *out) {
    if (c.kind != Kind::Full || c.noop || c.count == 0) return false;
    int64_t first = 0;
    if (layout_is_dense(c.in_l)) first = (int64_t)c.in_l.offset;
    else if (!layout_covers_dense_block(c.in_l, &first)) return false;
    const size_t es = dtype_size(c.in->dtype), os = dtype_size(c.out->dtype);
    f->in = static_cast<const char *>(c.in->ptr) + first * (int64_t)es;
    f->n = c.count;
    f->out = static_cast<char *>(c.out->ptr) + c.out_l.offset * os;
    in->lo = reinterpret_cast<uintptr_t>(f->in);
    in->hi = in->lo + c.count * es;
    out->lo = reinterpret_cast<uintptr_t>(f->out);
    out->hi = out->lo + os;
    return true;
}

}  // namespace

struct heph_batch {
    heph_device *device = nullptr;
    cudaStream_t capture = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    std::vector<Segment> segments;
    void *fused_mem = nullptr;  // fused runs' tables, partials and tickets
};

extern "C" heph_status heph_batch_create(heph_device *device, const heph_prepared *const *items, uint32_t count,
                                         heph_batch **out) {
    if (!device || !out || (count && !items)) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    *out = nullptr;
    for (uint32_t i = 0; i < count; ++i) {
        if (!items[i]) return fail(HEPH_INVALID_CONFIGURATION, "null prepared item");
        if (items[i]->call.kind == Kind::Scan)
            return fail(HEPH_INVALID_CONFIGURATION, "prepared scans cannot be batched; dispatch them directly");
        if (items[i]->call.in->device != device)
            return fail(HEPH_DISPATCH_FAILED, "prepared operands belong to another device");
    }
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    heph_batch *b = new heph_batch();
    b->device = device;
    auto cleanup = [&](heph_status s) {
        if (b->exec) cudaGraphExecDestroy(b->exec);
        if (b->graph) cudaGraphDestroy(b->graph);
        if (b->capture) cudaStreamDestroy(b->capture);
        if (b->fused_mem) cudaFree(b->fused_mem);
        delete b;
        return s;
    };

    // Segments: maximal hazard-free runs of fusable full reductions sharing
    // (operator, input type, output type); everything else one item each.
    std::vector<std::vector<FusedFull>> tables;
    for (uint32_t i = 0; i < count;) {
        Segment seg;
        seg.first = i;
        FusedFull f{};
        ByteRange rin{}, rout{};
        if (fusable_full(items[i]->call, &f, &rin, &rout)) {
            const Call &c0 = items[i]->call;
            std::vector<FusedFull> table{f};
            std::vector<ByteRange> ins{rin}, outs{rout};
            uint32_t j = i + 1;
            for (; j < count; ++j) {
                const Call &c = items[j]->call;
                if (c.op != c0.op || c.in->dtype != c0.in->dtype || c.out->dtype != c0.out->dtype) break;
                if (!fusable_full(c, &f, &rin, &rout)) break;
                bool hazard = rout.overlaps(rin);
                for (size_t k = 0; k < ins.size() && !hazard; ++k)
                    hazard = rout.overlaps(ins[k]) || rout.overlaps(outs[k]) || outs[k].overlaps(rin);
                if (hazard) break;
                table.push_back(f);
                ins.push_back(rin);
                outs.push_back(rout);
            }
            if (j - i >= 2) {
                seg.count = j - i;
                seg.fused = true;
                tables.push_back(std::move(table));
            }
        }
        i = seg.first + seg.count;
        b->segments.push_back(seg);
    }
    if (!tables.empty()) {
        auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
        size_t bytes = 0, t = 0;
        for (Segment &seg : b->segments) {
            if (!seg.fused) continue;
            std::vector<FusedFull> &table = tables[t++];
            seg.grid = plan_reduce_full_fused(device, items[seg.first]->call.in->dtype, table.data(), seg.count);
            seg.table_off = bytes;
            bytes += up(seg.count * sizeof(FusedFull));
            seg.partials_off = bytes;
            bytes += up((size_t)seg.grid * sizeof(double));
            seg.tickets_off = bytes;
            bytes += up(seg.count * sizeof(unsigned int));
        }
        if (cudaMalloc(&b->fused_mem, bytes) != cudaSuccess)
            return cleanup(cuda_fail(HEPH_ALLOCATION_FAILED, cudaGetLastError(), "batch tables"));
        if (cudaMemset(b->fused_mem, 0, bytes) != cudaSuccess)
            return cleanup(cuda_fail(HEPH_DISPATCH_FAILED, cudaGetLastError(), "batch tables"));
        t = 0;
        for (Segment &seg : b->segments) {
            if (!seg.fused) continue;
            std::vector<FusedFull> &table = tables[t++];
            if (cudaMemcpy(static_cast<char *>(b->fused_mem) + seg.table_off, table.data(),
                           seg.count * sizeof(FusedFull), cudaMemcpyHostToDevice) != cudaSuccess)
                return cleanup(cuda_fail(HEPH_TRANSFER_FAILED, cudaGetLastError(), "batch tables"));
        }
    }
    auto enqueue = [&](cudaStream_t s) -> heph_status {
        for (const Segment &seg : b->segments) {
            heph_status r;
            if (seg.fused) {
                const Call &c = items[seg.first]->call;
                char *m = static_cast<char *>(b->fused_mem);
                r = launch_reduce_full_fused(s, c.op, c.in->dtype, c.out->dtype,
                                             reinterpret_cast<const FusedFull *>(m + seg.table_off), seg.count,
                                             seg.grid, m + seg.partials_off,
                                             reinterpret_cast<unsigned int *>(m + seg.tickets_off));
            } else {
                r = run(device, items[seg.first]->call, s);
            }
            if (r != HEPH_OK) return r;
        }
        return HEPH_OK;
    };

    if (cudaStreamCreateWithFlags(&b->capture, cudaStreamNonBlocking) != cudaSuccess)
        return cleanup(cuda_fail(HEPH_DISPATCH_FAILED, cudaGetLastError(), "batch stream"));
    // One eager pass sets up the capture stream's workspace, so that the
    // captured launches allocate nothing.
    st = enqueue(b->capture);
    if (st != HEPH_OK) return cleanup(st);
    if (cudaStreamSynchronize(b->capture) != cudaSuccess)
        return cleanup(cuda_fail(HEPH_DISPATCH_FAILED, cudaGetLastError(), "batch warm-up"));
    if (cudaStreamBeginCapture(b->capture, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return cleanup(cuda_fail(HEPH_DISPATCH_FAILED, cudaGetLastError(), "batch capture"));
    st = enqueue(b->capture);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(b->capture, &g);
    b->graph = g;
    if (st != HEPH_OK) return cleanup(st);
    if (e != cudaSuccess) return cleanup(cuda_fail(HEPH_DISPATCH_FAILED, e, "batch capture"));
    e = cudaGraphInstantiate(&b->exec, b->graph, 0);
    if (e != cudaSuccess) return cleanup(cuda_fail(HEPH_DISPATCH_FAILED, e, "batch instantiate"));
    *out = b;
    return HEPH_OK;
}

extern "C" heph_status heph_batch_launch(heph_batch *batch, heph_stream stream) {
    if (!batch) return fail(HEPH_INVALID_CONFIGURATION, "null batch");
    heph_status st = bind(batch->device);
    if (st != HEPH_OK) return st;
    HEPH_CUDA_TRY(cudaGraphLaunch(batch->exec, resolve_stream(batch->device, stream)), HEPH_DISPATCH_FAILED,
                  "batch launch");
    return HEPH_OK;
}

extern "C" heph_status heph_batch_free(heph_batch *batch) {
    if (!batch) return HEPH_OK;
    cudaSetDevice(batch->device->ordinal);
    if (batch->exec) cudaGraphExecDestroy(batch->exec);
    if (batch->graph) cudaGraphDestroy(batch->graph);
    if (batch->capture) {
        cudaStreamSynchronize(batch->capture);
        cudaStreamDestroy(batch->capture);
    }
    if (batch->fused_mem) {
        cudaDeviceSynchronize();  // a replay on another stream may still read the tables
        cudaFree(batch->fused_mem);
    }
    delete batch;
    return HEPH_OK;
}
