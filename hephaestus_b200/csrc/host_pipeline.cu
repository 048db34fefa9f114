// host_pipeline.cu — scan of a host-resident buffer with the transfers
// overlapped: the reference's path for host data is upload -> scan -> download
// (ComputeDevice::upload / ScanOps::scan_axis_into / download,
// crates/hephaestus-core/src/domain/device.rs:135,147, scan.rs:219), three
// serial phases.  Here the buffer is cut into chunks that flow through a ring
// of device slots on three streams: host->device copies on one copy engine,
// the seeded single-pass scans on the device's stream, device->host copies on
// the other copy engine.  Chunk k is seeded with the running total after
// chunk k-1, kept on the device by a one-thread kernel, so the result equals
// the whole-buffer scan and no host synchronisation happens between chunks.
#include <algorithm>
#include <cstring>
#include <utility>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace heph {
namespace {

// carry = running total after a chunk whose scan output ends in `last_out`
// and whose input ends in `last_in`.
template <typename T, int OP>
__global__ void carry_after_chunk(const T *last_out, const T *last_in, int exclusive, T *carry) {
    *carry = exclusive ? combine<T, OP>(*last_out, *last_in) : *last_out;
}

// acc = part (first chunk) or combine(acc, part): the running reduction of
// the chunks so far, folded in chunk order.
template <typename Tacc>
__global__ void fold_chunk_partial(Tacc *acc, const Tacc *part, int op, int first) {
    Tacc v = *part;
    if (!first) {
        const Tacc a = *acc;
        switch (op) {
            case OP_SUM: v = combine<Tacc, OP_SUM>(a, v); break;
            case OP_PROD: v = combine<Tacc, OP_PROD>(a, v); break;
            case OP_MIN: v = combine<Tacc, OP_MIN>(a, v); break;
            default: v = combine<Tacc, OP_MAX>(a, v); break;
        }
    }
    *acc = v;
}

// Optional full reduction of the same host input, computed chunk by chunk
// while the scan pipeline runs.
struct HostReduce {
    int op = -1;  // -1: none
    heph_dtype acc = HEPH_F32;
    void *host_out = nullptr;
};

constexpr int kSlots = 3;

// Piece boundaries of the pipeline: full chunks in the middle, and at each
// end pieces of 1/8, 1/4, 1/2 chunk, so the lone first upload and the lone
// last download (nothing to overlap them with) are short.
std::vector<std::pair<uint64_t, uint64_t>> pipeline_pieces(uint64_t n, uint64_t chunk) {
    std::vector<std::pair<uint64_t, uint64_t>> pieces;
    const uint64_t ramp[3] = {std::max<uint64_t>(1, chunk / 8), std::max<uint64_t>(1, chunk / 4),
                              std::max<uint64_t>(1, chunk / 2)};
    const uint64_t ramp_total = ramp[0] + ramp[1] + ramp[2];
    if (n < 2 * ramp_total + 2 * chunk) {  // short input: plain chunks
        for (uint64_t off = 0; off < n; off += chunk) pieces.push_back({off, std::min(chunk, n - off)});
        return pieces;
    }
    uint64_t off = 0;
    for (uint64_t r : ramp) {
        pieces.push_back({off, r});
        off += r;
    }
    const uint64_t middle_end = n - ramp_total;
    while (off < middle_end) {
        const uint64_t len = std::min(chunk, middle_end - off);
        pieces.push_back({off, len});
        off += len;
    }
    for (int k = 2; k >= 0; --k) {
        pieces.push_back({off, ramp[k]});
        off += ramp[k];
    }
    return pieces;
}

struct PipelineStreams {
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaEvent_t loaded[kSlots] = {}, scanned[kSlots] = {}, drained[kSlots] = {};
    ~PipelineStreams() {
        for (int s = 0; s < kSlots; ++s) {
            if (loaded[s]) cudaEventDestroy(loaded[s]);
            if (scanned[s]) cudaEventDestroy(scanned[s]);
            if (drained[s]) cudaEventDestroy(drained[s]);
        }
        if (h2d) cudaStreamDestroy(h2d);
        if (d2h) cudaStreamDestroy(d2h);
    }
};

template <typename T, int OP>
heph_status scan_host_typed(Device *dev, int exclusive, const T *host_in, T *host_out, uint64_t n, uint64_t chunk,
                            const HostReduce &red) {
    cudaStream_t cs = dev->stream;
    PipelineStreams ps;
    HEPH_CUDA_TRY(cudaStreamCreateWithFlags(&ps.h2d, cudaStreamNonBlocking), HEPH_DISPATCH_FAILED, "stream");
    HEPH_CUDA_TRY(cudaStreamCreateWithFlags(&ps.d2h, cudaStreamNonBlocking), HEPH_DISPATCH_FAILED, "stream");
    for (int s = 0; s < kSlots; ++s) {
        HEPH_CUDA_TRY(cudaEventCreateWithFlags(&ps.loaded[s], cudaEventDisableTiming), HEPH_DISPATCH_FAILED, "event");
        HEPH_CUDA_TRY(cudaEventCreateWithFlags(&ps.scanned[s], cudaEventDisableTiming), HEPH_DISPATCH_FAILED, "event");
        HEPH_CUDA_TRY(cudaEventCreateWithFlags(&ps.drained[s], cudaEventDisableTiming), HEPH_DISPATCH_FAILED, "event");
    }
    // Slots: [in chunk][out chunk] per slot, one carry element, then (with a
    // reduction) the chunk's partial and the running reduction, 8 bytes each.
    const uint64_t slots = std::min<uint64_t>(kSlots, (n + chunk - 1) / chunk);
    const uint64_t carry_bytes = (2 * slots * chunk + 1) * sizeof(T);
    const uint64_t red_off = (carry_bytes + 7) / 8 * 8;
    T *mem = nullptr;
    HEPH_CUDA_TRY(cudaMallocFromPoolAsync((void **)&mem, red_off + 16, dev->pool, cs),
                  HEPH_ALLOCATION_FAILED, "pipeline staging allocation");
    T *carry = mem + 2 * slots * chunk;
    void *red_part = reinterpret_cast<char *>(mem) + red_off;
    void *red_acc = reinterpret_cast<char *>(mem) + red_off + 8;
    // The copy streams must not touch the staging memory before it exists.
    cudaEvent_t ready;
    HEPH_CUDA_TRY(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming), HEPH_DISPATCH_FAILED, "event");
    cudaEventRecord(ready, cs);
    cudaStreamWaitEvent(ps.h2d, ready, 0);
    cudaEventDestroy(ready);

    heph_status st = HEPH_OK;
    const auto pieces = pipeline_pieces(n, chunk);
    for (uint64_t k = 0; k < pieces.size() && st == HEPH_OK; ++k) {
        const int s = (int)(k % slots);
        const uint64_t off = pieces[k].first, len = pieces[k].second;
        T *din = mem + (uint64_t)s * 2 * chunk, *dout = din + chunk;
        if (k >= slots) cudaStreamWaitEvent(ps.h2d, ps.drained[s], 0);  // slot's previous chunk is out
        if (cudaMemcpyAsync(din, host_in + off, len * sizeof(T), cudaMemcpyHostToDevice, ps.h2d) != cudaSuccess) {
            st = cuda_fail(HEPH_TRANSFER_FAILED, cudaGetLastError(), "host-to-device copy");
            break;
        }
        cudaEventRecord(ps.loaded[s], ps.h2d);
        cudaStreamWaitEvent(cs, ps.loaded[s], 0);
        AxisProblem p{};
        p.outer = 1;
        p.len = len;
        p.in_r = p.out_r = 1;
        st = launch_scan(dev, cs, OP, DtypeOf<T>::value, din, dout, p, false, exclusive != 0, k ? carry : nullptr);
        if (st != HEPH_OK) break;
        if (red.op >= 0) {
            heph_layout l{};
            l.rank = 1;
            l.shape[0] = len;
            l.strides[0] = 1;
            st = launch_reduce_full(dev, cs, red.op, DtypeOf<T>::value, red.acc, din, l, len, red_part);
            if (st != HEPH_OK) break;
            st = dispatch_dtype(red.acc, [&]<typename A>() -> heph_status {
                fold_chunk_partial<A><<<1, 1, 0, cs>>>(static_cast<A *>(red_acc), static_cast<const A *>(red_part),
                                                       red.op, k == 0);
                return HEPH_OK;
            });
            if (st != HEPH_OK) break;
        }
        carry_after_chunk<T, OP><<<1, 1, 0, cs>>>(dout + len - 1, din + len - 1, exclusive, carry);
        cudaEventRecord(ps.scanned[s], cs);
        cudaStreamWaitEvent(ps.d2h, ps.scanned[s], 0);
        if (cudaMemcpyAsync(host_out + off, dout, len * sizeof(T), cudaMemcpyDeviceToHost, ps.d2h) != cudaSuccess) {
            st = cuda_fail(HEPH_TRANSFER_FAILED, cudaGetLastError(), "device-to-host copy");
            break;
        }
        cudaEventRecord(ps.drained[s], ps.d2h);
    }
    if (st == HEPH_OK && red.op >= 0 &&
        cudaMemcpyAsync(red.host_out, red_acc, dtype_size(red.acc), cudaMemcpyDeviceToHost, cs) != cudaSuccess)
        st = cuda_fail(HEPH_TRANSFER_FAILED, cudaGetLastError(), "device-to-host copy of the reduction");
    cudaError_t e1 = cudaStreamSynchronize(ps.d2h), e2 = cudaStreamSynchronize(ps.h2d);
    cudaFreeAsync(mem, cs);
    cudaError_t e3 = cudaStreamSynchronize(cs);
    if (st != HEPH_OK) return st;
    if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess)
        return cuda_fail(HEPH_TRANSFER_FAILED, e1 != cudaSuccess ? e1 : e2 != cudaSuccess ? e2 : e3, "pipelined scan");
    return HEPH_OK;
}

}  // namespace
}  // namespace heph

using namespace heph;

namespace heph {
namespace {

heph_status scan_host_entry(heph_device *device, heph_op op, int exclusive, heph_dtype dtype, const void *host_in,
                            void *host_out, uint64_t count, uint64_t chunk_elems, const HostReduce &red) {
    if (!device) return fail(HEPH_INVALID_CONFIGURATION, "null device");
    if (count && (!host_in || !host_out)) return fail(HEPH_INVALID_CONFIGURATION, "null host pointer");
    if (op != HEPH_SUM && op != HEPH_PROD)
        return fail(HEPH_INVALID_CONFIGURATION, "scans support the sum (cumsum) and product (cumprod) operators");
    if (!dtype_valid(dtype)) return fail(HEPH_INVALID_CONFIGURATION, "unknown element type");
    if (host_in == host_out && count) return fail(HEPH_DISPATCH_FAILED, "scan output buffer must not alias input buffer");
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    if (count == 0) {
        if (red.op < 0) return HEPH_OK;
        // The empty reduction is the operator's identity.
        return dispatch_dtype(red.acc, [&]<typename A>() -> heph_status {
            A v{};
            switch (red.op) {
                case OP_SUM: v = identity<A, OP_SUM>(); break;
                case OP_PROD: v = identity<A, OP_PROD>(); break;
                case OP_MIN: v = identity<A, OP_MIN>(); break;
                default: v = identity<A, OP_MAX>(); break;
            }
            std::memcpy(red.host_out, &v, sizeof(A));
            return HEPH_OK;
        });
    }
    const uint64_t chunk = chunk_elems ? chunk_elems : (64ull << 20) / dtype_size(dtype);
    return dispatch_dtype(dtype, [&]<typename T>() -> heph_status {
        if (op == HEPH_SUM)
            return scan_host_typed<T, OP_SUM>(device, exclusive, static_cast<const T *>(host_in),
                                              static_cast<T *>(host_out), count, chunk, red);
        return scan_host_typed<T, OP_PROD>(device, exclusive, static_cast<const T *>(host_in),
                                           static_cast<T *>(host_out), count, chunk, red);
    });
}

}  // namespace
}  // namespace heph

extern "C" heph_status heph_scan_host(heph_device *device, heph_op op, int exclusive, heph_dtype dtype,
                                      const void *host_in, void *host_out, uint64_t count, uint64_t chunk_elems) {
    return scan_host_entry(device, op, exclusive, dtype, host_in, host_out, count, chunk_elems, HostReduce{});
}

extern "C" heph_status heph_scan_reduce_host(heph_device *device, heph_op scan_op, int exclusive, heph_dtype dtype,
                                             const void *host_in, void *host_out, uint64_t count, heph_op reduce_op,
                                             heph_dtype acc_dtype, void *host_reduce_out, uint64_t chunk_elems) {
    if (!host_reduce_out) return fail(HEPH_INVALID_CONFIGURATION, "null host pointer");
    if (reduce_op != HEPH_SUM && reduce_op != HEPH_PROD && reduce_op != HEPH_MIN && reduce_op != HEPH_MAX)
        return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
    const bool widen = (dtype == HEPH_I32 && acc_dtype == HEPH_I64) || (dtype == HEPH_F32 && acc_dtype == HEPH_F64);
    if (acc_dtype != dtype && !widen)
        return fail(HEPH_INVALID_CONFIGURATION,
                    "full reduction output type must match the input type or widen it (i32->i64, f32->f64)");
    HostReduce red;
    red.op = (int)reduce_op;
    red.acc = acc_dtype;
    red.host_out = host_reduce_out;
    return scan_host_entry(device, scan_op, exclusive, dtype, host_in, host_out, count, chunk_elems, red);
}
