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
heph_status scan_host_typed(Device *dev, int exclusive, const T *host_in, T *host_out, uint64_t n, uint64_t chunk) {
    cudaStream_t cs = dev->stream;
    PipelineStreams ps;
    HEPH_CUDA_TRY(cudaStreamCreateWithFlags(&ps.h2d, cudaStreamNonBlocking), HEPH_DISPATCH_FAILED, "stream");
    HEPH_CUDA_TRY(cudaStreamCreateWithFlags(&ps.d2h, cudaStreamNonBlocking), HEPH_DISPATCH_FAILED, "stream");
    for (int s = 0; s < kSlots; ++s) {
        HEPH_CUDA_TRY(cudaEventCreateWithFlags(&ps.loaded[s], cudaEventDisableTiming), HEPH_DISPATCH_FAILED, "event");
        HEPH_CUDA_TRY(cudaEventCreateWithFlags(&ps.scanned[s], cudaEventDisableTiming), HEPH_DISPATCH_FAILED, "event");
        HEPH_CUDA_TRY(cudaEventCreateWithFlags(&ps.drained[s], cudaEventDisableTiming), HEPH_DISPATCH_FAILED, "event");
    }
    // Slots: [in chunk][out chunk] per slot, plus one carry element.
    const uint64_t slots = std::min<uint64_t>(kSlots, (n + chunk - 1) / chunk);
    T *mem = nullptr;
    HEPH_CUDA_TRY(cudaMallocFromPoolAsync((void **)&mem, (2 * slots * chunk + 1) * sizeof(T), dev->pool, cs),
                  HEPH_ALLOCATION_FAILED, "pipeline staging allocation");
    T *carry = mem + 2 * slots * chunk;
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
        carry_after_chunk<T, OP><<<1, 1, 0, cs>>>(dout + len - 1, din + len - 1, exclusive, carry);
        cudaEventRecord(ps.scanned[s], cs);
        cudaStreamWaitEvent(ps.d2h, ps.scanned[s], 0);
        if (cudaMemcpyAsync(host_out + off, dout, len * sizeof(T), cudaMemcpyDeviceToHost, ps.d2h) != cudaSuccess) {
            st = cuda_fail(HEPH_TRANSFER_FAILED, cudaGetLastError(), "device-to-host copy");
            break;
        }
        cudaEventRecord(ps.drained[s], ps.d2h);
    }
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

extern "C" heph_status heph_scan_host(heph_device *device, heph_op op, int exclusive, heph_dtype dtype,
                                      const void *host_in, void *host_out, uint64_t count, uint64_t chunk_elems) {
    if (!device) return fail(HEPH_INVALID_CONFIGURATION, "null device");
    if (count && (!host_in || !host_out)) return fail(HEPH_INVALID_CONFIGURATION, "null host pointer");
    if (op != HEPH_SUM && op != HEPH_PROD)
        return fail(HEPH_INVALID_CONFIGURATION, "scans support the sum (cumsum) and product (cumprod) operators");
    if (!dtype_valid(dtype)) return fail(HEPH_INVALID_CONFIGURATION, "unknown element type");
    if (host_in == host_out && count) return fail(HEPH_DISPATCH_FAILED, "scan output buffer must not alias input buffer");
    if (count == 0) return HEPH_OK;
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    const uint64_t chunk = chunk_elems ? chunk_elems : (64ull << 20) / dtype_size(dtype);
    return dispatch_dtype(dtype, [&]<typename T>() -> heph_status {
        if (op == HEPH_SUM)
            return scan_host_typed<T, OP_SUM>(device, exclusive, static_cast<const T *>(host_in),
                                              static_cast<T *>(host_out), count, chunk);
        return scan_host_typed<T, OP_PROD>(device, exclusive, static_cast<const T *>(host_in),
                                           static_cast<T *>(host_out), count, chunk);
    });
}
