// scan.cu — prefix scans for sm_100a.
//
// The reference scans each line with ONE block of 256 threads in which every
// lane walks a private contiguous chunk, lane 0 folds the chunk totals
// serially, and a second pass re-reads and rewrites the output
// (core accelerator/scan.rs:94-147): a 1-D vector runs on a single SM and
// moves 4N elements.  Here a line that is contiguous along the scan axis is
// scanned by a single-pass decoupled look-back (Merrill & Garland, "Single-pass
// Parallel Prefix Scan with Decoupled Look-back", NVIDIA TR 2016):
//   * each CTA draws its tile id from an atomic counter (so every
//     predecessor of a running tile has already started: forward progress
//     does not depend on block scheduling order), loads its 16 KiB tile with
//     128-bit streaming loads (4 vectors in flight per thread), scans it in
//     registers (thread-local, then warp shuffles, then the 8 warp totals);
//   * publishes its aggregate, looks back over its predecessors one warp
//     window (32 tiles) at a time, publishes its inclusive prefix and writes
//     the tile with 128-bit stores: 2N elements of traffic in one launch;
//   * tile status words carry an epoch tag so the status array never needs
//     clearing between calls; 4-byte element types pack (value, flag) in one
//     64-bit word, 8-byte types use a flag word with release/acquire ordering;
//   * every look-back wait is bounded: when it runs out the tile raises a
//     device error bit (reported by synchronize as DispatchFailed), publishes
//     a prefix anyway so its successors do not wait in turn, and finishes.
// Reverse scans process the same physical tiles from the last one backwards
// and mirror every intra-tile step.  Lines whose scan axis is not unit-stride
// (column scans, transposed views) take a warp-per-line kernel that walks the
// line in 32-element chunks with a warp scan and a running carry.
#include <algorithm>

#include "device_utils.cuh"
#include "kernels.h"

namespace heph {

constexpr int kScanThreads = 256;
constexpr int kScanWarps = kScanThreads / 32;
constexpr uint32_t kLookbackPolls = 1u << 20;

template <typename T> struct ScanShape {
    static constexpr int V = 16 / sizeof(T);  // elements per 128-bit vector
    static constexpr int J = 4;               // vectors per thread
    static constexpr int WARP_ITEMS = 32 * V * J;
    static constexpr int TILE = kScanThreads * V * J;  // 16 KiB
};

enum : uint32_t { kStateInvalid = 0, kStateAggregate = 1, kStatePrefix = 2 };

template <typename T> struct ScanParams {
    const T *in;
    T *out;
    uint64_t len;             // elements per line
    uint64_t tiles_per_line;
    int64_t in_line, out_line;  // element distance between line starts
    unsigned long long *tile_counter;
    unsigned long long tile_base;
    uint32_t epoch;
    unsigned long long *packed;  // 4-byte T: (value << 32) | flag
    uint32_t *flags;             // 8-byte T: flag words
    T *aggs, *incls;             // 8-byte T: values
    const T *carry;              // nullable seed of line 0
    unsigned int *err;
    int reverse, exclusive;
};

template <typename T>
__device__ __forceinline__ void publish(const ScanParams<T> &p, uint64_t tile, uint32_t state,
                                        T value) {
    const uint32_t f = (p.epoch << 2) | state;
    if constexpr (sizeof(T) == 4) {
        const unsigned long long w =
            ((unsigned long long)bitcast<uint32_t>(value) << 32) | f;
        asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p.packed + tile), "l"(w)
                     : "memory");
    } else {
        T *dst = (state == kStatePrefix ? p.incls : p.aggs) + tile;
        asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(dst),
                     "l"(bitcast<unsigned long long>(value))
                     : "memory");
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p.flags + tile), "r"(f)
                     : "memory");
    }
}

template <typename T>
__device__ __forceinline__ void read_status(const ScanParams<T> &p, uint64_t tile,
                                            uint32_t &state, T &value) {
    if constexpr (sizeof(T) == 4) {
        unsigned long long w;
        asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p.packed + tile) : "memory");
        const uint32_t f = (uint32_t)w;
        state = ((f >> 2) == p.epoch) ? (f & 3u) : kStateInvalid;
        value = bitcast<T>((uint32_t)(w >> 32));
    } else {
        uint32_t f;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(f) : "l"(p.flags + tile) : "memory");
        state = ((f >> 2) == p.epoch) ? (f & 3u) : kStateInvalid;
        if (state != kStateInvalid) {
            const T *src = (state == kStatePrefix ? p.incls : p.aggs) + tile;
            unsigned long long v;
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
            value = bitcast<T>(v);
        }
    }
}

// Exclusive prefix of `tile` within its line: fold of the predecessors back to
// the nearest one that has published its inclusive prefix.  Runs on one warp.
template <typename T, int OP>
__device__ T lookback(const ScanParams<T> &p, uint64_t tile, uint64_t line_first, int lane,
                      bool *timed_out) {
    T excl = identity<T, OP>();
    int64_t cur = (int64_t)tile - 1;
    uint32_t polls = 0;
    while (true) {
        const int64_t idx = cur - lane;
        const bool in_range = idx >= (int64_t)line_first;
        uint32_t state = kStatePrefix;  // lanes before the line start act as an identity prefix
        T val = identity<T, OP>();
        if (in_range) read_status(p, (uint64_t)idx, state, val);
        while (__any_sync(kFullMask, state == kStateInvalid)) {
            if (++polls > kLookbackPolls) {
                if (lane == 0) raise_device_error(p.err, DEVERR_LOOKBACK_TIMEOUT);
                *timed_out = true;
                return excl;
            }
            __nanosleep(64);
            if (state == kStateInvalid) read_status(p, (uint64_t)idx, state, val);
        }
        const unsigned pm = __ballot_sync(kFullMask, state == kStatePrefix);
        const int stop = pm ? __ffs(pm) - 1 : 31;
        T v = lane <= stop ? val : identity<T, OP>();
        v = warp_fold<T, OP>(v);
        excl = combine<T, OP>(v, excl);
        if (pm) return excl;
        cur -= 32;
    }
}

// Inclusive warp scan in logical lane order (descending lanes when `rev`).
template <typename T, int OP> __device__ __forceinline__ T warp_scan(T v, int lane, bool rev) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const T o = rev ? shfl_down(v, d) : shfl_up(v, d);
        const bool ok = rev ? (lane + d < 32) : (lane >= d);
        if (ok) v = combine<T, OP>(o, v);
    }
    return v;
}

template <typename T, int OP, bool VEC>
__global__ void __launch_bounds__(kScanThreads) scan_lookback_kernel(const ScanParams<T> p) {
    using S = ScanShape<T>;
    constexpr int V = S::V, J = S::J, TILE = S::TILE;
    __shared__ unsigned long long s_tile;
    __shared__ T s_warp[kScanWarps];
    __shared__ T s_prefix;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_tile = atomicAdd(p.tile_counter, 1ull) - p.tile_base;
    __syncthreads();
    const uint64_t tile = s_tile;
    const uint64_t line = tile / p.tiles_per_line;
    const uint64_t t_in_line = tile - line * p.tiles_per_line;
    const bool rev = p.reverse != 0;
    const uint64_t ptile = rev ? p.tiles_per_line - 1 - t_in_line : t_in_line;
    const T *lin = p.in + (int64_t)line * p.in_line;
    T *lout = p.out + (int64_t)line * p.out_line;
    const uint64_t start = ptile * (uint64_t)TILE;
    const uint64_t valid = min((uint64_t)TILE, p.len - start);
    const bool full = VEC && valid == (uint64_t)TILE;
    // Physical position in the tile of this thread's element (j, c):
    // base + j*32*V + c — warp-striped 128-bit vectors, coalesced per j.
    const int base = warp * S::WARP_ITEMS + lane * V;

    T x[J][V];
    if (full) {
        uint4 raw[J];
#pragma unroll
        for (int j = 0; j < J; ++j)
            raw[j] = ld_stream(reinterpret_cast<const uint4 *>(lin + start + base + j * 32 * V));
#pragma unroll
        for (int j = 0; j < J; ++j) {
            Vec16<T> e = as_elems<T>(raw[j]);
#pragma unroll
            for (int c = 0; c < V; ++c) x[j][c] = e.e[c];
        }
    } else {
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int c = 0; c < V; ++c) {
                const uint64_t pos = (uint64_t)(base + j * 32 * V + c);
                x[j][c] = pos < valid ? lin[start + pos] : identity<T, OP>();
            }
    }

    // Inclusive scan inside each vector, in logical order.
    T tt[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        if (!rev) {
#pragma unroll
            for (int c = 1; c < V; ++c) x[j][c] = combine<T, OP>(x[j][c - 1], x[j][c]);
            tt[j] = x[j][V - 1];
        } else {
#pragma unroll
            for (int c = V - 2; c >= 0; --c) x[j][c] = combine<T, OP>(x[j][c + 1], x[j][c]);
            tt[j] = x[j][0];
        }
    }

    // Warp scans of the vector totals, chunk by chunk in logical order.
    T pre[J];
    T running = identity<T, OP>();
    const bool first_lane = rev ? (lane == 31) : (lane == 0);
#pragma unroll
    for (int jl = 0; jl < J; ++jl) {
        const int jp = rev ? J - 1 - jl : jl;
        const T inc = warp_scan<T, OP>(tt[jp], lane, rev);
        T exc = rev ? shfl_down(inc, 1) : shfl_up(inc, 1);
        if (first_lane) exc = identity<T, OP>();
        const T tot = shfl_idx(inc, rev ? 0 : 31);
        pre[jp] = combine<T, OP>(running, exc);
        running = combine<T, OP>(running, tot);
    }

    // Block: fold the warp totals in logical warp order.
    if (lane == 0) s_warp[warp] = running;
    __syncthreads();
    T wpre = identity<T, OP>(), agg = identity<T, OP>();
#pragma unroll
    for (int wl = 0; wl < kScanWarps; ++wl) {
        const int wp = rev ? kScanWarps - 1 - wl : wl;
        if (wp == warp) wpre = agg;
        agg = combine<T, OP>(agg, s_warp[wp]);
    }

    // Tile prefix: seed for the first tile of a line, look-back otherwise.
    if (warp == 0) {
        T tp;
        if (t_in_line == 0) {
            tp = (p.carry != nullptr && line == 0) ? *p.carry : identity<T, OP>();
            if (lane == 0) publish(p, tile, kStatePrefix, combine<T, OP>(tp, agg));
        } else {
            if (lane == 0) publish(p, tile, kStateAggregate, agg);
            bool timed_out = false;
            tp = lookback<T, OP>(p, tile, tile - t_in_line, lane, &timed_out);
            if (lane == 0) publish(p, tile, kStatePrefix, combine<T, OP>(tp, agg));
        }
        if (lane == 0) s_prefix = tp;
    }
    __syncthreads();
    const T thread_base = combine<T, OP>(s_prefix, wpre);

    // Outputs.
    T y[J][V];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const T tpj = combine<T, OP>(thread_base, pre[j]);
#pragma unroll
        for (int c = 0; c < V; ++c) {
            if (p.exclusive) {
                const bool first = rev ? (c == V - 1) : (c == 0);
                const T prev = rev ? x[j][(c + 1) % V] : x[j][(c + V - 1) % V];
                y[j][c] = first ? tpj : combine<T, OP>(tpj, prev);
            } else {
                y[j][c] = combine<T, OP>(tpj, x[j][c]);
            }
        }
    }
    if (full) {
#pragma unroll
        for (int j = 0; j < J; ++j) {
            Vec16<T> e;
#pragma unroll
            for (int c = 0; c < V; ++c) e.e[c] = y[j][c];
            *reinterpret_cast<uint4 *>(lout + start + base + j * 32 * V) = as_uint4(e);
        }
    } else {
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int c = 0; c < V; ++c) {
                const uint64_t pos = (uint64_t)(base + j * 32 * V + c);
                if (pos < valid) lout[start + pos] = y[j][c];
            }
    }
}

// ------------------------------------------------ strided / short-line scan

template <typename T> struct StridedScanParams {
    const T *in;
    T *out;
    uint64_t lines, len;
    int64_t in_base, in_o, in_r, out_base, out_o, out_r;
    const T *carry;
    int reverse, exclusive;
};

// One warp per line, 32 logical positions per step.
template <typename T, int OP>
__global__ void __launch_bounds__(256) scan_strided_kernel(const StridedScanParams<T> p) {
    const uint64_t line = ((uint64_t)blockIdx.x * 256 + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (line >= p.lines) return;
    T running = (p.carry != nullptr && line == 0) ? *p.carry : identity<T, OP>();
    const int64_t ib = p.in_base + (int64_t)line * p.in_o;
    const int64_t ob = p.out_base + (int64_t)line * p.out_o;
    for (uint64_t c0 = 0; c0 < p.len; c0 += 32) {
        const uint64_t q = c0 + lane;
        const bool ok = q < p.len;
        const uint64_t idx = p.reverse ? p.len - 1 - q : q;
        const T x = ok ? p.in[ib + (int64_t)idx * p.in_r] : identity<T, OP>();
        const T inc = warp_scan<T, OP>(x, lane, false);
        T exc = shfl_up(inc, 1);
        if (lane == 0) exc = identity<T, OP>();
        if (ok) p.out[ob + (int64_t)idx * p.out_r] = combine<T, OP>(running, p.exclusive ? exc : inc);
        running = combine<T, OP>(running, shfl_idx(inc, 31));
    }
}

// ------------------------------------------------------------------ launch

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T, int OP>
static heph_status launch_scan_typed(Device *dev, cudaStream_t stream, const T *in, T *out,
                                     const AxisProblem &pr, bool reverse, bool exclusive,
                                     const T *carry) {
    using S = ScanShape<T>;
    const bool contiguous = pr.in_r == 1 && pr.out_r == 1;
    if (!contiguous || pr.len < (uint64_t)S::TILE / 2) {
        StridedScanParams<T> sp{in, out, pr.outer, pr.len, pr.in_base, pr.in_o, pr.in_r,
                                pr.out_base, pr.out_o, pr.out_r, carry, reverse, exclusive};
        const uint64_t blocks = (pr.outer * 32 + 255) / 256;
        if (blocks > 0x7fffffffull) return fail(HEPH_DISPATCH_FAILED, "scan grid too large");
        scan_strided_kernel<T, OP><<<(unsigned)blocks, 256, 0, stream>>>(sp);
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "scan launch");
        return HEPH_OK;
    }
    const uint64_t tiles_per_line = (pr.len + S::TILE - 1) / S::TILE;
    const uint64_t tiles = tiles_per_line * pr.outer;
    if (tiles > 0x7fffffffull) return fail(HEPH_DISPATCH_FAILED, "scan grid too large");
    const bool vec = aligned16(in + pr.in_base) && aligned16(out + pr.out_base) &&
                     (pr.outer == 1 || (((uint64_t)pr.in_o * sizeof(T)) % 16 == 0 &&
                                        ((uint64_t)pr.out_o * sizeof(T)) % 16 == 0));

    std::lock_guard<std::mutex> lock(dev->mu);
    Workspace *ws = nullptr;
    // Status layout: [packed u64 x tiles][flags u32 x tiles][aggs 8B x tiles][incls 8B x tiles]
    const size_t status_bytes = (size_t)tiles * (8 + 4 + 8 + 8);
    heph_status st = workspace_for(dev, stream, 0, status_bytes, &ws);
    if (st != HEPH_OK) return st;
    // Epoch tag: flags of earlier calls never match; restart (after clearing)
    // before the 30-bit tag wraps.
    if (ws->epoch >= (1u << 30) - 1) {
        HEPH_CUDA_TRY(cudaMemsetAsync(ws->scan_status, 0, ws->scan_status_bytes, stream),
                      HEPH_DISPATCH_FAILED, "scan status reset");
        ws->epoch = 0;
    }
    ws->epoch += 1;
    char *sbase = static_cast<char *>(ws->scan_status);
    const size_t cap = ws->scan_status_bytes / (8 + 4 + 8 + 8);
    ScanParams<T> p{};
    p.in = in + pr.in_base;
    p.out = out + pr.out_base;
    p.len = pr.len;
    p.tiles_per_line = tiles_per_line;
    p.in_line = pr.in_o;
    p.out_line = pr.out_o;
    p.tile_counter = ws->tile_counter;
    p.tile_base = ws->tiles_drawn;
    p.epoch = ws->epoch;
    p.packed = reinterpret_cast<unsigned long long *>(sbase);
    p.flags = reinterpret_cast<uint32_t *>(sbase + cap * 8);
    p.aggs = reinterpret_cast<T *>(sbase + cap * 12);
    p.incls = reinterpret_cast<T *>(sbase + cap * 20);
    p.carry = carry;
    p.err = dev->error_dev;
    p.reverse = reverse;
    p.exclusive = exclusive;
    if (vec)
        scan_lookback_kernel<T, OP, true><<<(unsigned)tiles, kScanThreads, 0, stream>>>(p);
    else
        scan_lookback_kernel<T, OP, false><<<(unsigned)tiles, kScanThreads, 0, stream>>>(p);
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "scan launch");
    ws->tiles_drawn += tiles;
    return HEPH_OK;
}

heph_status launch_scan(Device *dev, cudaStream_t stream, int op, heph_dtype dtype,
                        const void *in, void *out, const AxisProblem &p, bool reverse,
                        bool exclusive, const void *carry) {
    return dispatch_dtype(dtype, [&]<typename T>() -> heph_status {
        const T *ti = static_cast<const T *>(in);
        T *to = static_cast<T *>(out);
        const T *tc = static_cast<const T *>(carry);
        if (op == OP_SUM) return launch_scan_typed<T, OP_SUM>(dev, stream, ti, to, p, reverse, exclusive, tc);
        if (op == OP_PROD) return launch_scan_typed<T, OP_PROD>(dev, stream, ti, to, p, reverse, exclusive, tc);
        return fail(HEPH_INVALID_CONFIGURATION, "scans support the sum (cumsum) and product (cumprod) operators");
    });
}

}  // namespace heph
