// scan.cu — prefix scans for sm_100a.
//
// The reference scans each line with ONE block of 256 threads in which every
// lane walks a private contiguous chunk, lane 0 folds the chunk totals
// serially, and a second pass re-reads and rewrites the output
// (core accelerator/scan.rs:94-147): a 1-D vector runs on a single SM and
// moves 4N elements.  Three kernels replace it, chosen by the shape of the
// problem:
//
// * scan_chunked_kernel — one long contiguous line (the 1-D case).  A
//   co-resident (cooperative) grid of G CTAs walks the line in chunks of G
//   parts.  Each CTA keeps three of its parts in shared memory, filled by TMA
//   bulk copies, so ~100 KiB of input per SM is always in flight.  Per chunk
//   it reduces its next part, publishes the part's total, folds the totals of
//   the parts before its own, scans its part from
//   shared memory and streams the results out.  HBM moves each element
//   exactly twice and the only cross-CTA exchange is G totals per chunk.
// * scan_lookback_kernel — contiguous lines too short (or too many) for the
//   chunked kernel: single-pass decoupled look-back (Merrill & Garland,
//   "Single-pass Parallel Prefix Scan with Decoupled Look-back", NVIDIA TR
//   2016), one 32 KiB tile per CTA, tile id = blockIdx.x (blocks of a grid are
//   dispatched in increasing order, so every predecessor of a running tile has
//   been dispatched).  Measured on B200 the tile-prefix chain across the two
//   dies bounds it near 3.5 TB/s for one long line, hence the chunked kernel.
// * scan_strided_kernel — non-unit-stride scan axes (column scans, transposed
//   views): one warp per line, 32 logical positions per step.
//
// All device-side waits are bounded: when a wait runs out the kernel raises a
// device error bit (reported by synchronize as DispatchFailed), substitutes
// the identity and finishes, so a fault never turns into a hang.
#include <algorithm>
#include <cstdlib>

#include "device_utils.cuh"
#include "kernels.h"

namespace heph {

constexpr int kScanThreads = 256;
constexpr int kScanWarps = kScanThreads / 32;
constexpr int kLookbackVectors = 8;          // look-back tile: 8 x 128-bit per thread (32 KiB)
constexpr int kLookbackVectorsSmall = 4;     // look-back tile for lines under 32 KiB (16 KiB)
constexpr uint64_t kInterleaveMinTiles = 2;  // look-back tiles per line from which lines interleave
constexpr int kChunkVectors = 4;             // chunked kernel tile: 4 x 128-bit per thread (16 KiB)
constexpr uint64_t kTwoPassMinTiles = 640;              // single lines of 640+ look-back tiles ...
constexpr uint64_t kTwoPassMaxBytes = 64ull << 20;      // ... and at most 64 MiB take the two-pass scan
constexpr uint64_t kMultiLineChunkedBytes = 8ull << 20;  // lines of several that take the chunked kernel
constexpr int kMaxCachedDevices = 64;        // device ordinals with cached launch queries
constexpr int kChunkMaxBuffers = 6;          // part buffers per CTA of the chunked scan
constexpr int kChunkMaxPartsPerThread = 2;   // chunked grids have at most 2 x 256 CTAs

// Scan status workspace, per entry (tile or part): a packed 64-bit word for
// 4-byte types, then two 8-byte value arrays and a 32-bit flag array for
// 8-byte types.  Section offsets are the entry capacity times 8, 16 and 24
// bytes, so every 8-byte array stays 8-byte aligned for any capacity.
constexpr size_t kStatusValsA = 8, kStatusValsB = 16, kStatusFlags = 24;
constexpr size_t kStatusBytesPerEntry = 28;

// Tuning knobs, read at each call (tests shrink the chunked kernel's parts).
static int scan_knob(const char *name, int fallback) {
    const char *e = getenv(name);
    return e ? atoi(e) : fallback;
}
static uint64_t scan_knob_u64(const char *name, uint64_t fallback) {
    const char *e = getenv(name);
    return e ? strtoull(e, nullptr, 10) : fallback;
}

template <typename T, int JV> struct ScanShape {
    static constexpr int V = 16 / sizeof(T);  // elements per 128-bit vector
    static constexpr int J = JV;              // vectors per thread
    static constexpr int WARP_ITEMS = 32 * V * J;
    static constexpr int TILE = kScanThreads * V * J;
};

enum : uint32_t { kStateInvalid = 0, kStateAggregate = 1, kStatePrefix = 2 };

// ------------------------------------------------------------ status words

struct StatusView {
    uint32_t epoch;
    unsigned long long *packed;  // 4-byte T: (value << 32) | (epoch << 2) | state
    uint32_t *flags;             // 8-byte T: (epoch << 2) | state
    void *vals_a, *vals_b;       // 8-byte T: aggregate / inclusive values
};

template <typename T>
__device__ __forceinline__ void publish(const StatusView &s, uint64_t idx, uint32_t state, T value) {
    const uint32_t f = (s.epoch << 2) | state;
    if constexpr (sizeof(T) == 4) {
        const unsigned long long w = ((unsigned long long)bitcast<uint32_t>(value) << 32) | f;
        asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(s.packed + idx), "l"(w) : "memory");
    } else {
        T *dst = static_cast<T *>(state == kStatePrefix ? s.vals_b : s.vals_a) + idx;
        asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(dst), "l"(bitcast<unsigned long long>(value))
                     : "memory");
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(s.flags + idx), "r"(f) : "memory");
    }
}

template <typename T>
__device__ __forceinline__ uint32_t read_status(const StatusView &s, uint64_t idx, T &value) {
    if constexpr (sizeof(T) == 4) {
        unsigned long long w;
        asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(s.packed + idx) : "memory");
        value = bitcast<T>((uint32_t)(w >> 32));
        const uint32_t f = (uint32_t)w;
        return ((f >> 2) == s.epoch) ? (f & 3u) : kStateInvalid;
    } else {
        uint32_t f;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(f) : "l"(s.flags + idx) : "memory");
        const uint32_t state = ((f >> 2) == s.epoch) ? (f & 3u) : kStateInvalid;
        if (state != kStateInvalid) {
            const T *src = static_cast<const T *>(state == kStatePrefix ? s.vals_b : s.vals_a) + idx;
            unsigned long long v;
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
            value = bitcast<T>(v);
        }
        return state;
    }
}

// ------------------------------------------------------------ tile scans

// Inclusive warp scan in logical lane order (descending lanes when `rev`).
template <typename T, int OP, bool REV> __device__ __forceinline__ T warp_scan(T v, int lane) {
    constexpr bool rev = REV;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const T o = rev ? shfl_down(v, d) : shfl_up(v, d);
        const bool ok = rev ? (lane + d < 32) : (lane >= d);
        if (ok) v = combine<T, OP>(o, v);
    }
    return v;
}

// Physical position in the tile of thread (warp, lane)'s element (j, c) is
// base + j*32*V + c with base = warp*WARP_ITEMS + lane*V: warp-striped
// 128-bit vectors, so every load and store instruction of a warp covers 512
// contiguous bytes.
template <typename T, int JV> __device__ __forceinline__ int tile_base_pos(int warp, int lane) {
    return warp * ScanShape<T, JV>::WARP_ITEMS + lane * ScanShape<T, JV>::V;
}

// Intra-tile part of a tile scan: in-vector inclusive scans (in place in x),
// warp scans of the vector totals and the fold of the warp totals, all in
// logical order (descending positions when `rev`).  Leaves the exclusive
// prefix of every vector (pre), of the thread's warp (wpre) and the tile
// aggregate (agg).  One __syncthreads; `s_warp` holds kScanWarps values.
template <typename T, int JV> struct TileScan {
    T pre[JV];
    T wpre, agg;
};

// The in-vector inclusive scans of a tile (in place), in logical order.
template <typename T, int OP, int JV, bool REV>
__device__ __forceinline__ void vector_local_scan(T (&x)[JV][ScanShape<T, JV>::V]) {
    constexpr int V = ScanShape<T, JV>::V;
#pragma unroll
    for (int j = 0; j < JV; ++j) {
        if (!REV) {
#pragma unroll
            for (int c = 1; c < V; ++c) x[j][c] = combine<T, OP>(x[j][c - 1], x[j][c]);
        } else {
#pragma unroll
            for (int c = V - 2; c >= 0; --c) x[j][c] = combine<T, OP>(x[j][c + 1], x[j][c]);
        }
    }
}

template <typename T, int OP, int JV, bool REV>
__device__ __forceinline__ void tile_local_scan(T (&x)[JV][ScanShape<T, JV>::V], T *s_warp, TileScan<T, JV> &r) {
    constexpr bool rev = REV;
    constexpr int V = ScanShape<T, JV>::V, J = JV;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
    T running = identity<T, OP>();
    const bool first_lane = rev ? (lane == 31) : (lane == 0);
#pragma unroll
    for (int jl = 0; jl < J; ++jl) {
        const int jp = rev ? J - 1 - jl : jl;
        const T inc = warp_scan<T, OP, REV>(tt[jp], lane);
        T exc = rev ? shfl_down(inc, 1) : shfl_up(inc, 1);
        if (first_lane) exc = identity<T, OP>();
        const T tot = shfl_idx(inc, rev ? 0 : 31);
        r.pre[jp] = combine<T, OP>(running, exc);
        running = combine<T, OP>(running, tot);
    }
    if (lane == 0) s_warp[warp] = running;
    __syncthreads();
    r.wpre = identity<T, OP>();
    r.agg = identity<T, OP>();
#pragma unroll
    for (int wl = 0; wl < kScanWarps; ++wl) {
        const int wp = rev ? kScanWarps - 1 - wl : wl;
        if (wp == warp) r.wpre = r.agg;
        r.agg = combine<T, OP>(r.agg, s_warp[wp]);
    }
}

// Final values of the tile given the exclusive prefix of the whole tile.
template <typename T, int OP, int JV, bool REV, bool EXCL>
__device__ __forceinline__ void tile_outputs(const T (&x)[JV][ScanShape<T, JV>::V], const TileScan<T, JV> &r,
                                             T tile_prefix, T (&y)[JV][ScanShape<T, JV>::V]) {
    constexpr bool rev = REV, exclusive = EXCL;
    constexpr int V = ScanShape<T, JV>::V;
    const T thread_base = combine<T, OP>(tile_prefix, r.wpre);
#pragma unroll
    for (int j = 0; j < JV; ++j) {
        const T tpj = combine<T, OP>(thread_base, r.pre[j]);
#pragma unroll
        for (int c = 0; c < V; ++c) {
            if (exclusive) {
                const bool first = rev ? (c == V - 1) : (c == 0);
                const T prev = rev ? x[j][(c + 1) % V] : x[j][(c + V - 1) % V];
                y[j][c] = first ? tpj : combine<T, OP>(tpj, prev);
            } else {
                y[j][c] = combine<T, OP>(tpj, x[j][c]);
            }
        }
    }
}

// Loads a full tile with 128-bit loads from global or shared memory.
template <typename T, int JV>
__device__ __forceinline__ void load_tile_vec(const T *src, int base, T (&x)[JV][ScanShape<T, JV>::V],
                                              bool streaming) {
    constexpr int V = ScanShape<T, JV>::V;
    uint4 raw[JV];
#pragma unroll
    for (int j = 0; j < JV; ++j) {
        const uint4 *p = reinterpret_cast<const uint4 *>(src + base + j * 32 * V);
        raw[j] = streaming ? ld_stream(p) : *p;
    }
#pragma unroll
    for (int j = 0; j < JV; ++j) {
        Vec16<T> e = as_elems<T>(raw[j]);
#pragma unroll
        for (int c = 0; c < V; ++c) x[j][c] = e.e[c];
    }
}

// A full tile from shared memory with explicit shared-space loads (a
// generic pointer would be loaded through the global path's scoreboard).
template <typename T, int JV>
__device__ __forceinline__ void load_tile_smem(const T *src, int base, T (&x)[JV][ScanShape<T, JV>::V]) {
    constexpr int V = ScanShape<T, JV>::V;
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(src + base);
    uint4 raw[JV];
#pragma unroll
    for (int j = 0; j < JV; ++j)
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(raw[j].x), "=r"(raw[j].y), "=r"(raw[j].z), "=r"(raw[j].w)
                     : "r"(a + (uint32_t)(j * 32 * V * sizeof(T))));
#pragma unroll
    for (int j = 0; j < JV; ++j) {
        Vec16<T> e = as_elems<T>(raw[j]);
#pragma unroll
        for (int c = 0; c < V; ++c) x[j][c] = e.e[c];
    }
}

// Guarded element loads of a partial (or unaligned) tile; identity padding.
template <typename T, int OP, int JV>
__device__ __forceinline__ void load_tile_scalar(const T *src, uint64_t valid, int base,
                                                 T (&x)[JV][ScanShape<T, JV>::V]) {
    constexpr int V = ScanShape<T, JV>::V;
#pragma unroll
    for (int j = 0; j < JV; ++j)
#pragma unroll
        for (int c = 0; c < V; ++c) {
            const uint64_t pos = (uint64_t)(base + j * 32 * V + c);
            x[j][c] = pos < valid ? src[pos] : identity<T, OP>();
        }
}

// A partial tile whose start is 16-byte aligned: whole vectors inside
// `valid` with 128-bit loads, the vector that straddles its end element by
// element, identity padding beyond it.
template <typename T, int OP, int JV>
__device__ __forceinline__ void load_tile_partial_vec(const T *src, uint64_t valid, int base,
                                                      T (&x)[JV][ScanShape<T, JV>::V]) {
    constexpr int V = ScanShape<T, JV>::V;
#pragma unroll
    for (int j = 0; j < JV; ++j) {
        const uint64_t pos = (uint64_t)(base + j * 32 * V);
        if (pos + V <= valid) {
            Vec16<T> e = as_elems<T>(ld_stream(reinterpret_cast<const uint4 *>(src + pos)));
#pragma unroll
            for (int c = 0; c < V; ++c) x[j][c] = e.e[c];
        } else {
#pragma unroll
            for (int c = 0; c < V; ++c) x[j][c] = pos + c < valid ? src[pos + c] : identity<T, OP>();
        }
    }
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));  // pure: hoisted and shared
    return pol;
}
__device__ __forceinline__ void st_policy(uint4 *p, uint4 v, uint64_t pol) {
    asm volatile("st.global.L1::no_allocate.L2::cache_hint.v4.u32 [%0], {%1,%2,%3,%4}, %5;" ::"l"(p), "r"(v.x),
                 "r"(v.y), "r"(v.z), "r"(v.w), "l"(pol)
                 : "memory");
}

// Stores a tile: 128-bit stores for a full tile (store_mode 0: streaming
// .cs hint, 1: L2 evict-first policy, 2: plain), element stores otherwise.
template <typename T, int JV>
__device__ __forceinline__ void store_tile(T *dst, uint64_t valid, bool full, int base,
                                           const T (&y)[JV][ScanShape<T, JV>::V], int store_mode = 0) {
    constexpr int V = ScanShape<T, JV>::V;
    if (full) {
#pragma unroll
        for (int j = 0; j < JV; ++j) {
            Vec16<T> e;
#pragma unroll
            for (int c = 0; c < V; ++c) e.e[c] = y[j][c];
            uint4 *q = reinterpret_cast<uint4 *>(dst + base + j * 32 * V);
            if (store_mode == 1) st_policy(q, as_uint4(e), l2_policy_evict_first());
            else if (store_mode == 2) *q = as_uint4(e);
            else st_stream(q, as_uint4(e));
        }
    } else {
#pragma unroll
        for (int j = 0; j < JV; ++j)
#pragma unroll
            for (int c = 0; c < V; ++c) {
                const uint64_t pos = (uint64_t)(base + j * 32 * V + c);
                if (pos < valid) dst[pos] = y[j][c];
            }
    }
}

// A partial tile whose start is 16-byte aligned: whole vectors inside
// `valid` with 128-bit streaming stores, the straddling one element-wise.
template <typename T, int JV>
__device__ __forceinline__ void store_tile_partial_vec(T *dst, uint64_t valid, int base,
                                                       const T (&y)[JV][ScanShape<T, JV>::V]) {
    constexpr int V = ScanShape<T, JV>::V;
#pragma unroll
    for (int j = 0; j < JV; ++j) {
        const uint64_t pos = (uint64_t)(base + j * 32 * V);
        if (pos + V <= valid) {
            Vec16<T> e;
#pragma unroll
            for (int c = 0; c < V; ++c) e.e[c] = y[j][c];
            st_stream(reinterpret_cast<uint4 *>(dst + pos), as_uint4(e));
        } else {
#pragma unroll
            for (int c = 0; c < V; ++c)
                if (pos + c < valid) dst[pos + c] = y[j][c];
        }
    }
}

// --------------------------------------------------- decoupled look-back

template <typename T> struct LookbackParams {
    const T *in;
    T *out;
    uint64_t len;               // elements per line
    uint64_t tiles_per_line;
    uint64_t lines;
    // Tile numbering: line-major (id = line * tiles_per_line + position) or,
    // when `interleaved`, position-major (id = position * lines + line).
    // Either way a tile's predecessors in its line have lower ids.
    uint64_t pos_step;          // id distance between neighbouring positions: 1, or lines
    int interleaved;
    int64_t in_line, out_line;  // element distance between line starts
    StatusView status;
    const T *carry;             // nullable seed of line 0
    unsigned int *err;
    int reverse, exclusive;
};

// Exclusive prefix of `tile` (at position `pos` of its line) within its
// line: fold of the predecessors back to the nearest one that has published
// its inclusive prefix, 32 predecessors per round trip.  The predecessor at
// distance j is tile - j * pos_step.  Runs on one warp.
template <typename T, int OP>
__device__ T lookback(const LookbackParams<T> &p, uint64_t tile, uint64_t pos, int lane) {
    T excl = identity<T, OP>();
    int64_t back = 1;  // distance of this round's first predecessor
    WaitDeadline deadline;  // every lane keeps the same count; lane 0 decides
    while (true) {
        const int64_t d = back + lane;
        const bool in_range = d <= (int64_t)pos;
        uint32_t state = kStatePrefix;  // positions before the line start act as an identity prefix
        T val = identity<T, OP>();
        const uint64_t idx = tile - (uint64_t)d * p.pos_step;
        if (in_range) state = read_status(p.status, idx, val);
        while (__any_sync(kFullMask, state == kStateInvalid)) {
            if (__shfl_sync(kFullMask, (int)deadline.expired(), 0)) {
                if (lane == 0) raise_device_error(p.err, DEVERR_LOOKBACK_TIMEOUT);
                return excl;
            }
            __nanosleep(32);
            if (state == kStateInvalid) state = read_status(p.status, idx, val);
        }
        const unsigned pm = __ballot_sync(kFullMask, state == kStatePrefix);
        const int stop = pm ? __ffs(pm) - 1 : 31;
        T v = lane <= stop ? val : identity<T, OP>();
        v = warp_fold<T, OP>(v);
        excl = combine<T, OP>(v, excl);
        if (pm) return excl;
        back += 32;
    }
}

// One tile per CTA.  Lines of several tiles are numbered position-major (the
// first tile of every line, then the second, ...) so the resident CTAs
// advance all lines' prefix chains at once instead of waiting along one
// line's chain.
template <typename T, int OP, bool VEC, int JV, bool REV, bool EXCL>
__global__ void __launch_bounds__(kScanThreads) scan_lookback_kernel(const LookbackParams<T> p) {
    using S = ScanShape<T, JV>;
    constexpr int V = S::V, TILE = S::TILE;
    __shared__ T s_warp[kScanWarps];
    __shared__ T s_prefix;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr bool rev = REV;
    const uint64_t tile = blockIdx.x;
    uint64_t line, t_in_line;
    if (p.interleaved) {
        t_in_line = tile / p.lines;
        line = tile - t_in_line * p.lines;
    } else {
        line = tile / p.tiles_per_line;
        t_in_line = tile - line * p.tiles_per_line;
    }
    const uint64_t ptile = rev ? p.tiles_per_line - 1 - t_in_line : t_in_line;
    const T *lin = p.in + (int64_t)line * p.in_line;
    T *lout = p.out + (int64_t)line * p.out_line;
    const uint64_t start = ptile * (uint64_t)TILE;
    const uint64_t valid = min((uint64_t)TILE, p.len - start);
    const bool full = VEC && valid == (uint64_t)TILE;
    const int base = tile_base_pos<T, JV>(warp, lane);

    T x[JV][V];
    if (full) load_tile_vec<T, JV>(lin + start, base, x, true);
    else if (VEC) load_tile_partial_vec<T, OP, JV>(lin + start, valid, base, x);
    else load_tile_scalar<T, OP, JV>(lin + start, valid, base, x);
    TileScan<T, JV> r;
    tile_local_scan<T, OP, JV, REV>(x, s_warp, r);

    if (warp == 0) {
        T tp;
        if (t_in_line == 0) {
            tp = (p.carry != nullptr && line == 0) ? *p.carry : identity<T, OP>();
            if (lane == 0) publish(p.status, tile, kStatePrefix, combine<T, OP>(tp, r.agg));
        } else {
            if (lane == 0) publish(p.status, tile, kStateAggregate, r.agg);
            tp = lookback<T, OP>(p, tile, t_in_line, lane);
            if (lane == 0) publish(p.status, tile, kStatePrefix, combine<T, OP>(tp, r.agg));
        }
        if (lane == 0) s_prefix = tp;
    }
    __syncthreads();
    T y[JV][V];
    tile_outputs<T, OP, JV, REV, EXCL>(x, r, s_prefix, y);
    if (VEC && !full) store_tile_partial_vec<T, JV>(lout + start, valid, base, y);
    else store_tile<T, JV>(lout + start, valid, full, base, y);
}

// ------------------------------------------ two-pass scan of a mid-size line
//
// A single line too short for the chunked kernel but long enough that a
// look-back chain would dominate (its inclusive-prefix front advances 32
// tiles per status round trip): pass 1 writes every tile's total, pass 2
// folds, per tile, the totals before it (in scan order) and scans the tile
// with that prefix.  The line is at most a few tens of MB, so pass 2 reads
// it back from L2.

// Tile `blockIdx.x` of the line into x (identity past the end).
template <typename T, int OP, bool VEC, int JV>
__device__ __forceinline__ void load_line_tile(const T *in, uint64_t len, int base, T (&x)[JV][ScanShape<T, JV>::V],
                                               uint64_t &start, uint64_t &valid) {
    constexpr int TILE = ScanShape<T, JV>::TILE;
    start = (uint64_t)blockIdx.x * TILE;
    valid = min((uint64_t)TILE, len - start);
    if (VEC && valid == (uint64_t)TILE) load_tile_vec<T, JV>(in + start, base, x, false);
    else if (VEC) load_tile_partial_vec<T, OP, JV>(in + start, valid, base, x);
    else load_tile_scalar<T, OP, JV>(in + start, valid, base, x);
}

template <typename T, int OP, bool VEC, int JV>
__global__ void __launch_bounds__(kScanThreads) scan_tile_totals_kernel(const T *__restrict__ in, uint64_t len,
                                                                       T *__restrict__ totals) {
    constexpr int V = ScanShape<T, JV>::V;
    __shared__ T scratch[kScanWarps];
    const int base = tile_base_pos<T, JV>(threadIdx.x >> 5, threadIdx.x & 31);
    T x[JV][V];
    uint64_t start, valid;
    load_line_tile<T, OP, VEC, JV>(in, len, base, x, start, valid);
    T acc = identity<T, OP>();
#pragma unroll
    for (int j = 0; j < JV; ++j)
#pragma unroll
        for (int c = 0; c < V; ++c) acc = combine<T, OP>(acc, x[j][c]);
    acc = block_fold<T, OP, kScanThreads>(acc, scratch);
    if (threadIdx.x == 0) totals[blockIdx.x] = acc;
}

template <typename T, int OP, bool VEC, int JV, bool REV, bool EXCL>
__global__ void __launch_bounds__(kScanThreads) scan_tile_apply_kernel(const T *__restrict__ in, T *__restrict__ out,
                                                                      uint64_t len, uint64_t ntiles,
                                                                      const T *__restrict__ totals,
                                                                      const T *__restrict__ carry) {
    constexpr int V = ScanShape<T, JV>::V;
    __shared__ T s_warp[kScanWarps];
    __shared__ T scratch[kScanWarps];
    const int base = tile_base_pos<T, JV>(threadIdx.x >> 5, threadIdx.x & 31);
    T x[JV][V];
    uint64_t start, valid;
    load_line_tile<T, OP, VEC, JV>(in, len, base, x, start, valid);  // in flight during the fold below
    // The fold of the totals before this tile in scan order (after it, for a
    // reverse scan), seeded with the carry.
    const uint64_t k = blockIdx.x;
    const uint64_t lo = REV ? k + 1 : 0, hi = REV ? ntiles : k;
    T pre = identity<T, OP>();
    for (uint64_t i = lo + threadIdx.x; i < hi; i += kScanThreads) pre = combine<T, OP>(pre, totals[i]);
    pre = block_fold<T, OP, kScanThreads>(pre, scratch);
    if (carry) pre = combine<T, OP>(*carry, pre);
    TileScan<T, JV> r;
    tile_local_scan<T, OP, JV, REV>(x, s_warp, r);
    T y[JV][V];
    tile_outputs<T, OP, JV, REV, EXCL>(x, r, pre, y);
    if (valid == (uint64_t)ScanShape<T, JV>::TILE && VEC) store_tile<T, JV>(out + start, valid, true, base, y);
    else if (VEC) store_tile_partial_vec<T, JV>(out + start, valid, base, y);
    else store_tile<T, JV>(out + start, valid, false, base, y);
}

// --------------------------------- chunked reduce-then-scan, parts in smem

// The lines of a chunked scan are cut into parts of `part` elements (the last
// part of a line is ragged when the part does not divide the line).  Part j
// of line l in scan order has the virtual index v = l * ppl + j; chunk c is
// the G parts v = c*G .. c*G+G-1, CTA b taking v = c*G + b.  A reverse scan
// takes the line's parts from its end (physical part ppl-1-j).  One long line
// is the case lines == 1.
template <typename T> struct ChunkParams {
    const T *in;
    T *out;
    uint64_t len;      // elements per line
    uint64_t lines;
    int64_t in_line, out_line;  // element distance between line starts
    uint64_t ppl;      // parts per line
    uint64_t parts;    // ppl * lines
    uint64_t part;     // elements per part (a multiple of the tile)
    uint64_t nchunks;
    StatusView status;
    const T *carry;    // nullable seed of line 0
    unsigned int *err;
    int reverse, exclusive;
    int buffers;       // shared-memory part buffers per CTA (2..kChunkMaxBuffers)
    int store_mode;    // see store_tile
};

// CTA b's part of logical chunk c: element range [lo, hi) within its line
// (empty past the last line), the line's element offsets, and for the
// exchange of the chunk's part totals: the index (relative to the chunk's
// first part) of the first part of this CTA's line (`my_first`) and of the
// chunk's last line (`last_first`), negative when that line began in an
// earlier chunk (line 0 counts as begun earlier: the kernel's running carry
// is its seed).  Thread 0 computes it when it stages the part and keeps it in
// shared memory beside the part's buffer, so the other threads never divide.
struct ChunkSlot {
    uint64_t lo, hi;
    int64_t in_off, out_off;
    int32_t my_first, last_first;
};

__device__ __forceinline__ int32_t clamp_first(int64_t f, int G) {
    return (int32_t)max((int64_t)-1, min(f, (int64_t)G));
}

// Thread 0's position of the next chunk to stage: line and part-in-line of
// this CTA's part (v = c*G + b) and of the chunk's last part (c*G + G - 1).
// Chunks are staged in increasing order, so the cursor advances by G parts
// with a subtraction or two instead of a 64-bit division per chunk (thread 0
// stages in the middle of the output step, where extra latency delays the
// whole CTA at its next barrier).
struct PartCursor {
    uint64_t line, j, last_line, last_j;
};

template <typename T> __device__ __forceinline__ PartCursor part_cursor_start(const ChunkParams<T> &p, int b) {
    PartCursor q;
    q.line = (uint64_t)b / p.ppl;
    q.j = (uint64_t)b - q.line * p.ppl;
    q.last_line = (uint64_t)(gridDim.x - 1) / p.ppl;
    q.last_j = (uint64_t)(gridDim.x - 1) - q.last_line * p.ppl;
    return q;
}

template <typename T> __device__ __forceinline__ void part_cursor_advance(const ChunkParams<T> &p, PartCursor &q) {
    q.j += gridDim.x;
    while (q.j >= p.ppl) {
        q.j -= p.ppl;
        ++q.line;
    }
    q.last_j += gridDim.x;
    while (q.last_j >= p.ppl) {
        q.last_j -= p.ppl;
        ++q.last_line;
    }
}

template <typename T>
__device__ __forceinline__ ChunkSlot chunk_slot(const ChunkParams<T> &p, uint64_t c, const PartCursor &q) {
    ChunkSlot r{0, 0, 0, 0, (int32_t)gridDim.x, (int32_t)gridDim.x};
    const uint64_t c0 = c * gridDim.x;
    const uint64_t last_line = min(q.last_line, p.lines - 1);
    r.last_first = last_line == 0 ? -1 : clamp_first((int64_t)(last_line * p.ppl) - (int64_t)c0, gridDim.x);
    if (q.line >= p.lines) return r;  // past the last line's last part
    const uint64_t jp = p.reverse ? p.ppl - 1 - q.j : q.j;
    r.lo = jp * p.part;
    r.hi = min(p.len, r.lo + p.part);
    r.in_off = (int64_t)q.line * p.in_line;
    r.out_off = (int64_t)q.line * p.out_line;
    r.my_first = q.line == 0 ? -1 : clamp_first((int64_t)(q.line * p.ppl) - (int64_t)c0, gridDim.x);
    return r;
}

// Thread 0: record CTA b's part of logical chunk c (the cursor's chunk) in
// its slot, start the bulk copy of the part into its buffer (full parts only;
// a ragged part, the last of a line, is read from global memory), and move the
// cursor to chunk c + 1.
template <typename T>
__device__ __forceinline__ void chunk_stage_in(const ChunkParams<T> &p, uint32_t c, T *buf, uint64_t *bar,
                                               ChunkSlot *slots, PartCursor &q) {
    const ChunkSlot r = chunk_slot(p, c, q);
    part_cursor_advance(p, q);
    const uint32_t k = c % (uint32_t)p.buffers;
    slots[k] = r;
    if (r.hi - r.lo == p.part)
        bulk_load(buf + k * p.part, p.in + r.in_off + r.lo, (uint32_t)(p.part * sizeof(T)), &bar[k]);
}


// Step 1 of a chunk for CTA b's part of logical chunk c: everything of the
// part's tile scans that does not depend on the incoming prefix - in-vector
// scans, warp scans of the vector totals, fold of the warp totals - kept in
// `rs` for step 3 one iteration later, and the part total (the fold of the
// tile aggregates) published.  A ragged part (the line's last, read from
// global memory) only publishes its total; step 3 scans it from scratch.
template <typename T, int OP, int JV, bool REV, int TPP>
__device__ __forceinline__ void chunk_prescan_part(const ChunkParams<T> &p, int b, uint64_t c, const T *buf,
                                                   uint64_t *bar, uint32_t &phases, T (*s_warp)[kScanWarps],
                                                   int &parity, T *s_red, TileScan<T, JV> (&rs)[TPP],
                                                   const ChunkSlot *slots) {
    constexpr int TILE = ScanShape<T, JV>::TILE;
    const ChunkSlot pr = slots[(uint32_t)c % (uint32_t)p.buffers];
    const uint64_t n = pr.hi - pr.lo;
    if (n == p.part) {
        const int k = (int)((uint32_t)c % (uint32_t)p.buffers);
        mbar_wait(&bar[k], (phases >> k) & 1u, p.err);
        phases ^= 1u << k;
        const int base = tile_base_pos<T, JV>(threadIdx.x >> 5, threadIdx.x & 31);
        T agg = identity<T, OP>();
#pragma unroll
        for (int tl = 0; tl < TPP; ++tl) {
            const int tp = REV ? TPP - 1 - tl : tl;
            T x[JV][ScanShape<T, JV>::V];
            load_tile_smem<T, JV>(buf + k * p.part + tp * TILE, base, x);
            tile_local_scan<T, OP, JV, REV>(x, s_warp[parity], rs[tp]);
            parity ^= 1;
            agg = combine<T, OP>(agg, rs[tp].agg);
        }
        if (threadIdx.x == 0) publish(p.status, c * gridDim.x + b, kStatePrefix, agg);
        return;
    }
    constexpr int V = Vec16<T>::V;
    (void)V;
    T acc = identity<T, OP>();
    const T *lin = p.in + pr.in_off;
    for (uint64_t e = pr.lo + threadIdx.x; e < pr.hi; e += kScanThreads) acc = combine<T, OP>(acc, lin[e]);
    // One barrier, no trailing one: s_red is rewritten only by the next
    // ragged part, which cannot come before the next barriers.
    acc = warp_fold<T, OP>(acc);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        T r = s_red[0];
#pragma unroll
        for (int w = 1; w < kScanWarps; ++w) r = combine<T, OP>(r, s_red[w]);
        publish(p.status, c * gridDim.x + b, kStatePrefix, r);
    }
}

// L: parts prescanned ahead (their totals are published L iterations before
// the exchange that reads them - the slack a late CTA can use); TPP: tiles
// per staged part.  Needs p.buffers >= L + 2.
template <typename T, int OP, int JV, bool REV, bool EXCL, int L, int TPP>
__global__ void __launch_bounds__(kScanThreads, 3) scan_chunked_kernel(const ChunkParams<T> p) {
    using S = ScanShape<T, JV>;
    constexpr int V = S::V, TILE = S::TILE;
    extern __shared__ __align__(128) unsigned char dyn_smem[];
    T *buf = reinterpret_cast<T *>(dyn_smem);  // buffers x part elements
    __shared__ uint64_t bar[kChunkMaxBuffers];
    __shared__ T s_warp[2][kScanWarps];
    __shared__ T s_red[kScanWarps];
    __shared__ T s_pair[2][kScanWarps];
    __shared__ ChunkSlot s_slot[kChunkMaxBuffers];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int G = gridDim.x, b = blockIdx.x;
    const int NB = p.buffers;
    constexpr bool rev = REV;
    const int base = tile_base_pos<T, JV>(warp, lane);
    uint32_t phases = 0;
    int parity = 0;
    PartCursor cursor{};  // thread 0's: the next chunk to stage
    if (threadIdx.x == 0) cursor = part_cursor_start(p, b);

    if (threadIdx.x == 0) {
        for (int k = 0; k < NB; ++k) mbar_init(&bar[k], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int k = 0; k < NB && (uint64_t)k < p.nchunks; ++k) chunk_stage_in(p, (uint32_t)k, buf, bar, s_slot, cursor);
    }
    __syncthreads();

    T carry = p.carry ? *p.carry : identity<T, OP>();
    // Prefix-independent tile-scan results of the parts of chunks c .. c+L:
    // ring[0] is output in this iteration, ring[L] is prescanned in it.  The
    // ring shifts with constant indices (registers, no local memory).
    TileScan<T, JV> ring[L + 1][TPP];
#pragma unroll
    for (int k = 0; k < L; ++k)
        if ((uint64_t)k < p.nchunks)
            chunk_prescan_part<T, OP, JV, REV, TPP>(p, b, k, buf, bar, phases, s_warp, parity, s_red, ring[k], s_slot);
    for (uint64_t c = 0; c < p.nchunks; ++c) {
        // The part totals of chunk c were published one iteration ago: for
        // 4-byte T their status words are loaded here, before step 1, so the
        // L2 round trip overlaps it.
        unsigned long long early[kChunkMaxPartsPerThread];
        if constexpr (sizeof(T) == 4) {
#pragma unroll
            for (int i = 0; i < kChunkMaxPartsPerThread; ++i) {
                const int q = threadIdx.x + i * kScanThreads;
                early[i] = 0;
                if (q < G)
                    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];"
                                 : "=l"(early[i])
                                 : "l"(p.status.packed + c * G + q)
                                 : "memory");
            }
        }
        // Step 1: prescan of the part L chunks ahead, its total published.
        if (c + L < p.nchunks)
            chunk_prescan_part<T, OP, JV, REV, TPP>(p, b, c + L, buf, bar, phases, s_warp, parity, s_red, ring[L], s_slot);

        // Step 2: the part totals of chunk c.  `before` folds the parts of
        // this CTA's line before its own in the chunk; `tail` folds the parts
        // of the chunk's last line (the carry into the next chunk).
        const ChunkSlot pr = s_slot[(uint32_t)c % (uint32_t)NB];  // read before thread 0 can restage the slot
        const int32_t my_first = pr.my_first, last_first = pr.last_first;
        T before = identity<T, OP>(), tail = identity<T, OP>();
#pragma unroll
        for (int i = 0; i < kChunkMaxPartsPerThread; ++i) {
            const int q = threadIdx.x + i * kScanThreads;
            if (q >= G) break;
            T v = identity<T, OP>();
            bool ok;
            if constexpr (sizeof(T) == 4) {
                const uint32_t f = (uint32_t)early[i];
                v = bitcast<T>((uint32_t)(early[i] >> 32));
                ok = (f >> 2) == p.status.epoch && (f & 3u) != kStateInvalid;
            } else {
                ok = read_status(p.status, c * G + q, v) != kStateInvalid;
            }
            WaitDeadline deadline;
            while (!ok) {
                if (deadline.expired()) {
                    raise_device_error(p.err, DEVERR_LOOKBACK_TIMEOUT);
                    v = identity<T, OP>();
                    break;
                }
                __nanosleep(32);
                ok = read_status(p.status, c * G + q, v) != kStateInvalid;
            }
            if (q >= last_first) tail = combine<T, OP>(tail, v);
            if (q < b && q >= my_first) before = combine<T, OP>(before, v);
        }
        // Both folds share one barrier; s_pair is rewritten only in the next
        // iteration, after step 1's barriers.
        before = warp_fold<T, OP>(before);
        tail = warp_fold<T, OP>(tail);
        if (lane == 0) {
            s_pair[0][warp] = before;
            s_pair[1][warp] = tail;
        }
        __syncthreads();
        before = s_pair[0][0];
        tail = s_pair[1][0];
#pragma unroll
        for (int w = 1; w < kScanWarps; ++w) {
            before = combine<T, OP>(before, s_pair[0][w]);
            tail = combine<T, OP>(tail, s_pair[1][w]);
        }
        T run = my_first < 0 ? combine<T, OP>(carry, before) : before;
        carry = last_first < 0 ? combine<T, OP>(carry, tail) : tail;

        // Step 3: the part's outputs, tile by tile in logical order.
        const uint64_t lo = pr.lo, hi = pr.hi;
        const T *lin = p.in + pr.in_off;
        T *lout = p.out + pr.out_off;
        if (hi - lo == p.part) {
            // Staged and prescanned: reload, redo the in-vector scans, add
            // the prefixes.  No barrier.
            const T *src = buf + ((uint32_t)c % (uint32_t)NB) * p.part;
#pragma unroll
            for (int tl = 0; tl < TPP; ++tl) {
                const int tp = rev ? TPP - 1 - tl : tl;
                T x[JV][V];
                load_tile_smem<T, JV>(src + tp * TILE, base, x);
                if (tl + 1 == TPP) {
                    // Every thread has read the part: refill its buffer with
                    // chunk c+NB while the outputs are finished and stored.
                    __syncthreads();
                    if (threadIdx.x == 0 && c + NB < p.nchunks) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        chunk_stage_in(p, (uint32_t)(c + NB), buf, bar, s_slot, cursor);
                    }
                }
                vector_local_scan<T, OP, JV, REV>(x);
                T y[JV][V];
                tile_outputs<T, OP, JV, REV, EXCL>(x, ring[0][tp], run, y);
                run = combine<T, OP>(run, ring[0][tp].agg);
                store_tile<T, JV>(lout + lo + (uint64_t)tp * TILE, TILE, true, base, y, p.store_mode);
            }
        } else {
            const uint64_t ntiles = (hi - lo + TILE - 1) / TILE;
            for (uint64_t tl = 0; tl < ntiles; ++tl) {
                const uint64_t tp = rev ? ntiles - 1 - tl : tl;
                const uint64_t start = tp * TILE;  // relative to lo
                const uint64_t valid = min((uint64_t)TILE, hi - lo - start);
                const bool full = valid == (uint64_t)TILE;
                T x[JV][V];
                if (full) load_tile_vec<T, JV>(lin + lo + start, base, x, false);
                else load_tile_scalar<T, OP, JV>(lin + lo + start, valid, base, x);
                TileScan<T, JV> r;
                tile_local_scan<T, OP, JV, REV>(x, s_warp[parity], r);
                parity ^= 1;
                T y[JV][V];
                tile_outputs<T, OP, JV, REV, EXCL>(x, r, run, y);
                run = combine<T, OP>(run, r.agg);
                store_tile<T, JV>(lout + lo + start, valid, full, base, y, p.store_mode);
            }
            // A ragged or empty part never used its buffer.
            if (threadIdx.x == 0 && c + NB < p.nchunks) chunk_stage_in(p, (uint32_t)(c + NB), buf, bar, s_slot, cursor);
        }
#pragma unroll
        for (int k = 0; k < L; ++k)
#pragma unroll
            for (int t = 0; t < TPP; ++t) ring[k][t] = ring[k + 1][t];
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
        const T inc = warp_scan<T, OP, false>(x, lane);
        T exc = shfl_up(inc, 1);
        if (lane == 0) exc = identity<T, OP>();
        if (ok) p.out[ob + (int64_t)idx * p.out_r] = combine<T, OP>(running, p.exclusive ? exc : inc);
        running = combine<T, OP>(running, shfl_idx(inc, 31));
    }
}

// ------------------------------------------------------------------ launch

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Status view over the workspace for `entries` entries; bumps the epoch
// (clearing the status before the 30-bit tag wraps).  Caller holds dev->mu.
static heph_status status_for(Device *dev, cudaStream_t stream, uint64_t entries, StatusView *sv) {
    Workspace *ws = nullptr;
    heph_status st = workspace_for(dev, stream, 0, (size_t)entries * kStatusBytesPerEntry, &ws);
    if (st != HEPH_OK) return st;
    if (ws->epoch >= (1u << 30) - 1) {
        HEPH_CUDA_TRY(cudaMemsetAsync(ws->scan_status, 0, ws->scan_status_bytes, stream), HEPH_DISPATCH_FAILED,
                      "scan status reset");
        ws->epoch = 0;
    }
    ws->epoch += 1;
    char *base = static_cast<char *>(ws->scan_status);
    const size_t cap = ws->scan_status_bytes / kStatusBytesPerEntry;
    sv->epoch = ws->epoch;
    sv->packed = reinterpret_cast<unsigned long long *>(base);
    sv->vals_a = base + cap * kStatusValsA;
    sv->vals_b = base + cap * kStatusValsB;
    sv->flags = reinterpret_cast<uint32_t *>(base + cap * kStatusFlags);
    return HEPH_OK;
}

// The chunked kernel for `lines` aligned lines of `len` elements (line starts
// in_line / out_line elements apart).  Returns false (nothing launched) when
// the lines are too short to give every CTA four parts.
template <typename T, int OP, bool REV, bool EXCL, int L, int TPP>
static bool launch_chunked(Device *dev, cudaStream_t stream, const T *in, T *out, uint64_t len, uint64_t lines,
                           int64_t in_line, int64_t out_line, bool reverse, bool exclusive, const T *carry,
                           heph_status *st, int default_ctas) {
    using S = ScanShape<T, kChunkVectors>;
    const int nb = std::min(kChunkMaxBuffers, std::max(L + 2, scan_knob("HEPH_SCAN_BUFS", L + 2)));
    const uint64_t part = (uint64_t)TPP * S::TILE;
    const size_t smem = (size_t)nb * part * sizeof(T);
    if (smem > (200u << 10)) return false;
    auto kernel = scan_chunked_kernel<T, OP, kChunkVectors, REV, EXCL, L, TPP>;
    // The attribute and occupancy queries cost host time on every call (the
    // GPU idles behind them when lines are launched back to back): they run
    // once per (device, kernel, shared-memory size).  The caller holds the
    // device's lock, and each device has its own slot.
    struct Occupancy {
        size_t smem;
        int nb_sm;
    };
    static Occupancy occ[kMaxCachedDevices];
    int nb_sm = 0;
    Occupancy *oc = dev->ordinal >= 0 && dev->ordinal < kMaxCachedDevices ? &occ[dev->ordinal] : nullptr;
    if (oc && oc->nb_sm > 0 && oc->smem == smem) {
        nb_sm = oc->nb_sm;
    } else {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb_sm, kernel, kScanThreads, smem) != cudaSuccess ||
            nb_sm < 1) {
            cudaGetLastError();
            return false;
        }
        if (oc) *oc = Occupancy{smem, nb_sm};
    }
    const int per_sm = std::min(nb_sm, std::max(1, scan_knob("HEPH_SCAN_CHUNK_CTAS", default_ctas)));
    const uint64_t G =
        std::min<uint64_t>((uint64_t)dev->sm_count * per_sm, (uint64_t)kChunkMaxPartsPerThread * kScanThreads);
    const uint64_t ppl = (len + part - 1) / part;
    if (lines == 0 || ppl * lines < 4 * G) return false;
    ChunkParams<T> cp{};
    cp.in = in;
    cp.out = out;
    cp.len = len;
    cp.lines = lines;
    cp.in_line = in_line;
    cp.out_line = out_line;
    cp.ppl = ppl;
    cp.parts = ppl * lines;
    cp.part = part;
    cp.nchunks = (ppl * lines + G - 1) / G;
    cp.carry = carry;
    cp.err = dev->error_dev;
    cp.reverse = reverse;
    cp.exclusive = exclusive;
    cp.buffers = nb;
    cp.store_mode = scan_knob("HEPH_SCAN_STORE", 1);
    *st = status_for(dev, stream, cp.nchunks * G, &cp.status);
    if (*st != HEPH_OK) return true;
    void *args[] = {&cp};
    // Cooperative launch: every CTA is co-resident, so CTAs may wait on each
    // other's part totals.
    cudaError_t e = cudaLaunchCooperativeKernel((const void *)kernel, dim3((unsigned)G), dim3(kScanThreads), args,
                                                smem, stream);
    *st = e == cudaSuccess ? HEPH_OK : cuda_fail(HEPH_DISPATCH_FAILED, e, "chunked scan launch");
    return true;
}

// Shape of the chunked scan: parts are one 16 KiB tile, prescanned two
// chunks ahead, four part buffers (64 KiB) per CTA, three CTAs per SM.  Of
// the shapes measured - lookahead 1-3, 1-2 tiles per part, 1-4 CTAs per SM -
// this one streams fastest: the two-chunk slack absorbs late CTAs at the
// part-total exchange, and 24 warps per SM hide the tile-scan latency.
constexpr int kChunkLookahead = 2;
constexpr int kChunkTilesPerPart = 1;
constexpr int kChunkCtasPerSm = 3;

template <typename T, int OP, bool REV, bool EXCL>
static bool launch_chunked_any(Device *dev, cudaStream_t stream, const T *in, T *out, uint64_t len, uint64_t lines,
                               int64_t in_line, int64_t out_line, bool reverse, bool exclusive, const T *carry,
                               heph_status *st) {
    return launch_chunked<T, OP, REV, EXCL, kChunkLookahead, kChunkTilesPerPart>(
        dev, stream, in, out, len, lines, in_line, out_line, reverse, exclusive, carry, st, kChunkCtasPerSm);
}

template <typename T, int OP, int JV>
static void launch_lookback(int sel, dim3 grid, cudaStream_t stream, const LookbackParams<T> &p) {
    switch (sel) {
        case 0: scan_lookback_kernel<T, OP, false, JV, false, false><<<grid, kScanThreads, 0, stream>>>(p); break;
        case 1: scan_lookback_kernel<T, OP, false, JV, false, true><<<grid, kScanThreads, 0, stream>>>(p); break;
        case 2: scan_lookback_kernel<T, OP, false, JV, true, false><<<grid, kScanThreads, 0, stream>>>(p); break;
        case 3: scan_lookback_kernel<T, OP, false, JV, true, true><<<grid, kScanThreads, 0, stream>>>(p); break;
        case 4: scan_lookback_kernel<T, OP, true, JV, false, false><<<grid, kScanThreads, 0, stream>>>(p); break;
        case 5: scan_lookback_kernel<T, OP, true, JV, false, true><<<grid, kScanThreads, 0, stream>>>(p); break;
        case 6: scan_lookback_kernel<T, OP, true, JV, true, false><<<grid, kScanThreads, 0, stream>>>(p); break;
        default: scan_lookback_kernel<T, OP, true, JV, true, true><<<grid, kScanThreads, 0, stream>>>(p); break;
    }
}

// Both passes of the two-pass scan on `stream`; the tile totals live in the
// stream's workspace.  The caller holds the device's lock.
template <typename T, int OP>
static heph_status launch_two_pass(Device *dev, cudaStream_t stream, const T *in, T *out, uint64_t len,
                                   uint64_t ntiles, bool vec, bool reverse, bool exclusive, const T *carry) {
    Workspace *ws = nullptr;
    heph_status st = workspace_for(dev, stream, (size_t)ntiles * sizeof(T), 0, &ws);
    if (st != HEPH_OK) return st;
    T *totals = static_cast<T *>(ws->partials);
    constexpr int JV = kLookbackVectors;
    const dim3 grid((unsigned)ntiles);
    if (vec) scan_tile_totals_kernel<T, OP, true, JV><<<grid, kScanThreads, 0, stream>>>(in, len, totals);
    else scan_tile_totals_kernel<T, OP, false, JV><<<grid, kScanThreads, 0, stream>>>(in, len, totals);
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "scan tile totals launch");
    const int sel = (vec ? 4 : 0) | (reverse ? 2 : 0) | (exclusive ? 1 : 0);
    switch (sel) {
#define HEPH_APPLY(V_, R_, E_) \
    scan_tile_apply_kernel<T, OP, V_, JV, R_, E_><<<grid, kScanThreads, 0, stream>>>(in, out, len, ntiles, totals, carry)
        case 0: HEPH_APPLY(false, false, false); break;
        case 1: HEPH_APPLY(false, false, true); break;
        case 2: HEPH_APPLY(false, true, false); break;
        case 3: HEPH_APPLY(false, true, true); break;
        case 4: HEPH_APPLY(true, false, false); break;
        case 5: HEPH_APPLY(true, false, true); break;
        case 6: HEPH_APPLY(true, true, false); break;
        default: HEPH_APPLY(true, true, true); break;
#undef HEPH_APPLY
    }
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "scan apply launch");
    return HEPH_OK;
}

template <typename T, int OP>
static heph_status launch_scan_typed(Device *dev, cudaStream_t stream, const T *in, T *out, const AxisProblem &pr,
                                     bool reverse, bool exclusive, const T *carry) {
    using S = ScanShape<T, kLookbackVectors>;
    const bool contiguous = pr.in_r == 1 && pr.out_r == 1;
    if (!contiguous || pr.len < (uint64_t)S::TILE / 4) {
        StridedScanParams<T> sp{in, out, pr.outer, pr.len, pr.in_base, pr.in_o, pr.in_r,
                                pr.out_base, pr.out_o, pr.out_r, carry, reverse, exclusive};
        const uint64_t blocks = (pr.outer * 32 + 255) / 256;
        if (blocks > 0x7fffffffull) return fail(HEPH_DISPATCH_FAILED, "scan grid too large");
        scan_strided_kernel<T, OP><<<(unsigned)blocks, 256, 0, stream>>>(sp);
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "scan launch");
        return HEPH_OK;
    }
    const bool vec = aligned16(in + pr.in_base) && aligned16(out + pr.out_base) &&
                     (pr.outer == 1 || (((uint64_t)pr.in_o * sizeof(T)) % 16 == 0 &&
                                        ((uint64_t)pr.out_o * sizeof(T)) % 16 == 0));
    std::lock_guard<std::mutex> lock(dev->mu);
    // One line long enough for the chunked kernel takes it; several lines
    // take it too (one launch for all of them, each line's parts with their
    // own running prefix) once every line spans kMultiLineChunkedBytes:
    // along lines that long the look-back chains, not HBM, bound the
    // look-back kernel.
    const bool chunked_shape = pr.outer == 1 || pr.len * sizeof(T) >= (uint64_t)scan_knob_u64(
                                                      "HEPH_SCAN_MULTI_CHUNKED_BYTES", kMultiLineChunkedBytes);
    if (vec && chunked_shape && !scan_knob("HEPH_SCAN_NO_CHUNKED", 0)) {
        heph_status st = HEPH_OK;
        const T *ci = in + pr.in_base;
        T *co = out + pr.out_base;
        bool launched;
        if (reverse)
            launched = exclusive ? launch_chunked_any<T, OP, true, true>(dev, stream, ci, co, pr.len, pr.outer, pr.in_o, pr.out_o, reverse, exclusive, carry, &st)
                                 : launch_chunked_any<T, OP, true, false>(dev, stream, ci, co, pr.len, pr.outer, pr.in_o, pr.out_o, reverse, exclusive, carry, &st);
        else
            launched = exclusive ? launch_chunked_any<T, OP, false, true>(dev, stream, ci, co, pr.len, pr.outer, pr.in_o, pr.out_o, reverse, exclusive, carry, &st)
                                 : launch_chunked_any<T, OP, false, false>(dev, stream, ci, co, pr.len, pr.outer, pr.in_o, pr.out_o, reverse, exclusive, carry, &st);
        if (launched) return st;
    }
    // A single line of 640+ tiles below the chunked kernel's minimum: the
    // two-pass scan (see scan_tile_totals_kernel).  Measured per call, u32,
    // look-back -> two-pass: 6.3 M elements 18.3 -> 16.0 us, 7 M 19.1 ->
    // 15.4 us; below ~5 M the second launch costs more than the chain saves
    // (4.2 M 13.8 -> 15.7 us).
    if (pr.outer == 1) {
        const uint64_t nt = (pr.len + S::TILE - 1) / S::TILE;
        if (nt >= kTwoPassMinTiles && pr.len * sizeof(T) <= kTwoPassMaxBytes &&
            !scan_knob("HEPH_SCAN_NO_TWO_PASS", 0))
            return launch_two_pass<T, OP>(dev, stream, in + pr.in_base, out + pr.out_base, pr.len, nt, vec, reverse,
                                          exclusive, carry);
    }
    // A line shorter than one 32 KiB tile takes 16 KiB tiles (a 16 KiB line
    // fills its tile instead of idling half the CTA).
    const bool small_tile = pr.len < (uint64_t)S::TILE;
    const uint64_t tile_elems = small_tile ? (uint64_t)ScanShape<T, kLookbackVectorsSmall>::TILE : (uint64_t)S::TILE;
    const uint64_t tiles_per_line = (pr.len + tile_elems - 1) / tile_elems;
    const uint64_t tiles = tiles_per_line * pr.outer;
    if (tiles > 0x7fffffffull) return fail(HEPH_DISPATCH_FAILED, "scan grid too large");
    LookbackParams<T> p{};
    heph_status st = status_for(dev, stream, tiles, &p.status);
    if (st != HEPH_OK) return st;
    p.in = in + pr.in_base;
    p.out = out + pr.out_base;
    p.len = pr.len;
    p.tiles_per_line = tiles_per_line;
    p.lines = pr.outer;
    // Position-major numbering measured faster at every line length (u32,
    // 1 GiB, line-major -> position-major TB/s: 2 tiles per line 6.5 -> 6.8,
    // 8 tiles 5.4 -> 6.7, 64 tiles 4.3 -> 6.7, 256 tiles 3.9 -> 5.2).
    p.interleaved = pr.outer > 1 &&
                    tiles_per_line >= (uint64_t)scan_knob("HEPH_SCAN_INTERLEAVE_MIN", (int)kInterleaveMinTiles);
    p.pos_step = p.interleaved ? pr.outer : 1;
    p.in_line = pr.in_o;
    p.out_line = pr.out_o;
    p.carry = carry;
    p.err = dev->error_dev;
    p.reverse = reverse;
    p.exclusive = exclusive;
    const dim3 grid((unsigned)tiles);
    const int sel = (vec ? 4 : 0) | (reverse ? 2 : 0) | (exclusive ? 1 : 0);
    if (small_tile) launch_lookback<T, OP, kLookbackVectorsSmall>(sel, grid, stream, p);
    else launch_lookback<T, OP, kLookbackVectors>(sel, grid, stream, p);
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "scan launch");
    return HEPH_OK;
}

// ------------------------------------------------ bounded-wait self-test
//
// Runs the production waits against partners that never arrive: the
// look-back wait on a predecessor tile that never publishes (0), or the
// mbarrier wait of a staged part on a barrier nothing arrives on (1).  Each
// gives up after its bound, raises its error bit and returns, so the host
// sees the failure on its next synchronisation and the context stays usable.

__global__ void lookback_timeout_selftest_kernel(StatusView status, unsigned int *err) {
    LookbackParams<uint32_t> p{};
    p.status = status;
    p.err = err;
    p.lines = 1;
    p.pos_step = 1;
    (void)lookback<uint32_t, OP_SUM>(p, 1, 1, threadIdx.x & 31);
}

__global__ void mbar_timeout_selftest_kernel(unsigned int *err) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    mbar_wait(&bar, 0, err);
}

heph_status launch_wait_selftest(Device *dev, cudaStream_t stream, int which) {
    if (which == 1) {
        mbar_timeout_selftest_kernel<<<1, 32, 0, stream>>>(dev->error_dev);
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "wait self-test launch");
        return HEPH_OK;
    }
    unsigned long long *packed = nullptr;
    HEPH_CUDA_TRY(cudaMallocFromPoolAsync((void **)&packed, 2 * sizeof(unsigned long long), dev->pool, stream),
                  HEPH_ALLOCATION_FAILED, "wait self-test status");
    cudaMemsetAsync(packed, 0, 2 * sizeof(unsigned long long), stream);
    StatusView sv{};
    sv.epoch = 1;  // the zeroed entries carry epoch 0: never published
    sv.packed = packed;
    lookback_timeout_selftest_kernel<<<1, 32, 0, stream>>>(sv, dev->error_dev);
    const cudaError_t e = cudaGetLastError();
    cudaFreeAsync(packed, stream);
    HEPH_CUDA_TRY(e, HEPH_DISPATCH_FAILED, "wait self-test launch");
    return HEPH_OK;
}

heph_status launch_scan(Device *dev, cudaStream_t stream, int op, heph_dtype dtype, const void *in, void *out,
                        const AxisProblem &p, bool reverse, bool exclusive, const void *carry) {
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
