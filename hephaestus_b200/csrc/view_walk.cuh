// view_walk.cuh — grid-stride walks over strided N-D views without per-element
// division.
//
// A thread visits flat indices i, i + S, i + 2S, … of a (canonicalised) view,
// S = the grid's thread count.  It decodes its first index once; every later
// step adds S written in the view's mixed radix (its digits precomputed on the
// host) to the thread's coordinates, propagating at most one carry per dim, and
// moves each operand's element offset by a precomputed delta plus a per-dim
// correction when that dim wraps.  Adjacent lanes hold adjacent flat indices,
// so a unit-stride innermost dim is read coalesced.
#pragma once

#include <cstdint>

#include "device_utils.cuh"
#include "plan.h"

namespace heph {

// Kernel parameter block of a walk over NOPS operands.  Dims are outermost
// first; coordinates of dims >= 1 fit 32 bits (the host checks).
template <int NOPS> struct ViewWalk {
    uint32_t shape[HEPH_MAX_RANK];   // dims >= 1 (dim 0 is never wrapped)
    uint32_t digit[HEPH_MAX_RANK];   // S in the view's mixed radix, dims >= 1
    int64_t stride[NOPS][HEPH_MAX_RANK];
    int64_t offset[NOPS];
    int64_t delta[NOPS];             // sum over all dims of digit * stride
    int64_t adj[NOPS][HEPH_MAX_RANK];  // when dim d wraps: stride[d-1] - shape[d] * stride[d]
};

// Fills a walk of rank R (1, 2 or 4; a rank-3 view is padded with a leading
// unit dim) for a grid of `threads` threads.  False when an inner dim does not
// fit 32-bit coordinates.
template <int NOPS> inline bool make_walk(const StreamView &v, int R, uint64_t threads, ViewWalk<NOPS> *w) {
    const int pad = R - (int)v.rank;
    if (pad < 0) return false;
    uint64_t shape[HEPH_MAX_RANK];
    int64_t stride[NOPS][HEPH_MAX_RANK];
    for (int d = 0; d < R; ++d) {
        const int s = d - pad;
        shape[d] = s < 0 ? 1 : v.shape[s];
        for (int o = 0; o < NOPS; ++o) stride[o][d] = s < 0 ? 0 : v.strides[o][s];
        if (d >= 1 && shape[d] >= (1ull << 31)) return false;
    }
    *w = ViewWalk<NOPS>{};
    uint64_t rem = threads, digit0 = 0;
    for (int d = R - 1; d >= 0; --d) {
        const uint64_t dg = d == 0 ? rem : rem % shape[d];
        if (d == 0) digit0 = dg;
        else {
            rem /= shape[d];
            w->shape[d] = (uint32_t)shape[d];
            w->digit[d] = (uint32_t)dg;
        }
    }
    for (int o = 0; o < NOPS; ++o) {
        w->offset[o] = v.offset[o];
        int64_t delta = (int64_t)digit0 * stride[o][0];
        for (int d = 0; d < R; ++d) {
            w->stride[o][d] = stride[o][d];
            if (d >= 1) {
                delta += (int64_t)w->digit[d] * stride[o][d];
                w->adj[o][d] = stride[o][d - 1] - (int64_t)shape[d] * stride[o][d];
            }
        }
        w->delta[o] = delta;
    }
    return true;
}

template <int R, int NOPS> struct ViewCursor {
    uint32_t c[R];
    int64_t off[NOPS];

    __device__ __forceinline__ void seek(const ViewWalk<NOPS> &w, uint64_t i) {
#pragma unroll
        for (int o = 0; o < NOPS; ++o) off[o] = w.offset[o];
#pragma unroll
        for (int d = R - 1; d >= 1; --d) {
            c[d] = (uint32_t)(i % w.shape[d]);
            i /= w.shape[d];
#pragma unroll
            for (int o = 0; o < NOPS; ++o) off[o] += (int64_t)c[d] * w.stride[o][d];
        }
#pragma unroll
        for (int o = 0; o < NOPS; ++o) off[o] += (int64_t)i * w.stride[o][0];
    }

    __device__ __forceinline__ void advance(const ViewWalk<NOPS> &w) {
        uint32_t carry = 0;
#pragma unroll
        for (int d = R - 1; d >= 1; --d) {
            uint32_t x = c[d] + w.digit[d] + carry;  // < 2 * shape[d] < 2^32
            carry = x >= w.shape[d];
            c[d] = carry ? x - w.shape[d] : x;
#pragma unroll
            for (int o = 0; o < NOPS; ++o) off[o] += carry ? w.adj[o][d] : 0;
        }
#pragma unroll
        for (int o = 0; o < NOPS; ++o) off[o] += w.delta[o];
    }
};

}  // namespace heph

namespace heph {

// Row-run walk of a canonical view whose innermost dim has unit stride and
// `len` elements per run (a run = one setting of the outer dims): work items
// are (run, segment) pairs of at most `seg` elements, one warp per item.  A
// warp reads its segment's unaligned head and tail with scalar loads and the
// middle with 128-bit loads, so misaligned rows (a sub-block at an odd column
// offset, an odd leading dimension) still stream at full width; the run's
// offset is decoded once per item.
struct RunWalk {
    uint32_t outer_rank;                  // outer dims (0..3)
    uint64_t outer_shape[HEPH_MAX_RANK];  // outermost first
    int64_t outer_stride[HEPH_MAX_RANK];
    int64_t offset;
    uint64_t len;    // elements per run
    uint64_t seg;    // elements per segment (multiple of 32 vectors)
    uint64_t segs;   // segments per run
    uint64_t items;  // runs * segs
};

inline bool make_run_walk(const StreamView &v, size_t elem_size, uint64_t min_len, RunWalk *w) {
    const int in = (int)v.rank - 1;
    if (v.strides[0][in] != 1 || v.shape[in] < min_len) return false;
    *w = RunWalk{};
    w->outer_rank = (uint32_t)in;
    uint64_t runs = 1;
    for (int d = 0; d < in; ++d) {
        w->outer_shape[d] = v.shape[d];
        w->outer_stride[d] = v.strides[0][d];
        runs *= v.shape[d];
    }
    w->offset = v.offset[0];
    w->len = v.shape[in];
    w->seg = (16384 / elem_size);  // 16 KiB per item
    w->segs = (w->len + w->seg - 1) / w->seg;
    w->items = runs * w->segs;
    return true;
}

// Folds the view elements of RunWalk item `item` into `acc` with fold(acc, x);
// called by all 32 lanes of a warp.
template <typename T, int UNROLL, typename Acc, typename Fold>
__device__ __forceinline__ void run_item_fold(const T *__restrict__ base, const RunWalk &w, uint64_t item, int lane,
                                              Acc &acc, Fold fold) {
    constexpr int V = 16 / sizeof(T);
    const uint64_t run = item / w.segs, s = item - run * w.segs;
    int64_t off = w.offset;
    uint64_t rem = run;
#pragma unroll
    for (int d = HEPH_MAX_RANK - 1; d >= 0; --d) {
        if (d < (int)w.outer_rank) {  // constant indices keep the walk in registers
            const uint64_t c = rem % w.outer_shape[d];
            rem /= w.outer_shape[d];
            off += (int64_t)c * w.outer_stride[d];
        }
    }
    const uint64_t lo = s * w.seg;
    const uint64_t n = min(w.seg, w.len - lo);
    const T *p = base + off + (int64_t)lo;
    // Head up to a 128-byte boundary (at most one scalar per lane), so every
    // warp-wide 128-bit load covers exactly four whole cache lines.
    uint64_t head = ((128u - (reinterpret_cast<uintptr_t>(p) & 127u)) & 127u) / sizeof(T);
    if (head > n) head = n;
    const uint64_t nvec = (n - head) / V;
    if ((uint64_t)lane < head) fold(acc, __ldg(p + lane));
    const uint4 *vp = reinterpret_cast<const uint4 *>(p + head);
    uint64_t i = lane;
    for (; i + (UNROLL - 1) * 32 < nvec; i += UNROLL * 32) {
        uint4 r[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) r[u] = ld_stream(vp + i + u * 32);
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            Vec16<T> e = as_elems<T>(r[u]);
#pragma unroll
            for (int k = 0; k < V; ++k) fold(acc, e.e[k]);
        }
    }
    for (; i < nvec; i += 32) {
        Vec16<T> e = as_elems<T>(ld_stream(vp + i));
#pragma unroll
        for (int k = 0; k < V; ++k) fold(acc, e.e[k]);
    }
    const uint64_t tail = head + nvec * V;
    if ((uint64_t)lane < n - tail) fold(acc, __ldg(p + tail + lane));
}

// Grid-stride over RunWalk items, one warp per item.
template <typename T, int UNROLL, typename Acc, typename Fold>
__device__ __forceinline__ void run_walk_fold(const T *__restrict__ base, const RunWalk &w, Acc &acc, Fold fold) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t item = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); item < w.items;
         item += warps)
        run_item_fold<T, UNROLL>(base, w, item, lane, acc, fold);
}

}  // namespace heph
