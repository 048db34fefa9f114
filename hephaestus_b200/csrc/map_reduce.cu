// map_reduce.cu — fused map-reductions: dot product, trace, L1 / L2 / max
// norms of strided views (rank <= 4) in ONE launch each.
//
// The reference fuses a map into a multi-pass shared-memory tree, one element
// per thread, strided addressing decoded per element, then a separate sqrt
// kernel for the L2 norm (hephaestus-cuda application/linalg/norms.rs:91-140,
// 424-436).  Here: dense operands stream with 128-bit loads (both operands of a
// dot product in lockstep), other views decode their strides per element; the
// map is applied in registers, folded per warp / CTA, and the last CTA folds
// the per-CTA partials in order and applies the epilogue (sqrt for L2) before
// writing the scalar in place.  Views that are not one dense block are
// canonicalised jointly (both dot operands permuted / flipped / merged alike)
// and walked without per-element division (view_walk.cuh).
#include <algorithm>

#include "device_utils.cuh"
#include "kernels.h"
#include "view_walk.cuh"

namespace heph {
namespace {

constexpr int kMapThreads = 256;
constexpr int kMapUnroll = 4;

template <typename T> __device__ __forceinline__ T abs_value(T v) {
    if constexpr (is_float_v<T>) return v < T(0) ? -v : (v == T(0) ? T(0) : v);
    else if constexpr (std::is_same_v<T, uint32_t>) return v;
    else {
        using U = typename Unsigned<T>::type;
        return v < 0 ? T(U(0) - U(v)) : v;  // wraps for the most negative value, as abs() does
    }
}

// Map expressions of hephaestus-cuda application/linalg/norms.rs:55-89:
// DotMap "lhs * rhs", IdentityMap "lhs", AbsMap "abs(lhs)", SquareMap
// "lhs * lhs" (then sqrt), MaxAbsMap "abs(lhs)" folded with max.
template <typename T, int MAP> struct MapFn {
    static constexpr int REDUCE = MAP == HEPH_MAP_NORM_MAX ? OP_MAX : OP_SUM;
    static __device__ __forceinline__ T apply(T a, T b) {
        if constexpr (MAP == HEPH_MAP_DOT) return combine<T, OP_PROD>(a, b);
        else if constexpr (MAP == HEPH_MAP_SUM) return a;
        else if constexpr (MAP == HEPH_MAP_NORM_L2) return combine<T, OP_PROD>(a, a);
        else return abs_value(a);
    }
    static __device__ __forceinline__ T epilogue(T v) {
        if constexpr (MAP == HEPH_MAP_NORM_L2 && is_float_v<T>) return sqrt(v);
        else return v;
    }
};

template <typename T, int MAP>
__device__ __forceinline__ void finish_map(T acc, T *out, T *partials, unsigned int *ticket, T *scratch) {
    using F = MapFn<T, MAP>;
    acc = block_fold<T, F::REDUCE, kMapThreads>(acc, scratch);
    if (gridDim.x == 1) {
        if (threadIdx.x == 0) *out = F::epilogue(acc);
        return;
    }
    __shared__ bool am_last;
    if (threadIdx.x == 0) {
        partials[blockIdx.x] = acc;
        __threadfence();
        am_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!am_last) return;
    __threadfence();
    T a = identity<T, F::REDUCE>();
    for (unsigned int j = threadIdx.x; j < gridDim.x; j += kMapThreads) a = combine<T, F::REDUCE>(a, ld_cg(partials + j));
    a = block_fold<T, F::REDUCE, kMapThreads>(a, scratch);
    if (threadIdx.x == 0) {
        *out = F::epilogue(a);
        *ticket = 0u;
    }
}

// Both operands dense and 16-byte aligned (b == a for the unary maps).
template <typename T, int MAP>
__global__ void __launch_bounds__(kMapThreads)
    map_dense_kernel(const T *__restrict__ a, const T *__restrict__ b, uint64_t n, T *__restrict__ out,
                     T *__restrict__ partials, unsigned int *__restrict__ ticket) {
    using F = MapFn<T, MAP>;
    constexpr int V = Vec16<T>::V;
    constexpr bool BIN = MAP == HEPH_MAP_DOT;
    __shared__ T scratch[kMapThreads / 32];
    const uint64_t tid = (uint64_t)blockIdx.x * kMapThreads + threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * kMapThreads;
    const uint64_t nvec = n / V;
    const uint4 *va = reinterpret_cast<const uint4 *>(a), *vb = reinterpret_cast<const uint4 *>(b);
    T acc = identity<T, F::REDUCE>();
    auto fold = [&](uint4 ra, uint4 rb) {
        Vec16<T> ea = as_elems<T>(ra), eb = as_elems<T>(rb);
#pragma unroll
        for (int c = 0; c < V; ++c) acc = combine<T, F::REDUCE>(acc, F::apply(ea.e[c], eb.e[c]));
    };
    uint64_t i = tid;
    for (; i + (kMapUnroll - 1) * stride < nvec; i += kMapUnroll * stride) {
        uint4 ra[kMapUnroll], rb[kMapUnroll];
#pragma unroll
        for (int u = 0; u < kMapUnroll; ++u) {
            ra[u] = ld_stream(va + i + u * stride);
            rb[u] = BIN ? ld_stream(vb + i + u * stride) : ra[u];
        }
#pragma unroll
        for (int u = 0; u < kMapUnroll; ++u) fold(ra[u], rb[u]);
    }
    for (; i < nvec; i += stride) {
        const uint4 ra = ld_stream(va + i);
        fold(ra, BIN ? ld_stream(vb + i) : ra);
    }
    if (tid < n - nvec * V) {
        const uint64_t e = nvec * V + tid;
        acc = combine<T, F::REDUCE>(acc, F::apply(a[e], BIN ? b[e] : a[e]));
    }
    finish_map<T, MAP>(acc, out, partials, ticket, scratch);
}

struct MapView {
    uint32_t rank;
    uint64_t shape[HEPH_MAX_RANK];
    int64_t sa[HEPH_MAX_RANK], sb[HEPH_MAX_RANK];
    int64_t oa, ob;
};

template <typename T, int MAP>
__global__ void __launch_bounds__(kMapThreads)
    map_strided_kernel(const T *__restrict__ a, const T *__restrict__ b, MapView v, uint64_t n, T *__restrict__ out,
                       T *__restrict__ partials, unsigned int *__restrict__ ticket) {
    using F = MapFn<T, MAP>;
    __shared__ T scratch[kMapThreads / 32];
    T acc = identity<T, F::REDUCE>();
    const uint64_t stride = (uint64_t)gridDim.x * kMapThreads;
    for (uint64_t i = (uint64_t)blockIdx.x * kMapThreads + threadIdx.x; i < n; i += stride) {
        uint64_t rem = i;
        int64_t pa = v.oa, pb = v.ob;
        for (int d = (int)v.rank - 1; d >= 0; --d) {
            const uint64_t c = rem % v.shape[d];
            rem /= v.shape[d];
            pa += (int64_t)c * v.sa[d];
            pb += (int64_t)c * v.sb[d];
        }
        acc = combine<T, F::REDUCE>(acc, F::apply(a[pa], b[pb]));
    }
    finish_map<T, MAP>(acc, out, partials, ticket, scratch);
}

// Canonical strided view(s), walked without division; `n` counts walk units
// (elements, or 16-byte vectors when VEC).  NOPS = 2 walks the dot product's
// operands in lockstep.
template <typename T, int MAP, int R, bool VEC, int NOPS>
__global__ void __launch_bounds__(kMapThreads)
    map_walk_kernel(const T *__restrict__ a, const T *__restrict__ b, const ViewWalk<NOPS> w, uint64_t n,
                    T *__restrict__ out, T *__restrict__ partials, unsigned int *__restrict__ ticket) {
    using F = MapFn<T, MAP>;
    constexpr int V = Vec16<T>::V;
    __shared__ T scratch[kMapThreads / 32];
    const uint64_t stride = (uint64_t)gridDim.x * kMapThreads;
    uint64_t i = (uint64_t)blockIdx.x * kMapThreads + threadIdx.x;
    T acc = identity<T, F::REDUCE>();
    ViewCursor<R, NOPS> cur;
    if (i < n) cur.seek(w, i);
    const int64_t *ob = &cur.off[NOPS - 1];
    auto fold_vec = [&](uint4 ra, uint4 rb) {
        Vec16<T> ea = as_elems<T>(ra), eb = as_elems<T>(rb);
#pragma unroll
        for (int c = 0; c < V; ++c) acc = combine<T, F::REDUCE>(acc, F::apply(ea.e[c], eb.e[c]));
    };
    for (; i + (kMapUnroll - 1) * stride < n; i += kMapUnroll * stride) {
        if constexpr (VEC) {
            uint4 ra[kMapUnroll], rb[kMapUnroll];
#pragma unroll
            for (int u = 0; u < kMapUnroll; ++u) {
                ra[u] = ld_stream(reinterpret_cast<const uint4 *>(a) + cur.off[0]);
                rb[u] = NOPS == 2 ? ld_stream(reinterpret_cast<const uint4 *>(b) + *ob) : ra[u];
                cur.advance(w);
            }
#pragma unroll
            for (int u = 0; u < kMapUnroll; ++u) fold_vec(ra[u], rb[u]);
        } else {
            T ra[kMapUnroll], rb[kMapUnroll];
#pragma unroll
            for (int u = 0; u < kMapUnroll; ++u) {
                ra[u] = __ldg(a + cur.off[0]);
                rb[u] = NOPS == 2 ? __ldg(b + *ob) : ra[u];
                cur.advance(w);
            }
#pragma unroll
            for (int u = 0; u < kMapUnroll; ++u) acc = combine<T, F::REDUCE>(acc, F::apply(ra[u], rb[u]));
        }
    }
    for (; i < n; i += stride) {
        if constexpr (VEC) {
            const uint4 ra = ld_stream(reinterpret_cast<const uint4 *>(a) + cur.off[0]);
            fold_vec(ra, NOPS == 2 ? ld_stream(reinterpret_cast<const uint4 *>(b) + *ob) : ra);
        } else {
            const T ra = __ldg(a + cur.off[0]);
            acc = combine<T, F::REDUCE>(acc, F::apply(ra, NOPS == 2 ? __ldg(b + *ob) : ra));
        }
        cur.advance(w);
    }
    finish_map<T, MAP>(acc, out, partials, ticket, scratch);
}

// Unary map over unit-stride runs that are not 16-byte aligned (RunWalk).
template <typename T, int MAP>
__global__ void __launch_bounds__(kMapThreads)
    map_runs_kernel(const T *__restrict__ a, const RunWalk w, T *__restrict__ out, T *__restrict__ partials,
                    unsigned int *__restrict__ ticket) {
    using F = MapFn<T, MAP>;
    __shared__ T scratch[kMapThreads / 32];
    T acc = identity<T, F::REDUCE>();
    run_walk_fold<T, 2 * kMapUnroll>(a, w, acc, [](T &s, T x) { s = combine<T, F::REDUCE>(s, F::apply(x, x)); });
    finish_map<T, MAP>(acc, out, partials, ticket, scratch);
}

// Launches map_walk_kernel; false (nothing launched) when an inner dim of the
// canonical view exceeds 32-bit coordinates.
template <typename T, int MAP, int NOPS>
bool launch_map_walk(cudaStream_t stream, const T *a, const heph_layout &la, const T *b, const heph_layout &lb,
                     uint64_t n, unsigned grid, T *out, T *partials, unsigned int *ticket) {
    StreamView sv;
    const heph_layout *ls[2] = {&la, &lb};
    stream_view(ls, NOPS, &sv);
    constexpr uint32_t V = 16 / sizeof(T);
    const void *bases[2] = {a, b};
    const bool vec = sv.rank >= 2 && stream_view_vectorize(&sv, NOPS, V, bases, sizeof(T));
    const dim3 g(grid), bl(kMapThreads);
    if constexpr (NOPS == 1) {
        RunWalk runs;
        if (!vec && make_run_walk(sv, sizeof(T), 128, &runs)) {
            map_runs_kernel<T, MAP><<<g, bl, 0, stream>>>(a, runs, out, partials, ticket);
            return true;
        }
    }
    const uint64_t units = vec ? n / V : n;
    if (sv.rank == 1 && sv.strides[0][0] == 1 && sv.strides[NOPS - 1][0] == 1) {
        // Both operands one dense block, visited alike (e.g. both transposed).
        const T *pa = a + sv.offset[0], *pb = NOPS == 2 ? b + sv.offset[1] : pa;
        if (((reinterpret_cast<uintptr_t>(pa) | reinterpret_cast<uintptr_t>(pb)) & 15u) == 0) {
            map_dense_kernel<T, MAP><<<g, bl, 0, stream>>>(pa, pb, n, out, partials, ticket);
            return true;
        }
    }
    const int R = sv.rank == 1 ? 1 : sv.rank == 2 ? 2 : 4;
    ViewWalk<NOPS> w;
    if (!make_walk<NOPS>(sv, R, (uint64_t)grid * kMapThreads, &w)) return false;
    if (vec) {
        if (R == 2) map_walk_kernel<T, MAP, 2, true, NOPS><<<g, bl, 0, stream>>>(a, b, w, units, out, partials, ticket);
        else map_walk_kernel<T, MAP, 4, true, NOPS><<<g, bl, 0, stream>>>(a, b, w, units, out, partials, ticket);
    } else {
        if (R == 1) map_walk_kernel<T, MAP, 1, false, NOPS><<<g, bl, 0, stream>>>(a, b, w, units, out, partials, ticket);
        else if (R == 2) map_walk_kernel<T, MAP, 2, false, NOPS><<<g, bl, 0, stream>>>(a, b, w, units, out, partials, ticket);
        else map_walk_kernel<T, MAP, 4, false, NOPS><<<g, bl, 0, stream>>>(a, b, w, units, out, partials, ticket);
    }
    return true;
}

template <typename T, int MAP> __global__ void map_identity_kernel(T *out) {
    using F = MapFn<T, MAP>;
    *out = F::epilogue(identity<T, F::REDUCE>());
}

template <typename T, int MAP>
heph_status launch_map_typed(Device *dev, cudaStream_t stream, const T *a, const heph_layout &la, const T *b,
                             const heph_layout &lb, uint64_t n, T *out) {
    if (n == 0) {
        map_identity_kernel<T, MAP><<<1, 1, 0, stream>>>(out);
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "map reduction launch");
        return HEPH_OK;
    }
    const T *pa = a + la.offset, *pb = b + lb.offset;
    bool contiguous = layout_is_dense(la) && layout_is_dense(lb);
    int64_t first = 0;
    if (!contiguous && MAP != HEPH_MAP_DOT && layout_covers_dense_block(la, &first)) {
        // Unary maps fold order-insensitively: a permuted / reversed dense
        // block streams contiguously.
        pa = pb = a + first;
        contiguous = true;
    }
    const bool dense = contiguous && (reinterpret_cast<uintptr_t>(pa) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(pb) & 15u) == 0;
    const uint64_t per_cta = (uint64_t)kMapThreads * kMapUnroll * (16 / sizeof(T));
    const uint64_t cap = (uint64_t)dev->sm_count * (2048 / kMapThreads);
    const unsigned grid = (unsigned)std::max<uint64_t>(1, std::min((n + per_cta - 1) / per_cta, cap));
    std::lock_guard<std::mutex> lock(dev->mu);
    Workspace *ws = nullptr;
    heph_status st = workspace_for(dev, stream, (size_t)grid * sizeof(T), 0, &ws);
    if (st != HEPH_OK) return st;
    T *partials = static_cast<T *>(ws->partials);
    unsigned int *ticket = ws->tickets + 2;  // tickets[0]: full reductions, [1]: scans
    constexpr int NOPS = MAP == HEPH_MAP_DOT ? 2 : 1;
    if (dense) {
        map_dense_kernel<T, MAP><<<grid, kMapThreads, 0, stream>>>(pa, pb, n, out, partials, ticket);
    } else if (!launch_map_walk<T, MAP, NOPS>(stream, a, la, b, lb, n, grid, out, partials, ticket)) {
        MapView v{};
        v.rank = la.rank;
        for (uint32_t d = 0; d < la.rank; ++d) {
            v.shape[d] = la.shape[d];
            v.sa[d] = la.strides[d];
            v.sb[d] = lb.strides[d];
        }
        v.oa = (int64_t)la.offset;
        v.ob = (int64_t)lb.offset;
        map_strided_kernel<T, MAP><<<grid, kMapThreads, 0, stream>>>(a, b, v, n, out, partials, ticket);
    }
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "map reduction launch");
    return HEPH_OK;
}

}  // namespace

heph_status launch_map_reduce(Device *dev, cudaStream_t stream, int map, heph_dtype dtype, const void *a,
                              const heph_layout &la, const void *b, const heph_layout &lb, uint64_t count,
                              void *out) {
    return dispatch_dtype(dtype, [&]<typename T>() -> heph_status {
        const T *ta = static_cast<const T *>(a), *tb = static_cast<const T *>(b);
        T *to = static_cast<T *>(out);
        switch (map) {
            case HEPH_MAP_DOT: return launch_map_typed<T, HEPH_MAP_DOT>(dev, stream, ta, la, tb, lb, count, to);
            case HEPH_MAP_SUM: return launch_map_typed<T, HEPH_MAP_SUM>(dev, stream, ta, la, tb, lb, count, to);
            case HEPH_MAP_NORM_L1: return launch_map_typed<T, HEPH_MAP_NORM_L1>(dev, stream, ta, la, tb, lb, count, to);
            case HEPH_MAP_NORM_L2: return launch_map_typed<T, HEPH_MAP_NORM_L2>(dev, stream, ta, la, tb, lb, count, to);
            case HEPH_MAP_NORM_MAX: return launch_map_typed<T, HEPH_MAP_NORM_MAX>(dev, stream, ta, la, tb, lb, count, to);
        }
        return fail(HEPH_INVALID_CONFIGURATION, "unknown map reduction");
    });
}

}  // namespace heph
