// reduce_axis.cu — rank-2 keepdims axis reductions (and arg-reductions) for
// sm_100a.
//
// The reference runs one thread per output with a serial loop over the
// reduced axis (hephaestus-cuda application/reduction.rs:218-249): for
// axis 1 of a row-major matrix adjacent threads read addresses a whole row
// apart.  Here the canonical problem out[o] = fold_r in[base + o*so + r*sr]
// is mapped by the stride of the reduced axis:
//   * sr == 1 ("row" reduction): one warp per (row, segment); lanes read
//     128-bit vectors that are contiguous across the warp; warp fold of the
//     value (and of the (value, index) pair for arg-reductions, lowest index
//     winning ties).  Few long rows are split into segments whose partials a
//     second kernel folds in segment order.
//   * otherwise ("column" reduction): one thread per output (V adjacent
//     outputs per 128-bit vector when so == 1), a serial fold down its column
//     slice with 4 independent loads in flight; the rows are split into
//     slices across grid.y so that all SMs stream, and a second kernel folds
//     the slices in order.
#include <algorithm>

#include "device_utils.cuh"
#include "kernels.h"

namespace heph {

constexpr int kRowThreads = 256;  // 8 warps per CTA
constexpr int kColThreads = 256;

struct AxisArgs {
    int64_t in_base, in_o, in_r;
    uint64_t lead;  // column kernel, vector form: columns before output 0 in its first 16-byte vector
    int64_t out_base, out_o;
    int64_t idx_base, idx_o;
    uint64_t outer, len;
    uint64_t splits, seg;  // segments per output and elements per segment
};

template <typename T, int OP, bool MEAN>
__device__ __forceinline__ T finish_value(T acc, uint64_t len) {
    if constexpr (MEAN) return (T)(acc / (T)len);
    else return acc;
}

// -------------------------------------------------------------- row kernel

template <typename T, int OP, bool ARG, bool VEC, bool MEAN>
__global__ void __launch_bounds__(kRowThreads)
    row_reduce_kernel(const T *__restrict__ in, AxisArgs a, T *__restrict__ out,
                      uint32_t *__restrict__ idx, T *__restrict__ pv, uint32_t *__restrict__ pi) {
    constexpr int V = Vec16<T>::V;
    constexpr int U = 4;
    const uint64_t warp = ((uint64_t)blockIdx.x * kRowThreads + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= a.outer * a.splits) return;
    const uint64_t o = warp / a.splits, s = warp % a.splits;
    const uint64_t r0 = s * a.seg;
    const uint64_t r1 = min(a.len, r0 + a.seg);
    const T *row = in + a.in_base + (int64_t)o * a.in_o;

    T acc = ARG ? T(0) : identity<T, OP>();
    uint32_t best = 0xffffffffu;  // "no element yet" for arg-reductions
    auto take = [&](T v, uint64_t r) {
        if constexpr (ARG) {
            if (best == 0xffffffffu || (OP == OP_MAX ? v > acc : v < acc)) {
                acc = v;
                best = (uint32_t)r;
            }
        } else {
            acc = combine<T, OP>(acc, v);
        }
    };

    uint64_t r = r0;
    if constexpr (VEC) {
        // Each (row, segment) aligns itself: a head of at most V - 1 elements
        // (one per lane) up to the first 16-byte boundary, then 128-bit loads.
        // Every lane still visits its indices in increasing order, which the
        // arg-reductions' lowest-index tie-break relies on.
        uint64_t head = ((16u - (reinterpret_cast<uintptr_t>(row + r0) & 15u)) & 15u) / sizeof(T);
        if (head > r1 - r0) head = r1 - r0;
        // The head element is loaded now and folded after the body, so its
        // load does not hold back the vector loads.
        const bool has_head = (uint64_t)lane < head;
        const T hv = has_head ? row[r0 + lane] : T(0);
        const uint64_t rv = r0 + head;
        const uint64_t nv = (r1 - rv) / V;
        const uint4 *vrow = reinterpret_cast<const uint4 *>(row + rv);
        uint64_t k = lane;
        for (; k + 32 * (U - 1) < nv; k += 32 * U) {
            uint4 raw[U];
#pragma unroll
            for (int u = 0; u < U; ++u) raw[u] = ld_stream(vrow + k + 32 * u);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                Vec16<T> e = as_elems<T>(raw[u]);
#pragma unroll
                for (int c = 0; c < V; ++c) take(e.e[c], rv + (k + 32 * u) * V + c);
            }
        }
        for (; k < nv; k += 32) {
            Vec16<T> e = as_elems<T>(ld_stream(vrow + k));
#pragma unroll
            for (int c = 0; c < V; ++c) take(e.e[c], rv + k * V + c);
        }
        r = rv + nv * V;
        for (uint64_t q = r + lane; q < r1; q += 32) take(row[q], q);
        r = r1;
        if (has_head) {
            const uint32_t hi = (uint32_t)(r0 + lane);
            if constexpr (ARG) {
                // Folded out of index order: the index-aware comparison keeps
                // the lowest index among equal extrema.
                if (best == 0xffffffffu || arg_better<T, OP>(hv, hi, acc, best)) {
                    acc = hv;
                    best = hi;
                }
            } else {
                acc = combine<T, OP>(acc, hv);
            }
        }
    }
    for (uint64_t q = r + lane; q < r1; q += 32) take(row[q], q);

    if constexpr (ARG) {
        warp_arg_fold<T, OP>(acc, best);
    } else {
        acc = warp_fold<T, OP>(acc);
    }
    if (lane == 0) {
        if (a.splits == 1) {
            out[a.out_base + (int64_t)o * a.out_o] = finish_value<T, OP, MEAN>(acc, a.len);
            if constexpr (ARG) idx[a.idx_base + (int64_t)o * a.idx_o] = best;
        } else {
            pv[warp] = acc;
            if constexpr (ARG) pi[warp] = best;
        }
    }
}

// Folds the per-segment partials of each output in segment order.
template <typename T, int OP, bool ARG, bool MEAN>
__global__ void split_finalize_kernel(AxisArgs a, const T *__restrict__ pv,
                                      const uint32_t *__restrict__ pi, uint64_t pv_o,
                                      uint64_t pv_s, T *__restrict__ out,
                                      uint32_t *__restrict__ idx) {
    const uint64_t o = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= a.outer) return;
    T acc = ARG ? T(0) : identity<T, OP>();
    uint32_t best = 0xffffffffu;
    for (uint64_t s = 0; s < a.splits; ++s) {
        T v = pv[o * pv_o + s * pv_s];
        if constexpr (ARG) {
            uint32_t i = pi[o * pv_o + s * pv_s];
            if (i == 0xffffffffu) continue;
            if (best == 0xffffffffu || arg_better<T, OP>(v, i, acc, best)) {
                acc = v;
                best = i;
            }
        } else {
            acc = combine<T, OP>(acc, v);
        }
    }
    out[a.out_base + (int64_t)o * a.out_o] = finish_value<T, OP, MEAN>(acc, a.len);
    if constexpr (ARG) idx[a.idx_base + (int64_t)o * a.idx_o] = best;
}

// ----------------------------------------------------------- column kernel

// grid.x covers the outputs (V per thread when VEC), grid.y the row slices.
template <typename T, int OP, bool ARG, bool VEC, bool MEAN>
__global__ void __launch_bounds__(kColThreads)
    col_reduce_kernel(const T *__restrict__ in, AxisArgs a, T *__restrict__ out,
                      uint32_t *__restrict__ idx, T *__restrict__ pv, uint32_t *__restrict__ pi) {
    constexpr int V = VEC ? Vec16<T>::V : 1;
    constexpr int U = 4;
    const uint64_t t = (uint64_t)blockIdx.x * kColThreads + threadIdx.x;
    // Vector form: thread t covers the 16-byte vector of virtual columns
    // [tV, tV + V); virtual column v is output v - lead.  The first and last
    // vectors may hold columns outside the view: they are loaded (a 16-byte
    // vector never leaves the page of the view element it holds) and masked.
    const uint64_t lead = VEC ? a.lead : 0;
    const uint64_t o0 = t * V;
    if (o0 >= a.outer + lead) return;
    uint32_t vmask = 0;
#pragma unroll
    for (int c = 0; c < V; ++c)
        if (o0 + c >= lead && o0 + c < lead + a.outer) vmask |= 1u << c;
    const uint64_t s = blockIdx.y;
    const uint64_t r0 = s * a.seg;
    const uint64_t r1 = min(a.len, r0 + a.seg);

    T acc[V];
    uint32_t best[V];
#pragma unroll
    for (int c = 0; c < V; ++c) {
        acc[c] = ARG ? T(0) : identity<T, OP>();
        best[c] = 0xffffffffu;
    }
    auto take = [&](int c, T v, uint64_t r) {
        if constexpr (ARG) {
            if (best[c] == 0xffffffffu || (OP == OP_MAX ? v > acc[c] : v < acc[c])) {
                acc[c] = v;
                best[c] = (uint32_t)r;
            }
        } else {
            acc[c] = combine<T, OP>(acc[c], v);
        }
    };

    if constexpr (VEC) {
        // Full vector of V outputs (the launcher routes a ragged last vector
        // through the scalar instantiation).
        const T *col = in + a.in_base - (int64_t)lead + (int64_t)o0;
        const bool all = vmask == (1u << V) - 1;
        uint64_t r = r0;
        for (; r + U <= r1; r += U) {
            uint4 raw[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
                raw[u] = ld_stream(reinterpret_cast<const uint4 *>(col + (int64_t)(r + u) * a.in_r));
#pragma unroll
            for (int u = 0; u < U; ++u) {
                Vec16<T> e = as_elems<T>(raw[u]);
#pragma unroll
                for (int c = 0; c < V; ++c)
                    if (all || ((vmask >> c) & 1u)) take(c, e.e[c], r + u);
            }
        }
        for (; r < r1; ++r) {
            Vec16<T> e =
                as_elems<T>(ld_stream(reinterpret_cast<const uint4 *>(col + (int64_t)r * a.in_r)));
#pragma unroll
            for (int c = 0; c < V; ++c)
                if (all || ((vmask >> c) & 1u)) take(c, e.e[c], r);
        }
    } else {
        const T *col = in + a.in_base + (int64_t)o0 * a.in_o;
        uint64_t r = r0;
        for (; r + U <= r1; r += U) {
            T x[U];
#pragma unroll
            for (int u = 0; u < U; ++u) x[u] = __ldg(col + (int64_t)(r + u) * a.in_r);
#pragma unroll
            for (int u = 0; u < U; ++u) take(0, x[u], r + u);
        }
        for (; r < r1; ++r) take(0, __ldg(col + (int64_t)r * a.in_r), r);
    }

#pragma unroll
    for (int c = 0; c < V; ++c) {
        if (VEC && !((vmask >> c) & 1u)) continue;
        const uint64_t o = o0 + c - lead;
        if (o >= a.outer) break;
        if (gridDim.y == 1) {
            T v = acc[c];
            if (ARG && best[c] == 0xffffffffu)
                v = (OP == OP_MAX) ? Limits<T>::lowest() : Limits<T>::highest();
            out[a.out_base + (int64_t)o * a.out_o] = finish_value<T, OP, MEAN>(v, a.len);
            if constexpr (ARG) idx[a.idx_base + (int64_t)o * a.idx_o] = best[c];
        } else {
            pv[s * a.outer + o] = acc[c];
            if constexpr (ARG) pi[s * a.outer + o] = best[c];
        }
    }
}

// Small column reductions in ONE launch: a CTA covers 32 column vectors (V
// columns each when VEC), its 8 warps stride over the rows (warp w takes rows
// w, w+8, ...), and the per-warp partials are folded in shared memory in warp
// order (index-aware for arg-reductions, so the lowest row index wins ties).
// No row split, no second kernel: for a 256 x 256 matrix the whole reduction
// is two CTAs and one launch.
constexpr int kTileWarps = 8;
template <typename T, int OP, bool ARG, bool VEC, bool MEAN>
__global__ void __launch_bounds__(32 * kTileWarps)
    col_tile_kernel(const T *__restrict__ in, AxisArgs a, T *__restrict__ out, uint32_t *__restrict__ idx) {
    constexpr int V = VEC ? Vec16<T>::V : 1;
    constexpr int U = 4;
    __shared__ T s_acc[kTileWarps][32 * V];
    __shared__ uint32_t s_idx[ARG ? kTileWarps : 1][ARG ? 32 * V : 1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t lead = VEC ? a.lead : 0;
    const uint64_t o0 = ((uint64_t)blockIdx.x * 32 + lane) * V;  // virtual column of element 0 of this lane
    uint32_t vmask = 0;
#pragma unroll
    for (int c = 0; c < V; ++c)
        if (o0 + c >= lead && o0 + c < lead + a.outer) vmask |= 1u << c;
    T acc[V];
    uint32_t best[V];
#pragma unroll
    for (int c = 0; c < V; ++c) {
        acc[c] = ARG ? T(0) : identity<T, OP>();
        best[c] = 0xffffffffu;
    }
    auto take = [&](int c, T v, uint64_t r) {
        if constexpr (ARG) {
            if (best[c] == 0xffffffffu || (OP == OP_MAX ? v > acc[c] : v < acc[c])) {
                acc[c] = v;
                best[c] = (uint32_t)r;
            }
        } else {
            acc[c] = combine<T, OP>(acc[c], v);
        }
    };
    if (vmask) {
        if constexpr (VEC) {
            const T *col = in + a.in_base - (int64_t)lead + (int64_t)o0;
            uint64_t r = warp;
            for (; r + (U - 1) * kTileWarps < a.len; r += U * kTileWarps) {
                uint4 raw[U];
#pragma unroll
                for (int u = 0; u < U; ++u)
                    raw[u] = ld_stream(reinterpret_cast<const uint4 *>(col + (int64_t)(r + u * kTileWarps) * a.in_r));
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    Vec16<T> e = as_elems<T>(raw[u]);
#pragma unroll
                    for (int c = 0; c < V; ++c)
                        if ((vmask >> c) & 1u) take(c, e.e[c], r + u * kTileWarps);
                }
            }
            for (; r < a.len; r += kTileWarps) {
                Vec16<T> e = as_elems<T>(ld_stream(reinterpret_cast<const uint4 *>(col + (int64_t)r * a.in_r)));
#pragma unroll
                for (int c = 0; c < V; ++c)
                    if ((vmask >> c) & 1u) take(c, e.e[c], r);
            }
        } else {
            const T *col = in + a.in_base + (int64_t)o0 * a.in_o;
            uint64_t r = warp;
            for (; r + (U - 1) * kTileWarps < a.len; r += U * kTileWarps) {
                T x[U];
#pragma unroll
                for (int u = 0; u < U; ++u) x[u] = __ldg(col + (int64_t)(r + u * kTileWarps) * a.in_r);
#pragma unroll
                for (int u = 0; u < U; ++u) take(0, x[u], r + u * kTileWarps);
            }
            for (; r < a.len; r += kTileWarps) take(0, __ldg(col + (int64_t)r * a.in_r), r);
        }
    }
#pragma unroll
    for (int c = 0; c < V; ++c) {
        s_acc[warp][lane * V + c] = acc[c];
        if constexpr (ARG) s_idx[warp][lane * V + c] = best[c];
    }
    __syncthreads();
    // Thread t folds column t of the CTA over the warps, in warp order.
    for (int t = threadIdx.x; t < 32 * V; t += 32 * kTileWarps) {
        const uint64_t vcol = (uint64_t)blockIdx.x * 32 * V + t;
        if (vcol < lead || vcol >= lead + a.outer) continue;
        const uint64_t o = vcol - lead;
        T f = ARG ? T(0) : identity<T, OP>();
        uint32_t fi = 0xffffffffu;
        for (int w = 0; w < kTileWarps; ++w) {
            const T v = s_acc[w][t];
            if constexpr (ARG) {
                const uint32_t i = s_idx[w][t];
                if (i != 0xffffffffu && (fi == 0xffffffffu || arg_better<T, OP>(v, i, f, fi))) {
                    f = v;
                    fi = i;
                }
            } else {
                f = combine<T, OP>(f, v);
            }
        }
        if (ARG && fi == 0xffffffffu) f = (OP == OP_MAX) ? Limits<T>::lowest() : Limits<T>::highest();
        out[a.out_base + (int64_t)o * a.out_o] = finish_value<T, OP, MEAN>(f, a.len);
        if constexpr (ARG) idx[a.idx_base + (int64_t)o * a.idx_o] = fi;
    }
}

// ------------------------------------------------------------------ launch


template <typename T, int OP, bool ARG, bool MEAN>
static heph_status launch_axis_typed(Device *dev, cudaStream_t stream, const T *in,
                                     const AxisProblem &p, T *out, uint32_t *idx, int64_t idx_base,
                                     int64_t idx_o) {
    constexpr int V = Vec16<T>::V;
    AxisArgs a{};
    a.in_base = p.in_base;
    a.in_o = p.in_o;
    a.in_r = p.in_r;
    a.out_base = p.out_base;
    a.out_o = p.out_o;
    a.idx_base = idx_base;
    a.idx_o = idx_o;
    a.outer = p.outer;
    a.len = p.len;
    const uint64_t resident_threads = (uint64_t)dev->sm_count * 2048;

    if (p.in_r == 1) {
        // Row reduction: one warp per (row, segment).
        // 128-bit loads whenever a row holds more than a few vectors: each
        // (row, segment) aligns its own start, so misaligned rows (odd column
        // offsets, odd leading dimensions) stream at full width too.
        const bool vec = p.len >= 4 * V;
        const uint64_t warps_wanted = resident_threads / 32 * 2;
        uint64_t splits = 1;
        if (p.outer < warps_wanted && p.len >= 8192) {
            splits = std::min<uint64_t>((warps_wanted + p.outer - 1) / p.outer, p.len / 4096);
            splits = std::max<uint64_t>(splits, 1);
        }
        uint64_t seg = (p.len + splits - 1) / splits;
        seg = (seg + 32 * V - 1) / (32 * V) * (32 * V);  // vector-aligned segments
        seg = std::max<uint64_t>(seg, 32 * V);             // an empty axis still gets one segment
        splits = std::max<uint64_t>(1, (p.len + seg - 1) / seg);
        a.splits = splits;
        a.seg = std::max<uint64_t>(seg, 1);
        const uint64_t warps = p.outer * splits;
        const uint64_t blocks = (warps * 32 + kRowThreads - 1) / kRowThreads;
        if (blocks > 0x7fffffffull) return fail(HEPH_DISPATCH_FAILED, "axis reduction grid too large");

        std::lock_guard<std::mutex> lock(dev->mu);
        Workspace *ws = nullptr;
        size_t pbytes = splits > 1 ? (size_t)warps * (sizeof(T) + sizeof(uint32_t)) : 0;
        heph_status st = workspace_for(dev, stream, pbytes, 0, &ws);
        if (st != HEPH_OK) return st;
        T *pv = static_cast<T *>(ws->partials);
        uint32_t *pi = reinterpret_cast<uint32_t *>(static_cast<char *>(ws->partials) + warps * sizeof(T));
        if (vec)
            row_reduce_kernel<T, OP, ARG, true, MEAN>
                <<<(unsigned)blocks, kRowThreads, 0, stream>>>(in, a, out, idx, pv, pi);
        else
            row_reduce_kernel<T, OP, ARG, false, MEAN>
                <<<(unsigned)blocks, kRowThreads, 0, stream>>>(in, a, out, idx, pv, pi);
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "row reduction launch");
        if (splits > 1) {
            unsigned fb = (unsigned)((p.outer + 255) / 256);
            split_finalize_kernel<T, OP, ARG, MEAN>
                <<<fb, 256, 0, stream>>>(a, pv, pi, splits, 1, out, idx);
            HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "row finalize launch");
        }
        return HEPH_OK;
    }

    // Column reduction: thread per output (vector of V outputs when the
    // outputs are adjacent in memory and the row stride is a multiple of 16
    // bytes).  A view starting off a 16-byte boundary (an odd column offset)
    // runs its first few columns scalar and vectorises the rest.
    const bool vec_ok = p.in_o == 1 && p.outer >= (uint64_t)V &&
                        (p.len <= 1 || ((uint64_t)p.in_r * sizeof(T)) % 16 == 0);
    const uint64_t lead = vec_ok ? (reinterpret_cast<uintptr_t>(in + p.in_base) & 15u) / sizeof(T) : 0;
    a.lead = lead;
    if (p.outer == 0) return HEPH_OK;
    if (p.len <= 1024 && p.len * p.outer <= (1u << 20)) {
        // Small: one launch of column tiles, rows spread over the CTA's warps.
        const uint64_t per_cta = 32 * (vec_ok ? (uint64_t)V : 1);
        const uint64_t ctas = (lead + p.outer + per_cta - 1) / per_cta;
        if (vec_ok)
            col_tile_kernel<T, OP, ARG, true, MEAN><<<(unsigned)ctas, 32 * kTileWarps, 0, stream>>>(in, a, out, idx);
        else
            col_tile_kernel<T, OP, ARG, false, MEAN><<<(unsigned)ctas, 32 * kTileWarps, 0, stream>>>(in, a, out, idx);
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "column reduction launch");
        return HEPH_OK;
    }
    std::lock_guard<std::mutex> lock(dev->mu);
    // One launch: vectors over all outputs (edge vectors masked), or scalar.
    struct Part {
        uint64_t o_begin, o_count;
        bool vec;
    } parts[1] = {{0, p.outer, vec_ok}};
    // Row slices: enough CTAs for two waves, slices of at least 64 rows.
    const uint64_t threads_x = vec_ok ? (lead + p.outer + V - 1) / V : p.outer;
    const uint64_t blocks_x_total = (threads_x + kColThreads - 1) / kColThreads;
    const uint64_t cta_wanted = (uint64_t)dev->sm_count * (2048 / kColThreads) * 2;
    uint64_t splits = 1;
    if (blocks_x_total < cta_wanted && p.len >= 128)
        splits = std::min<uint64_t>((cta_wanted + blocks_x_total - 1) / blocks_x_total, p.len / 64);
    splits = std::max<uint64_t>(1, std::min<uint64_t>(splits, 65535));
    uint64_t seg = std::max<uint64_t>(1, (p.len + splits - 1) / splits);
    splits = std::max<uint64_t>(1, (p.len + seg - 1) / seg);

    Workspace *ws = nullptr;
    size_t pbytes = splits > 1 ? (size_t)(splits * p.outer) * (sizeof(T) + sizeof(uint32_t)) : 0;
    heph_status st = workspace_for(dev, stream, pbytes, 0, &ws);
    if (st != HEPH_OK) return st;
    T *pv = static_cast<T *>(ws->partials);
    uint32_t *pi = reinterpret_cast<uint32_t *>(static_cast<char *>(ws->partials) +
                                                splits * p.outer * sizeof(T));
    for (const Part &part : parts) {
        if (part.o_count == 0) continue;
        AxisArgs b = a;
        b.splits = splits;
        b.seg = seg;
        // Shift the problem so that output 0 of this part is o_begin; the
        // partial arrays keep the full `outer` stride.
        b.in_base = a.in_base + (int64_t)part.o_begin * a.in_o;
        b.out_base = a.out_base + (int64_t)part.o_begin * a.out_o;
        b.idx_base = a.idx_base + (int64_t)part.o_begin * a.idx_o;
        b.outer = part.o_count;
        const uint64_t tx = part.vec ? threads_x : part.o_count;
        dim3 grid((unsigned)((tx + kColThreads - 1) / kColThreads), (unsigned)splits);
        // Partials of this part are written at [s * outer_part + o]; give each
        // part its own region so the finalize below can address them.
        T *ppv = pv + part.o_begin * splits;
        uint32_t *ppi = pi + part.o_begin * splits;
        if (part.vec)
            col_reduce_kernel<T, OP, ARG, true, MEAN><<<grid, kColThreads, 0, stream>>>(in, b, out, idx, ppv, ppi);
        else
            col_reduce_kernel<T, OP, ARG, false, MEAN><<<grid, kColThreads, 0, stream>>>(in, b, out, idx, ppv, ppi);
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "column reduction launch");
        if (splits > 1) {
            unsigned fb = (unsigned)((part.o_count + 255) / 256);
            split_finalize_kernel<T, OP, ARG, MEAN>
                <<<fb, 256, 0, stream>>>(b, ppv, ppi, 1, part.o_count, out, idx);
            HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "column finalize launch");
        }
    }
    return HEPH_OK;
}

template <typename T, int OP, bool ARG>
static heph_status launch_mean(Device *dev, cudaStream_t s, const T *in, const AxisProblem &p, T *out,
                               bool mean, uint32_t *idx, int64_t ib, int64_t io) {
    if (mean) return launch_axis_typed<T, OP, ARG, true>(dev, s, in, p, out, idx, ib, io);
    return launch_axis_typed<T, OP, ARG, false>(dev, s, in, p, out, idx, ib, io);
}

heph_status launch_reduce_axis(Device *dev, cudaStream_t stream, int op, heph_dtype dtype,
                               const void *in, const AxisProblem &p, void *out, bool mean,
                               uint32_t *indices, int64_t idx_base, int64_t idx_o) {
    return dispatch_dtype(dtype, [&]<typename T>() -> heph_status {
        const T *ti = static_cast<const T *>(in);
        T *to = static_cast<T *>(out);
        if (indices) {
            if (op == OP_MAX)
                return launch_axis_typed<T, OP_MAX, true, false>(dev, stream, ti, p, to, indices, idx_base, idx_o);
            if (op == OP_MIN)
                return launch_axis_typed<T, OP_MIN, true, false>(dev, stream, ti, p, to, indices, idx_base, idx_o);
            return fail(HEPH_INVALID_CONFIGURATION, "arg-reduction supports min and max");
        }
        switch (op) {
            case OP_SUM: return launch_mean<T, OP_SUM, false>(dev, stream, ti, p, to, mean, nullptr, 0, 0);
            case OP_PROD: return launch_axis_typed<T, OP_PROD, false, false>(dev, stream, ti, p, to, nullptr, 0, 0);
            case OP_MIN: return launch_axis_typed<T, OP_MIN, false, false>(dev, stream, ti, p, to, nullptr, 0, 0);
            case OP_MAX: return launch_axis_typed<T, OP_MAX, false, false>(dev, stream, ti, p, to, nullptr, 0, 0);
        }
        return fail(HEPH_INVALID_CONFIGURATION, "unknown axis reduction operator");
    });
}

}  // namespace heph
