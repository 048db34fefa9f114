// reduce_full.cu — single-kernel full reductions for sm_100a.
//
// Replaces the reference's multi-pass tree (hephaestus-cuda
// application/reduction.rs:19-64 + prepared_reduction.rs:38-128, one launch
// per 256-way level, a strided staging copy before it and a D2H/H2D scalar
// round trip after it, full_reduction_seam.rs:96-114) with ONE launch:
//   * dense views: grid-stride over 128-bit streaming loads, 4 vectors in
//     flight per thread, grid = resident CTAs of all SMs;
//   * warp fold with redux.sync (32-bit integer add/min/max) or xor-shuffles,
//     then a shared-memory fold of the warp results;
//   * per-CTA partial to the stream's workspace, atomic ticket, and the last
//     CTA folds the partials in CTA order and writes the scalar in place.
// Other views (sub-blocks with gaps, diagonals, broadcasts, negative strides;
// rank <= 4) are canonicalised on the host (unit dims dropped, negative
// strides flipped, dims ordered by stride and merged) and walked by a kernel
// that steps each thread's coordinates by the grid stride in the view's mixed
// radix — no division per element, coalesced along a unit-stride inner dim,
// 128-bit loads when the inner runs are 16-byte aligned.  The reference copies
// such a view into a contiguous staging buffer first
// (full_reduction_seam.rs:96-104).
#include <algorithm>
#include <cstdio>
#include <utility>
#include <cstdlib>

#include "device_utils.cuh"
#include "kernels.h"
#include "view_walk.cuh"

namespace heph {

constexpr int kReduceThreads = 256;
constexpr int kReduceUnroll = 4;
// Unaligned unit-stride runs at least this long take the row-run kernel.
constexpr uint64_t kMinRunLength = 128;

template <typename Tin, typename Tacc, int OP>
__device__ __forceinline__ Tacc fold_vec(Tacc acc, uint4 raw) {
    Vec16<Tin> v = as_elems<Tin>(raw);
#pragma unroll
    for (int c = 0; c < Vec16<Tin>::V; ++c) acc = combine<Tacc, OP>(acc, (Tacc)v.e[c]);
    return acc;
}

// Folds the block's value into the output of a slice of `nblocks` CTAs (this
// one is `block` of them): per-CTA partial, ticket, and the slice's last CTA
// folds the slice's partials in CTA order and writes the output in place.
template <typename Tacc, int OP>
__device__ __forceinline__ void finish_slice(Tacc acc, Tacc *out, Tacc *partials, unsigned int *ticket,
                                             unsigned int block, unsigned int nblocks, Tacc *scratch) {
    acc = block_fold<Tacc, OP, kReduceThreads>(acc, scratch);
    if (nblocks == 1) {
        if (threadIdx.x == 0) *out = acc;
        return;
    }
    __shared__ bool am_last;
    if (threadIdx.x == 0) {
        partials[block] = acc;
        // One acquire-release ticket increment: it publishes this CTA's
        // partial (release) and, for the last CTA, makes every other CTA's
        // partial visible to it (acquire); the barrier below carries that to
        // the CTA's other threads.
        unsigned int t;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(t) : "l"(ticket) : "memory");
        am_last = (t == nblocks - 1);
    }
    __syncthreads();
    if (!am_last) return;
    Tacc a = identity<Tacc, OP>();
    for (unsigned int j = threadIdx.x; j < nblocks; j += kReduceThreads)
        a = combine<Tacc, OP>(a, ld_cg(partials + j));
    a = block_fold<Tacc, OP, kReduceThreads>(a, scratch);
    if (threadIdx.x == 0) {
        *out = a;
        *ticket = 0u;  // leave the ticket at rest for the next launch
    }
}

template <typename Tacc, int OP>
__device__ __forceinline__ void finish_grid(Tacc acc, Tacc *out, Tacc *partials,
                                            unsigned int *ticket, Tacc *scratch) {
    finish_slice<Tacc, OP>(acc, out, partials, ticket, blockIdx.x, gridDim.x, scratch);
}

// This thread's fold of a dense run of n elements read by a slice of
// `nblocks` CTAs (this one is `block`): 128-bit streaming loads, 4 in flight,
// scalar head and tail around the 16-byte-aligned middle.
template <typename Tin, typename Tacc, int OP, int THREADS = kReduceThreads, int UNROLL = kReduceUnroll>
__device__ __forceinline__ Tacc dense_fold(const Tin *__restrict__ in, uint64_t n, unsigned int block,
                                           unsigned int nblocks) {
    constexpr int V = Vec16<Tin>::V;
    const uint64_t tid = (uint64_t)block * THREADS + threadIdx.x;
    const uint64_t stride = (uint64_t)nblocks * THREADS;

    // Elements before the first 16-byte boundary and after the last one.
    const uintptr_t addr = reinterpret_cast<uintptr_t>(in);
    uint64_t head = ((16u - (addr & 15u)) & 15u) / sizeof(Tin);
    if (head > n) head = n;
    const uint64_t nvec = (n - head) / V;
    const uint64_t tail = head + nvec * V;
    const uint4 *vin = reinterpret_cast<const uint4 *>(in + head);

    Tacc acc = identity<Tacc, OP>();
    uint64_t i = tid;
    for (; i + (UNROLL - 1) * stride < nvec; i += UNROLL * stride) {
        uint4 r[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) r[u] = ld_stream(vin + i + u * stride);
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) acc = fold_vec<Tin, Tacc, OP>(acc, r[u]);
    }
    for (; i < nvec; i += stride) acc = fold_vec<Tin, Tacc, OP>(acc, ld_stream(vin + i));
    if (tid < head) acc = combine<Tacc, OP>(acc, (Tacc)in[tid]);
    if (tid < n - tail) acc = combine<Tacc, OP>(acc, (Tacc)in[tail + tid]);
    return acc;
}

template <typename Tin, typename Tacc, int OP>
__global__ void __launch_bounds__(kReduceThreads)
    reduce_dense_kernel(const Tin *__restrict__ in, uint64_t n, Tacc *__restrict__ out,
                        Tacc *__restrict__ partials, unsigned int *__restrict__ ticket) {
    __shared__ Tacc scratch[kReduceThreads / 32];
    // Programmatic dependent launch: the next kernel of the stream may be
    // scheduled now; this one waits for its predecessor's results before it
    // touches memory (a no-op when launched without the attribute).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const Tacc acc = dense_fold<Tin, Tacc, OP>(in, n, blockIdx.x, gridDim.x);
    finish_grid<Tacc, OP>(acc, out, partials, ticket, scratch);
}

// Large dense reductions staged through shared memory by bulk copies (TMA,
// no multicast): each CTA keeps kBulkStages copies of 16 KiB in flight, so
// the bytes in flight per SM are set by shared memory, not by registers;
// CTA b folds 16 KiB blocks b, b + G, b + 2G, ...  The unaligned head and the
// ragged tail are folded with plain loads by the whole grid.
constexpr int kBulkStages = 6;
constexpr uint32_t kBulkBlockBytes = 16384;
constexpr int kBulkCtasPerSm = 2;
constexpr uint64_t kBulkMinBytes = 256ull << 20;

// This CTA's share of a dense run through the shared-memory stages: calls
// fv(uint4) for every 16-byte vector of its 16 KiB blocks and fo(Tin) for
// its elements of the head and the tail.
template <typename Tin, typename FV, typename FO>
__device__ __forceinline__ void bulk_stream(const Tin *__restrict__ in, uint64_t n, unsigned int *err,
                                            unsigned char *stage, uint64_t *bar, FV &&fv, FO &&fo) {
    constexpr uint64_t BE = kBulkBlockBytes / sizeof(Tin);
    const uintptr_t addr = reinterpret_cast<uintptr_t>(in);
    uint64_t head = ((16u - (addr & 15u)) & 15u) / sizeof(Tin);
    if (head > n) head = n;
    const uint64_t nblocks = (n - head) / BE;
    const Tin *body = in + head;
    const uint64_t tail0 = head + nblocks * BE;
    const uint64_t G = gridDim.x, b = blockIdx.x;
    const uint64_t mine = nblocks > b ? (nblocks - b + G - 1) / G : 0;
    if (threadIdx.x == 0) {
        for (int k = 0; k < kBulkStages; ++k) mbar_init(&bar[k], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (uint64_t k = 0; k < (uint64_t)kBulkStages && k < mine; ++k)
            bulk_load(stage + k * kBulkBlockBytes, body + (b + k * G) * BE, kBulkBlockBytes, &bar[k]);
    }
    __syncthreads();
    constexpr int U = kBulkBlockBytes / 16 / kReduceThreads;  // 16-byte vectors per thread per block
    for (uint64_t i = 0; i < mine; ++i) {
        const int k = (int)(i % kBulkStages);
        mbar_wait(&bar[k], (uint32_t)((i / kBulkStages) & 1u), err);
        const uint4 *src = reinterpret_cast<const uint4 *>(stage + k * kBulkBlockBytes);
        uint4 r[U];
#pragma unroll
        for (int u = 0; u < U; ++u) r[u] = src[threadIdx.x + u * kReduceThreads];
        __syncthreads();  // every thread has read stage k: refill it
        if (threadIdx.x == 0 && i + kBulkStages < mine) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            bulk_load(stage + k * kBulkBlockBytes, body + (b + (i + kBulkStages) * G) * BE, kBulkBlockBytes, &bar[k]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) fv(r[u]);
    }
    const uint64_t tid = b * kReduceThreads + threadIdx.x;
    if (tid < head) fo(in[tid]);
    for (uint64_t e = tail0 + tid; e < n; e += G * kReduceThreads) fo(in[e]);
}

// Dense runs of kBulkMinBytes and more stream through the shared-memory
// stages (i32 -> i64 sum of 2^32 elements: 6736 -> 7176 GB/s; 1 GiB of f32 the
// same either way; a 64 MiB f32 sum, partly in L2, slower: 6958 -> 6072).
// HEPH_REDUCE_BULK_MIN (bytes, read once) moves the threshold; 0 turns the
// bulk kernels off.
static bool use_bulk(uint64_t bytes) {
    static const uint64_t bulk_min = [] {
        const char *e = getenv("HEPH_REDUCE_BULK_MIN");
        return e ? strtoull(e, nullptr, 10) : kBulkMinBytes;
    }();
    return bulk_min && bytes >= bulk_min;
}

// Raises a kernel's dynamic shared-memory limit to the bulk stages, once per
// (kernel, device ordinal); the caller holds the device's lock.
template <typename K> static heph_status bulk_attr(K kernel, int ordinal) {
    static bool set[64] = {};
    if (ordinal >= 0 && ordinal < 64 && set[ordinal]) return HEPH_OK;
    HEPH_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)(kBulkStages * kBulkBlockBytes)),
                  HEPH_DISPATCH_FAILED, "bulk reduction attribute");
    if (ordinal >= 0 && ordinal < 64) set[ordinal] = true;
    return HEPH_OK;
}

template <typename Tin, typename Tacc, int OP>
__global__ void __launch_bounds__(kReduceThreads, kBulkCtasPerSm)
    reduce_bulk_kernel(const Tin *__restrict__ in, uint64_t n, Tacc *__restrict__ out, Tacc *__restrict__ partials,
                       unsigned int *__restrict__ ticket, unsigned int *err) {
    extern __shared__ __align__(128) unsigned char stage[];  // kBulkStages x 16 KiB
    __shared__ uint64_t bar[kBulkStages];
    __shared__ Tacc scratch[kReduceThreads / 32];
    Tacc acc = identity<Tacc, OP>();
    bulk_stream<Tin>(
        in, n, err, stage, bar, [&](uint4 v) { acc = fold_vec<Tin, Tacc, OP>(acc, v); },
        [&](Tin v) { acc = combine<Tacc, OP>(acc, (Tacc)v); });
    finish_grid<Tacc, OP>(acc, out, partials, ticket, scratch);
}

// A fused batch of dense full reductions in one launch: problem p owns CTAs
// [cta_begin, cta_begin + ctas) of the grid, its own partial slots (indexed
// like its CTAs) and ticket.  A CTA finds its problem with one parallel read
// of the table (each thread checks one entry), so its first data load waits
// for a single table load instead of a chain of dependent ones.
template <typename Tin, typename Tacc, int OP>
__global__ void __launch_bounds__(kReduceThreads)
    reduce_fused_kernel(const FusedFull *__restrict__ table, uint32_t nprob, Tacc *__restrict__ partials,
                        unsigned int *__restrict__ tickets) {
    __shared__ Tacc scratch[kReduceThreads / 32];
    __shared__ FusedFull s_f;
    __shared__ uint32_t s_prob;
    for (uint32_t q0 = 0; q0 < nprob; q0 += kReduceThreads) {
        const uint32_t q = q0 + threadIdx.x;
        if (q < nprob) {
            const FusedFull e = table[q];
            if (e.cta_begin <= blockIdx.x && blockIdx.x - e.cta_begin < e.ctas) {
                s_f = e;
                s_prob = q;
            }
        }
    }
    __syncthreads();
    const uint32_t p = s_prob;
    const FusedFull f = s_f;
    const unsigned int block = blockIdx.x - f.cta_begin;
    const Tacc acc = dense_fold<Tin, Tacc, OP>(static_cast<const Tin *>(f.in), f.n, block, f.ctas);
    finish_slice<Tacc, OP>(acc, static_cast<Tacc *>(f.out), partials + f.cta_begin, tickets + p, block, f.ctas,
                           scratch);
}

struct StridedView4 {
    uint32_t rank;
    uint64_t shape[HEPH_MAX_RANK];
    int64_t strides[HEPH_MAX_RANK];
    int64_t offset;
};

template <typename Tin, typename Tacc, int OP>
__global__ void __launch_bounds__(kReduceThreads)
    reduce_strided_kernel(const Tin *__restrict__ base, StridedView4 v, uint64_t n,
                          Tacc *__restrict__ out, Tacc *__restrict__ partials,
                          unsigned int *__restrict__ ticket) {
    __shared__ Tacc scratch[kReduceThreads / 32];
    Tacc acc = identity<Tacc, OP>();
    const uint64_t stride = (uint64_t)gridDim.x * kReduceThreads;
    for (uint64_t i = (uint64_t)blockIdx.x * kReduceThreads + threadIdx.x; i < n; i += stride) {
        uint64_t rem = i;
        int64_t off = v.offset;
        for (int d = (int)v.rank - 1; d >= 0; --d) {
            uint64_t c = rem % v.shape[d];
            rem /= v.shape[d];
            off += (int64_t)c * v.strides[d];
        }
        acc = combine<Tacc, OP>(acc, (Tacc)base[off]);
    }
    finish_grid<Tacc, OP>(acc, out, partials, ticket, scratch);
}

// Canonical strided view, walked without division (view_walk.cuh).  `n`
// counts walk units: elements, or 16-byte vectors when VEC.
template <typename Tin, typename Tacc, int OP, int R, bool VEC>
__global__ void __launch_bounds__(kReduceThreads)
    reduce_walk_kernel(const Tin *__restrict__ base, const ViewWalk<1> w, uint64_t n, Tacc *__restrict__ out,
                       Tacc *__restrict__ partials, unsigned int *__restrict__ ticket) {
    __shared__ Tacc scratch[kReduceThreads / 32];
    const uint64_t stride = (uint64_t)gridDim.x * kReduceThreads;
    uint64_t i = (uint64_t)blockIdx.x * kReduceThreads + threadIdx.x;
    Tacc acc = identity<Tacc, OP>();
    ViewCursor<R, 1> cur;
    if (i < n) cur.seek(w, i);
    auto fold_at = [&](int64_t o) {
        if constexpr (VEC) acc = fold_vec<Tin, Tacc, OP>(acc, ld_stream(reinterpret_cast<const uint4 *>(base) + o));
        else acc = combine<Tacc, OP>(acc, (Tacc)__ldg(base + o));
    };
    for (; i + (kReduceUnroll - 1) * stride < n; i += kReduceUnroll * stride) {
        if constexpr (VEC) {
            uint4 r[kReduceUnroll];
#pragma unroll
            for (int u = 0; u < kReduceUnroll; ++u) {
                r[u] = ld_stream(reinterpret_cast<const uint4 *>(base) + cur.off[0]);
                cur.advance(w);
            }
#pragma unroll
            for (int u = 0; u < kReduceUnroll; ++u) acc = fold_vec<Tin, Tacc, OP>(acc, r[u]);
        } else {
            Tin r[kReduceUnroll];
#pragma unroll
            for (int u = 0; u < kReduceUnroll; ++u) {
                r[u] = __ldg(base + cur.off[0]);
                cur.advance(w);
            }
#pragma unroll
            for (int u = 0; u < kReduceUnroll; ++u) acc = combine<Tacc, OP>(acc, (Tacc)r[u]);
        }
    }
    for (; i < n; i += stride) {
        fold_at(cur.off[0]);
        cur.advance(w);
    }
    finish_grid<Tacc, OP>(acc, out, partials, ticket, scratch);
}

// Unit-stride runs that are not 16-byte aligned: warp per (run, segment),
// scalar head/tail, 128-bit middle (view_walk.cuh RunWalk).
template <typename Tin, typename Tacc, int OP>
__global__ void __launch_bounds__(kReduceThreads)
    reduce_runs_kernel(const Tin *__restrict__ base, const RunWalk w, Tacc *__restrict__ out,
                       Tacc *__restrict__ partials, unsigned int *__restrict__ ticket) {
    __shared__ Tacc scratch[kReduceThreads / 32];
    Tacc acc = identity<Tacc, OP>();
    run_walk_fold<Tin, 2 * kReduceUnroll>(base, w, acc, [](Tacc &a, Tin x) { a = combine<Tacc, OP>(a, (Tacc)x); });
    finish_grid<Tacc, OP>(acc, out, partials, ticket, scratch);
}

template <typename Tacc, int OP> __global__ void write_identity_kernel(Tacc *out) {
    *out = identity<Tacc, OP>();
}

// ------------------------------------------------------------------ launch

// Launches reduce_walk_kernel for a non-dense view; false (nothing launched)
// when an inner dim of the canonical view exceeds 32-bit coordinates.
template <typename Tin, typename Tacc, int OP>
static bool launch_walk(cudaStream_t stream, const Tin *base, const heph_layout &l, uint64_t count, unsigned grid,
                        Tacc *out, Tacc *partials, unsigned int *tickets) {
    StreamView sv;
    const heph_layout *ls[1] = {&l};
    stream_view(ls, 1, &sv);
    constexpr uint32_t V = 16 / sizeof(Tin);
    const void *bases[1] = {base};
    const bool vec = sv.rank >= 2 && stream_view_vectorize(&sv, 1, V, bases, sizeof(Tin));
    RunWalk runs;
    if (!vec && make_run_walk(sv, sizeof(Tin), kMinRunLength, &runs)) {
        reduce_runs_kernel<Tin, Tacc, OP><<<grid, kReduceThreads, 0, stream>>>(base, runs, out, partials, tickets);
        return true;
    }
    const uint64_t units = vec ? count / V : count;
    const int R = sv.rank == 1 ? 1 : sv.rank == 2 ? 2 : 4;
    ViewWalk<1> w;
    if (!make_walk<1>(sv, R, (uint64_t)grid * kReduceThreads, &w)) return false;
    const dim3 g(grid), b(kReduceThreads);
    if (vec) {
        if (R == 2) reduce_walk_kernel<Tin, Tacc, OP, 2, true><<<g, b, 0, stream>>>(base, w, units, out, partials, tickets);
        else reduce_walk_kernel<Tin, Tacc, OP, 4, true><<<g, b, 0, stream>>>(base, w, units, out, partials, tickets);
    } else {
        if (R == 1) reduce_walk_kernel<Tin, Tacc, OP, 1, false><<<g, b, 0, stream>>>(base, w, units, out, partials, tickets);
        else if (R == 2) reduce_walk_kernel<Tin, Tacc, OP, 2, false><<<g, b, 0, stream>>>(base, w, units, out, partials, tickets);
        else reduce_walk_kernel<Tin, Tacc, OP, 4, false><<<g, b, 0, stream>>>(base, w, units, out, partials, tickets);
    }
    return true;
}

template <typename Tin, typename Tacc, int OP>
static heph_status launch_typed(Device *dev, cudaStream_t stream, const void *base_v,
                                const heph_layout &l, uint64_t count, void *out_v) {
    const Tin *base = static_cast<const Tin *>(base_v);
    Tacc *out = static_cast<Tacc *>(out_v);
    if (count == 0) {
        write_identity_kernel<Tacc, OP><<<1, 1, 0, stream>>>(out);
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "full reduction launch");
        return HEPH_OK;
    }
    const bool dense = layout_is_dense(l);
    // Work per CTA: at least kReduceUnroll vectors per thread before adding CTAs.
    const uint64_t per_cta = (uint64_t)kReduceThreads * kReduceUnroll * (16 / sizeof(Tin));
    uint64_t want = (count + per_cta - 1) / per_cta;
    const uint64_t cap = (uint64_t)dev->sm_count * (2048 / kReduceThreads);
    unsigned int grid = (unsigned int)std::max<uint64_t>(1, std::min(want, cap));
    // Experiment knob (read once per process): a fixed grid for dense views.
    static const int grid_knob = [] {
        const char *e = getenv("HEPH_REDUCE_GRID");
        return e ? atoi(e) : 0;
    }();
    if (grid_knob > 0) grid = (unsigned int)std::min<uint64_t>((uint64_t)grid_knob, cap);

    std::lock_guard<std::mutex> lock(dev->mu);
    Workspace *ws = nullptr;
    heph_status st = workspace_for(dev, stream, (size_t)grid * sizeof(Tacc), 0, &ws);
    if (st != HEPH_OK) return st;
    Tacc *partials = static_cast<Tacc *>(ws->partials);
    int64_t first = 0;
    if (dense || layout_covers_dense_block(l, &first)) {
        // Dense, or a permutation / reversal of a dense block: the fold is
        // order-insensitive, so the block streams contiguously.
        // Launched as a programmatic dependent of the stream's previous
        // kernel: its CTAs are scheduled while that kernel drains and wait
        // for its results in griddepcontrol.wait, which hides most of the
        // launch latency of back-to-back small reductions (2^20 f32 per call
        // 6.2 -> 4.4 us measured).  HEPH_REDUCE_PDL=0 turns it off.
        if (use_bulk(count * sizeof(Tin))) {
            auto kernel = reduce_bulk_kernel<Tin, Tacc, OP>;
            const size_t smem = (size_t)kBulkStages * kBulkBlockBytes;
            st = bulk_attr(kernel, dev->ordinal);
            if (st != HEPH_OK) return st;
            const unsigned bg = (unsigned)std::min<uint64_t>((uint64_t)dev->sm_count * kBulkCtasPerSm, (uint64_t)grid);
            kernel<<<bg, kReduceThreads, smem, stream>>>(base + (dense ? (int64_t)l.offset : first), count, out, partials,
                                                        ws->tickets, dev->error_dev);
            HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "full reduction launch");
            return HEPH_OK;
        }
        static const bool pdl = [] {
            const char *e = getenv("HEPH_REDUCE_PDL");
            return !e || atoi(e) != 0;
        }();
        const Tin *src = base + (dense ? (int64_t)l.offset : first);
        if (pdl) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(grid);
            cfg.blockDim = dim3(kReduceThreads);
            cfg.stream = stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            HEPH_CUDA_TRY(cudaLaunchKernelEx(&cfg, reduce_dense_kernel<Tin, Tacc, OP>, src, count, out, partials,
                                             ws->tickets),
                          HEPH_DISPATCH_FAILED, "full reduction launch");
        } else {
            reduce_dense_kernel<Tin, Tacc, OP><<<grid, kReduceThreads, 0, stream>>>(src, count, out, partials,
                                                                                    ws->tickets);
        }
    } else if (!launch_walk<Tin, Tacc, OP>(stream, base, l, count, grid, out, partials, ws->tickets)) {
        StridedView4 v{};
        v.rank = l.rank;
        for (uint32_t d = 0; d < l.rank; ++d) {
            v.shape[d] = l.shape[d];
            v.strides[d] = l.strides[d];
        }
        v.offset = (int64_t)l.offset;
        reduce_strided_kernel<Tin, Tacc, OP>
            <<<grid, kReduceThreads, 0, stream>>>(base, v, count, out, partials, ws->tickets);
    }
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "full reduction launch");
    return HEPH_OK;
}

template <typename Tin, typename Tacc>
static heph_status launch_op(Device *dev, cudaStream_t stream, int op, const void *base,
                             const heph_layout &l, uint64_t count, void *out) {
    switch (op) {
        case OP_SUM: return launch_typed<Tin, Tacc, OP_SUM>(dev, stream, base, l, count, out);
        case OP_PROD: return launch_typed<Tin, Tacc, OP_PROD>(dev, stream, base, l, count, out);
        case OP_MIN: return launch_typed<Tin, Tacc, OP_MIN>(dev, stream, base, l, count, out);
        case OP_MAX: return launch_typed<Tin, Tacc, OP_MAX>(dev, stream, base, l, count, out);
    }
    return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
}

heph_status launch_reduce_full(Device *dev, cudaStream_t stream, int op, heph_dtype in_dtype,
                               heph_dtype acc_dtype, const void *base, const heph_layout &l,
                               uint64_t count, void *out) {
    if (in_dtype == acc_dtype) {
        return dispatch_dtype(in_dtype, [&]<typename T>() {
            return launch_op<T, T>(dev, stream, op, base, l, count, out);
        });
    }
    if (in_dtype == HEPH_I32 && acc_dtype == HEPH_I64)
        return launch_op<int32_t, int64_t>(dev, stream, op, base, l, count, out);
    if (in_dtype == HEPH_F32 && acc_dtype == HEPH_F64)
        return launch_op<float, double>(dev, stream, op, base, l, count, out);
    return fail(HEPH_INVALID_CONFIGURATION,
                "full reduction output type must match the input type or widen it (i32->i64, "
                "f32->f64)");
}

// Two reductions of one dense run in one read: op1 in T (e.g. the total a
// partitioned scan needs for its carry) and op2 in Tacc (e.g. a widening sum
// of the same slice).  Per-CTA partials of both, last-CTA finalize of both.
template <typename Tin, int OP1, typename Tacc, int OP2, bool BULK>
__global__ void __launch_bounds__(kReduceThreads)
    reduce_dual_kernel(const Tin *__restrict__ in, uint64_t n, Tin *__restrict__ out1, Tacc *__restrict__ out2,
                       Tin *__restrict__ partials1, Tacc *__restrict__ partials2, unsigned int *__restrict__ ticket,
                       unsigned int *err) {
    __shared__ Tin scratch1[kReduceThreads / 32];
    __shared__ Tacc scratch2[kReduceThreads / 32];
    constexpr int V = Vec16<Tin>::V;
    const uint64_t tid = (uint64_t)blockIdx.x * kReduceThreads + threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * kReduceThreads;
    const uintptr_t addr = reinterpret_cast<uintptr_t>(in);
    uint64_t head = ((16u - (addr & 15u)) & 15u) / sizeof(Tin);
    if (head > n) head = n;
    const uint64_t nvec = (n - head) / V;
    const uint64_t tail = head + nvec * V;
    const uint4 *vin = reinterpret_cast<const uint4 *>(in + head);
    Tin a1 = identity<Tin, OP1>();
    Tacc a2 = identity<Tacc, OP2>();
    auto fold = [&](uint4 raw) {
        Vec16<Tin> e = as_elems<Tin>(raw);
#pragma unroll
        for (int c = 0; c < V; ++c) {
            a1 = combine<Tin, OP1>(a1, e.e[c]);
            a2 = combine<Tacc, OP2>(a2, (Tacc)e.e[c]);
        }
    };
    auto fold_one = [&](Tin v) {
        a1 = combine<Tin, OP1>(a1, v);
        a2 = combine<Tacc, OP2>(a2, (Tacc)v);
    };
    if constexpr (BULK) {
        extern __shared__ __align__(128) unsigned char stage[];  // kBulkStages x 16 KiB
        __shared__ uint64_t bar[kBulkStages];
        bulk_stream<Tin>(in, n, err, stage, bar, fold, fold_one);
    } else {
        (void)err;
        uint64_t i = tid;
        for (; i + (kReduceUnroll - 1) * stride < nvec; i += kReduceUnroll * stride) {
            uint4 r[kReduceUnroll];
#pragma unroll
            for (int u = 0; u < kReduceUnroll; ++u) r[u] = ld_stream(vin + i + u * stride);
#pragma unroll
            for (int u = 0; u < kReduceUnroll; ++u) fold(r[u]);
        }
        for (; i < nvec; i += stride) fold(ld_stream(vin + i));
        if (tid < head) fold_one(in[tid]);
        if (tid < n - tail) fold_one(in[tail + tid]);
    }

    a1 = block_fold<Tin, OP1, kReduceThreads>(a1, scratch1);
    a2 = block_fold<Tacc, OP2, kReduceThreads>(a2, scratch2);
    if (gridDim.x == 1) {
        if (threadIdx.x == 0) {
            *out1 = a1;
            *out2 = a2;
        }
        return;
    }
    __shared__ bool am_last;
    if (threadIdx.x == 0) {
        partials1[blockIdx.x] = a1;
        partials2[blockIdx.x] = a2;
        __threadfence();
        am_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!am_last) return;
    __threadfence();
    Tin b1 = identity<Tin, OP1>();
    Tacc b2 = identity<Tacc, OP2>();
    for (unsigned int j = threadIdx.x; j < gridDim.x; j += kReduceThreads) {
        b1 = combine<Tin, OP1>(b1, ld_cg(partials1 + j));
        b2 = combine<Tacc, OP2>(b2, ld_cg(partials2 + j));
    }
    b1 = block_fold<Tin, OP1, kReduceThreads>(b1, scratch1);
    b2 = block_fold<Tacc, OP2, kReduceThreads>(b2, scratch2);
    if (threadIdx.x == 0) {
        *out1 = b1;
        *out2 = b2;
        *ticket = 0u;
    }
}

template <typename Tin, int OP1, typename Tacc>
static heph_status launch_dual_typed(Device *dev, cudaStream_t stream, int op2, const Tin *in, uint64_t n,
                                     void *out1, void *out2) {
    const uint64_t per_cta = (uint64_t)kReduceThreads * kReduceUnroll * (16 / sizeof(Tin));
    const uint64_t cap = (uint64_t)dev->sm_count * (2048 / kReduceThreads);
    const unsigned grid = (unsigned)std::max<uint64_t>(1, std::min((n + per_cta - 1) / per_cta, cap));
    std::lock_guard<std::mutex> lock(dev->mu);
    Workspace *ws = nullptr;
    heph_status st = workspace_for(dev, stream, (size_t)grid * (sizeof(Tin) + sizeof(Tacc)) + 16, 0, &ws);
    if (st != HEPH_OK) return st;
    Tacc *p2 = static_cast<Tacc *>(ws->partials);
    Tin *p1 = reinterpret_cast<Tin *>(static_cast<char *>(ws->partials) + (size_t)grid * sizeof(Tacc));
    Tin *o1 = static_cast<Tin *>(out1);
    Tacc *o2 = static_cast<Tacc *>(out2);
    auto go = [&]<int OP2>() -> heph_status {
        if (use_bulk(n * sizeof(Tin))) {
            auto kernel = reduce_dual_kernel<Tin, OP1, Tacc, OP2, true>;
            heph_status s2 = bulk_attr(kernel, dev->ordinal);
            if (s2 != HEPH_OK) return s2;
            const unsigned bg = (unsigned)std::min<uint64_t>((uint64_t)dev->sm_count * kBulkCtasPerSm, grid);
            kernel<<<bg, kReduceThreads, (size_t)kBulkStages * kBulkBlockBytes, stream>>>(in, n, o1, o2, p1, p2,
                                                                                          ws->tickets, dev->error_dev);
        } else {
            reduce_dual_kernel<Tin, OP1, Tacc, OP2, false><<<grid, kReduceThreads, 0, stream>>>(in, n, o1, o2, p1, p2,
                                                                                               ws->tickets, nullptr);
        }
        return HEPH_OK;
    };
    switch (op2) {
        case OP_SUM: st = go.template operator()<OP_SUM>(); break;
        case OP_PROD: st = go.template operator()<OP_PROD>(); break;
        case OP_MIN: st = go.template operator()<OP_MIN>(); break;
        case OP_MAX: st = go.template operator()<OP_MAX>(); break;
        default: return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
    }
    if (st != HEPH_OK) return st;
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "dual reduction launch");
    return HEPH_OK;
}

heph_status launch_reduce_dual(Device *dev, cudaStream_t stream, int op1, int op2, heph_dtype dtype,
                               heph_dtype acc2_dtype, const void *in, uint64_t n, void *out1, void *out2) {
    auto by_op1 = [&]<typename Tin, typename Tacc>() -> heph_status {
        const Tin *ti = static_cast<const Tin *>(in);
        if (op1 == OP_SUM) return launch_dual_typed<Tin, OP_SUM, Tacc>(dev, stream, op2, ti, n, out1, out2);
        if (op1 == OP_PROD) return launch_dual_typed<Tin, OP_PROD, Tacc>(dev, stream, op2, ti, n, out1, out2);
        return fail(HEPH_INVALID_CONFIGURATION, "scans support the sum (cumsum) and product (cumprod) operators");
    };
    if (dtype == acc2_dtype)
        return dispatch_dtype(dtype, [&]<typename T>() { return by_op1.template operator()<T, T>(); });
    if (dtype == HEPH_I32 && acc2_dtype == HEPH_I64) return by_op1.template operator()<int32_t, int64_t>();
    if (dtype == HEPH_F32 && acc2_dtype == HEPH_F64) return by_op1.template operator()<float, double>();
    return fail(HEPH_DISPATCH_FAILED,
                "full reduction output element type must match the input or widen it (i32->i64, f32->f64)");
}

uint32_t plan_reduce_full_fused(const Device *dev, heph_dtype in_dtype, FusedFull *table, uint32_t nprob) {
    const uint64_t per_cta = (uint64_t)kReduceThreads * kReduceUnroll * (16 / dtype_size(in_dtype));
    const uint64_t cap = (uint64_t)dev->sm_count * (2048 / kReduceThreads);
    uint64_t want_total = 0, n_total = 0;
    for (uint32_t p = 0; p < nprob; ++p) {
        want_total += std::max<uint64_t>(1, (table[p].n + per_cta - 1) / per_cta);
        n_total += table[p].n;
    }
    uint32_t next = 0;
    for (uint32_t p = 0; p < nprob; ++p) {
        const uint64_t want = std::max<uint64_t>(1, (table[p].n + per_cta - 1) / per_cta);
        // Within the resident-CTA budget every problem gets its own grid's
        // worth; beyond it, CTAs in proportion to the elements.
        const uint64_t c = want_total <= cap ? want
                                             : std::max<uint64_t>(1, std::min(want, cap * table[p].n / std::max<uint64_t>(1, n_total)));
        table[p].cta_begin = next;
        table[p].ctas = (uint32_t)c;
        next += (uint32_t)c;
    }
    return next;
}

heph_status launch_reduce_full_fused(cudaStream_t stream, int op, heph_dtype in_dtype, heph_dtype acc_dtype,
                                     const FusedFull *table, uint32_t nprob, uint32_t grid, void *partials,
                                     unsigned int *tickets) {
    auto go = [&]<typename Tin, typename Tacc>() -> heph_status {
        Tacc *pp = static_cast<Tacc *>(partials);
        switch (op) {
            case OP_SUM: reduce_fused_kernel<Tin, Tacc, OP_SUM><<<grid, kReduceThreads, 0, stream>>>(table, nprob, pp, tickets); break;
            case OP_PROD: reduce_fused_kernel<Tin, Tacc, OP_PROD><<<grid, kReduceThreads, 0, stream>>>(table, nprob, pp, tickets); break;
            case OP_MIN: reduce_fused_kernel<Tin, Tacc, OP_MIN><<<grid, kReduceThreads, 0, stream>>>(table, nprob, pp, tickets); break;
            case OP_MAX: reduce_fused_kernel<Tin, Tacc, OP_MAX><<<grid, kReduceThreads, 0, stream>>>(table, nprob, pp, tickets); break;
            default: return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
        }
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "fused full reduction launch");
        return HEPH_OK;
    };
    if (in_dtype == acc_dtype)
        return dispatch_dtype(in_dtype, [&]<typename T>() { return go.template operator()<T, T>(); });
    if (in_dtype == HEPH_I32 && acc_dtype == HEPH_I64) return go.template operator()<int32_t, int64_t>();
    if (in_dtype == HEPH_F32 && acc_dtype == HEPH_F64) return go.template operator()<float, double>();
    return fail(HEPH_INVALID_CONFIGURATION, "full reduction output type must match the input type or widen it");
}

}  // namespace heph

// ------------------------------------------- allocation-free full reduction
//
// For callers that cannot allocate device memory at call time — an embedder
// that runs inside a fixed memory budget or hands this library only the
// buffers it owns, or code whose allocator must not be re-entered from the
// call site.  The scratch the reduction needs (one partial per CTA plus the
// last-CTA ticket) lives in this file-scope array, which every GPU that loads
// the library holds for the life of the process.

namespace heph {
namespace {

constexpr int kStaticPartials = 2048;  // CTA partials (8 bytes each) the array holds
// [0, 16 KiB): partials of up to kStaticPartials CTAs; then the ticket.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticPartials * 8 + 256];

// Device address of g_static_scratch in the CURRENT context.  A symbol's
// address belongs to a context's load of this module, not to a device
// ordinal (a driver-API embedder may run on a non-primary context, and
// cudaDeviceReset unloads the module), so it is looked up on every call; the
// lookup allocates nothing.  The first call in a context loads the module
// there, so that first call should come before any stream capture.
heph_status static_scratch_address(void **out) {
    void *p = nullptr;
    HEPH_CUDA_TRY(cudaGetSymbolAddress(&p, g_static_scratch), HEPH_DEVICE_UNAVAILABLE,
                  "static scratch address lookup");
    *out = p;
    return HEPH_OK;
}

template <typename Tin, typename Tacc, int OP>
heph_status launch_static_typed(const void *in_v, uint64_t count, void *out_v, cudaStream_t stream, int sm_count) {
    const Tin *in = static_cast<const Tin *>(in_v);
    Tacc *out = static_cast<Tacc *>(out_v);
    if (count == 0) {
        write_identity_kernel<Tacc, OP><<<1, 1, 0, stream>>>(out);
        HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "full reduction launch");
        return HEPH_OK;
    }
    const uint64_t per_cta = (uint64_t)kReduceThreads * kReduceUnroll * (16 / sizeof(Tin));
    const uint64_t want = (count + per_cta - 1) / per_cta;
    const uint64_t cap = (uint64_t)sm_count * (2048 / kReduceThreads);
    const uint64_t grid = std::max<uint64_t>(1, std::min(want, cap));
    if (grid > (uint64_t)kStaticPartials)
        return fail(HEPH_INVALID_CONFIGURATION,
                    "allocation-free reduction needs " + std::to_string(grid) +
                        " CTA partials but its static scratch holds at most " + std::to_string(kStaticPartials));
    void *scratch = nullptr;
    heph_status st = static_scratch_address(&scratch);
    if (st != HEPH_OK) return st;
    Tacc *partials = static_cast<Tacc *>(scratch);
    unsigned int *ticket = reinterpret_cast<unsigned int *>(static_cast<char *>(scratch) + kStaticPartials * 8);
    // The ticket must start at zero; a previous call leaves it at zero, but
    // clear it in stream order so an earlier failed launch cannot poison it.
    HEPH_CUDA_TRY(cudaMemsetAsync(ticket, 0, sizeof(unsigned int), stream), HEPH_DISPATCH_FAILED,
                  "static scratch clear");
    reduce_dense_kernel<Tin, Tacc, OP><<<(unsigned)grid, kReduceThreads, 0, stream>>>(in, count, out, partials, ticket);
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "full reduction launch");
    return HEPH_OK;
}

template <typename Tin, typename Tacc>
heph_status launch_static_op(int op, const void *in, uint64_t count, void *out, cudaStream_t s, int sms) {
    switch (op) {
        case OP_SUM: return launch_static_typed<Tin, Tacc, OP_SUM>(in, count, out, s, sms);
        case OP_PROD: return launch_static_typed<Tin, Tacc, OP_PROD>(in, count, out, s, sms);
        case OP_MIN: return launch_static_typed<Tin, Tacc, OP_MIN>(in, count, out, s, sms);
        case OP_MAX: return launch_static_typed<Tin, Tacc, OP_MAX>(in, count, out, s, sms);
    }
    return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
}

}  // namespace
}  // namespace heph

using namespace heph;

extern "C" heph_status heph_reduce_full_noalloc(heph_op op, heph_dtype in_dtype, heph_dtype out_dtype,
                                                const void *in, uint64_t count, void *out, heph_stream stream) {
    if ((count && !in) || !out) return fail(HEPH_INVALID_CONFIGURATION, "null device pointer");
    if ((reinterpret_cast<uintptr_t>(in) % (dtype_size(in_dtype) ? dtype_size(in_dtype) : 1)) != 0 ||
        (reinterpret_cast<uintptr_t>(out) % (dtype_size(out_dtype) ? dtype_size(out_dtype) : 1)) != 0)
        return fail(HEPH_INVALID_CONFIGURATION, "device pointers must be aligned to their element size");
    int dev = 0, sms = 0;
    HEPH_CUDA_TRY(cudaGetDevice(&dev), HEPH_DEVICE_UNAVAILABLE, "cudaGetDevice");
    HEPH_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), HEPH_DEVICE_UNAVAILABLE,
                  "device query");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (in_dtype == out_dtype) {
        return dispatch_dtype(in_dtype, [&]<typename T>() {
            return launch_static_op<T, T>((int)op, in, count, out, s, sms);
        });
    }
    if (in_dtype == HEPH_I32 && out_dtype == HEPH_I64)
        return launch_static_op<int32_t, int64_t>((int)op, in, count, out, s, sms);
    if (in_dtype == HEPH_F32 && out_dtype == HEPH_F64)
        return launch_static_op<float, double>((int)op, in, count, out, s, sms);
    return fail(HEPH_INVALID_CONFIGURATION,
                "full reduction output type must match the input type or widen it (i32->i64, f32->f64)");
}
