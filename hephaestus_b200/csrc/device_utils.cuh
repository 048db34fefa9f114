// device_utils.cuh — device helpers shared by the reduce and scan kernels:
// streaming 128-bit loads, cache-global scalar access, warp/block folds.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace heph {

constexpr unsigned kFullMask = 0xffffffffu;

// 128-bit read-only load that does not allocate in L1 and asks L2 to fetch
// 256-byte sectors (the input is streamed exactly once).
__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// 128-bit store with the streaming (evict-first) hint.
__device__ __forceinline__ void st_stream(uint4 *p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Scalar loads that bypass L1 (values written by other CTAs of this grid).
template <typename T> __device__ __forceinline__ T ld_cg(const T *p) {
    if constexpr (sizeof(T) == 4) {
        uint32_t r;
        asm volatile("ld.global.cg.b32 %0, [%1];" : "=r"(r) : "l"(p));
        return bitcast<T>(r);
    } else {
        uint64_t r;
        asm volatile("ld.global.cg.b64 %0, [%1];" : "=l"(r) : "l"(p));
        return bitcast<T>(r);
    }
}

template <typename T> __device__ __forceinline__ T shfl_xor(T v, int m) {
    if constexpr (sizeof(T) == 4) {
        return bitcast<T>(__shfl_xor_sync(kFullMask, bitcast<uint32_t>(v), m));
    } else {
        return bitcast<
            T>(__shfl_xor_sync(kFullMask, bitcast<unsigned long long>(v), m));
    }
}
template <typename T> __device__ __forceinline__ T shfl_up(T v, int d) {
    if constexpr (sizeof(T) == 4) {
        return bitcast<T>(__shfl_up_sync(kFullMask, bitcast<uint32_t>(v), d));
    } else {
        return bitcast<
            T>(__shfl_up_sync(kFullMask, bitcast<unsigned long long>(v), d));
    }
}
template <typename T> __device__ __forceinline__ T shfl_down(T v, int d) {
    if constexpr (sizeof(T) == 4) {
        return bitcast<T>(__shfl_down_sync(kFullMask, bitcast<uint32_t>(v), d));
    } else {
        return bitcast<
            T>(__shfl_down_sync(kFullMask, bitcast<unsigned long long>(v), d));
    }
}
template <typename T> __device__ __forceinline__ T shfl_idx(T v, int src) {
    if constexpr (sizeof(T) == 4) {
        return bitcast<T>(__shfl_sync(kFullMask, bitcast<uint32_t>(v), src));
    } else {
        return bitcast<
            T>(__shfl_sync(kFullMask, bitcast<unsigned long long>(v), src));
    }
}

// Warp-wide fold of one value per lane; every lane receives the result.
// 32-bit integer add/min/max use the redux.sync instruction.
template <typename T, int OP> __device__ __forceinline__ T warp_fold(T v) {
    if constexpr (std::is_same_v<T, uint32_t> && OP == OP_SUM) {
        return __reduce_add_sync(kFullMask, v);
    } else if constexpr (std::is_same_v<T, uint32_t> && OP == OP_MIN) {
        return __reduce_min_sync(kFullMask, v);
    } else if constexpr (std::is_same_v<T, uint32_t> && OP == OP_MAX) {
        return __reduce_max_sync(kFullMask, v);
    } else if constexpr (std::is_same_v<T, int32_t> && OP == OP_SUM) {
        return (int32_t)__reduce_add_sync(kFullMask, (uint32_t)v);
    } else if constexpr (std::is_same_v<T, int32_t> && OP == OP_MIN) {
        return __reduce_min_sync(kFullMask, v);
    } else if constexpr (std::is_same_v<T, int32_t> && OP == OP_MAX) {
        return __reduce_max_sync(kFullMask, v);
    } else {
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) v = combine<T, OP>(v, shfl_xor(v, m));
        return v;
    }
}

// Block-wide fold (blockDim.x == THREADS, a multiple of 32).  The result is
// valid in every thread.  `scratch` holds THREADS/32 values.
template <typename T, int OP, int THREADS>
__device__ __forceinline__ T block_fold(T v, T *scratch) {
    constexpr int W = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_fold<T, OP>(v);
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    T r = scratch[0];
#pragma unroll
    for (int w = 1; w < W; ++w) r = combine<T, OP>(r, scratch[w]);
    __syncthreads();
    return r;
}

// Arg-fold helpers: (value, index) pairs, lowest index among equal extrema.
template <typename T, int OP>
__device__ __forceinline__ bool arg_better(T v, uint32_t i, T bv, uint32_t bi) {
    // Index 0xffffffff marks "no element seen" and loses to any element.
    if (i == 0xffffffffu) return false;
    if (bi == 0xffffffffu) return true;
    if constexpr (OP == OP_MAX) return v > bv || (v == bv && i < bi);
    else return v < bv || (v == bv && i < bi);
}

template <typename T, int OP> __device__ __forceinline__ void warp_arg_fold(T &v, uint32_t &i) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
        T ov = shfl_xor(v, m);
        uint32_t oi = __shfl_xor_sync(kFullMask, i, m);
        if (arg_better<T, OP>(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

// Reinterpret a 16-byte vector as V elements of T.
template <typename T> struct Vec16 {
    static constexpr int V = 16 / sizeof(T);
    T e[V];
};
template <typename T> __device__ __forceinline__ Vec16<T> as_elems(uint4 u) {
    return bitcast<Vec16<T>>(u);
}
template <typename T> __device__ __forceinline__ uint4 as_uint4(const Vec16<T> &v) {
    return bitcast<uint4>(v);
}

// Nanoseconds of the GPU's global timer (for time-bounded waits).
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Deadline of a wait on another CTA's (or another launch's) progress, kept by
// the global timer rather than by a poll count: __nanosleep is only a hint,
// and on a time-sliced GPU a slow but live partner must not be mistaken for
// a lost one.  The timer is read every 64 polls; the clock starts at the
// first read, so a wait that succeeds within 63 polls never reads it.
constexpr uint64_t kWaitDeadlineNs = 2000000000ull;  // 2 s
struct WaitDeadline {
    uint64_t start = 0;
    uint32_t polls = 0;
    __device__ __forceinline__ bool expired() {
        if ((++polls & 63u) != 0) return false;
        const uint64_t now = globaltimer_ns();
        if (start == 0) {
            start = now;
            return false;
        }
        return now - start > kWaitDeadlineNs;
    }
};

// Sets a device-side error bit visible to the host after synchronisation.
__device__ __forceinline__ void raise_device_error(unsigned int *err, unsigned int code) {
    if (err) atomicOr(err, code);
}

// ------------------------------------------- bulk copies into shared memory

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Thread 0: expect `bytes` on `bar` and start a bulk global->shared copy
// (a plain bulk copy; the source is this GPU's own memory).
__device__ __forceinline__ void bulk_load(void *dst_smem, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst_smem)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// Waits for phase `parity` of `bar`.  Bounded in time (WaitDeadline): past
// the deadline the device error bit is raised and the wait gives up.
__device__ __forceinline__ void mbar_wait(uint64_t *bar, uint32_t parity, unsigned int *err) {
    WaitDeadline deadline;
    while (true) {
        uint32_t done;
        asm volatile("{\n .reg .pred P;\n mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n selp.u32 %0, 1, 0, P;\n}"
                     : "=r"(done)
                     : "r"(smem_addr(bar)), "r"(parity)
                     : "memory");
        if (done) return;
        if (deadline.expired()) break;
    }
    if (threadIdx.x == 0) raise_device_error(err, DEVERR_BULK_TIMEOUT);
}

}  // namespace heph
