// kernels.h — host launchers of the sm_100a kernels (one per kernel family).
// Each launcher validates nothing (the C ABI layer has planned the call) and
// enqueues on `stream`; workspaces come from the device's per-stream pool.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"
#include "plan.h"

namespace heph {

// Full reduction of `count` elements of the view (base pointer = buffer
// start, layout in elements) into the single element at `out`.
// acc_dtype == in_dtype, or a widening pair (I32->I64, F32->F64).
heph_status launch_reduce_full(Device *dev, cudaStream_t stream, int op, heph_dtype in_dtype,
                               heph_dtype acc_dtype, const void *base, const heph_layout &layout,
                               uint64_t count, void *out);

// One problem of a fused batch of dense full reductions: `in` points at the
// first element of a dense run of n elements, `out` at the output element.
// cta_begin / ctas are filled by plan_reduce_full_fused.
struct FusedFull {
    const void *in;
    uint64_t n;
    void *out;
    uint32_t cta_begin;
    uint32_t ctas;
};

// Splits the resident-CTA budget of `dev` over the problems (all of
// in_dtype); returns the grid size (sum of ctas) = partial slots needed.
uint32_t plan_reduce_full_fused(const Device *dev, heph_dtype in_dtype, FusedFull *table, uint32_t nprob);

// One launch for the whole table (device copy); partials: grid x acc-size
// bytes, tickets: nprob zeroed words, both owned by the caller.
heph_status launch_reduce_full_fused(cudaStream_t stream, int op, heph_dtype in_dtype, heph_dtype acc_dtype,
                                     const FusedFull *table, uint32_t nprob, uint32_t grid, void *partials,
                                     unsigned int *tickets);

// Two reductions of one dense run of n elements in one read: op1 in the
// input type into out1, op2 in acc2_dtype (the input type or its widening)
// into out2.
heph_status launch_reduce_dual(Device *dev, cudaStream_t stream, int op1, int op2, heph_dtype dtype,
                               heph_dtype acc2_dtype, const void *in, uint64_t n, void *out1, void *out2);

// Rank-2 axis reduction.  `mean` divides the sum by the axis length;
// `indices` (u32, same layout as out) selects the arg-reduction form.
heph_status launch_reduce_axis(Device *dev, cudaStream_t stream, int op, heph_dtype dtype,
                               const void *in, const AxisProblem &p, void *out, bool mean,
                               uint32_t *indices, int64_t idx_base, int64_t idx_o);

// Fused map-reduction (dot / identity / |x| / x^2 then sqrt / max |x|) of two
// same-shape views into the single element at `out`.
heph_status launch_map_reduce(Device *dev, cudaStream_t stream, int map, heph_dtype dtype, const void *a,
                              const heph_layout &la, const void *b, const heph_layout &lb, uint64_t count,
                              void *out);

// Bounded-wait self-test: 0 = look-back wait, 1 = staged-part mbarrier wait,
// each against a partner that never arrives (raises the device error bit).
heph_status launch_wait_selftest(Device *dev, cudaStream_t stream, int which);

// Axis scan (rank 1 or 2).  `carry` (nullable, device) seeds line 0.
heph_status launch_scan(Device *dev, cudaStream_t stream, int op, heph_dtype dtype,
                        const void *in, void *out, const AxisProblem &p, bool reverse,
                        bool exclusive, const void *carry);

}  // namespace heph
