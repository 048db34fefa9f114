// plan.h — host-side validation and planning of the reduce/scan dispatches
// (the backend-neutral planners of hephaestus-core, with 64-bit extents).
#pragma once

#include <cstdint>
#include <string>

#include "heph/heph.h"

namespace heph {

std::string shape_debug(const heph_layout &l);  // Rust Debug form, e.g. "[3, 4]"
bool layout_size(const heph_layout &l, uint64_t *out);
// leto::Layout::validate_storage_len + checked_size; message without prefix.
bool layout_fits(const heph_layout &l, uint64_t buffer_len, std::string *why);
heph_status validate_layout(const heph_layout &l, uint64_t buffer_len);
bool has_zero_stride_aliasing(const heph_layout &l);

// Rank-2 axis problem in canonical form: out[o] = fold_r in[in_base + o*in_o + r*in_r],
// written to out_base + o*out_o.
struct AxisProblem {
    uint64_t outer = 0;  // number of outputs
    uint64_t len = 0;    // reduced-axis (or scan-line) length
    int64_t in_base = 0, in_o = 0, in_r = 0;
    int64_t out_base = 0, out_o = 0, out_r = 0;  // out_r used by scans only
};

heph_status plan_axis_reduction(const heph_layout &in, uint64_t in_len, const heph_layout &out,
                                uint64_t out_len, uint32_t axis, bool alias, bool *noop,
                                AxisProblem *p);
heph_status plan_axis_scan(const heph_layout &in, uint64_t in_len, const heph_layout &out,
                           uint64_t out_len, uint32_t axis, bool alias, bool *noop,
                           AxisProblem *p);
heph_status plan_full_reduction(const heph_layout &in, uint64_t in_len, const heph_layout &out,
                                uint64_t out_len, uint64_t *count);

// True when the view covers `count` consecutive elements starting at its
// offset in row-major order (so it can be read as one contiguous run).
bool layout_is_dense(const heph_layout &l);

// True when the view visits every element of one contiguous block exactly
// once, in some order (a transposed, permuted or reversed dense layout);
// *first receives the block's first element offset.  An order-insensitive
// fold (every operator here is commutative) can then read the block
// contiguously.
bool layout_covers_dense_block(const heph_layout &l, int64_t *first);

}  // namespace heph
