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

namespace heph {

// A view (or NOPS views of one shape, walked in lockstep) reshaped for
// streaming by an order-insensitive fold: unit dims dropped, dims ordered by
// the first operand's |stride| (largest outermost), dims where the first
// operand's stride is negative flipped in every operand (the pairing of
// elements is kept), and adjacent dims merged where every operand allows it.
// A dense or permuted-dense block comes out as rank 1, stride 1.
struct StreamView {
    uint32_t rank = 0;  // 1..HEPH_MAX_RANK (an empty view never gets here)
    uint64_t shape[HEPH_MAX_RANK] = {};
    int64_t strides[2][HEPH_MAX_RANK] = {};
    int64_t offset[2] = {};
};
void stream_view(const heph_layout *const *ls, int nops, StreamView *v);

// Divides the innermost dim into 16-byte units of `elems` elements when every
// operand's innermost stride is 1, its extent, the other strides and the
// offsets are multiples of `elems`, and every operand's first element address
// (base + offset) is 16-byte aligned.  Returns false and leaves *v unchanged
// otherwise.
bool stream_view_vectorize(StreamView *v, int nops, uint32_t elems, const void *const *bases, size_t elem_size);

}  // namespace heph
