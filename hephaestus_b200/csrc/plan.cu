// plan.cpp — validation and planning (host only; no CUDA calls).
//
// Follows the reference planners message for message:
//   plan_axis_reduction  crates/hephaestus-core/src/domain/reduction.rs:410-500
//   plan_axis_scan       crates/hephaestus-core/src/domain/scan.rs:87-178
//   full reduction       crates/hephaestus-cuda/src/application/full_reduction_seam.rs:59-72
//   layout errors        crates/hephaestus-core/src/domain/planning.rs:10-14 ("layout rejected: ")
// Extents, strides and offsets are 64-bit, so the u32/i32 narrowing errors of
// the reference (planning.rs:17-28) do not arise.
#include "plan.h"

#include <cstdio>
#include <cstdlib>
#include <utility>

#include "common.cuh"

namespace heph {

std::string shape_debug(const heph_layout &l) {
    std::string s = "[";
    for (uint32_t d = 0; d < l.rank && d < HEPH_MAX_RANK; ++d) {
        if (d) s += ", ";
        s += std::to_string(l.shape[d]);
    }
    return s + "]";
}

bool layout_size(const heph_layout &l, uint64_t *out) {
    unsigned __int128 n = 1;
    for (uint32_t d = 0; d < l.rank; ++d) {
        n *= l.shape[d];
        if (n > (unsigned __int128)UINT64_MAX) return false;
    }
    *out = (uint64_t)n;
    return true;
}

bool layout_fits(const heph_layout &l, uint64_t buffer_len, std::string *why) {
    if (l.rank < 1 || l.rank > HEPH_MAX_RANK) {
        *why = "rank " + std::to_string(l.rank) + " is outside 1..=" + std::to_string(HEPH_MAX_RANK);
        return false;
    }
    uint64_t size = 0;
    if (!layout_size(l, &size)) {
        *why = "element count of shape " + shape_debug(l) + " overflows";
        return false;
    }
    if (size == 0) return true;
    __int128 lo = (__int128)l.offset, hi = (__int128)l.offset;
    for (uint32_t d = 0; d < l.rank; ++d) {
        __int128 span = (__int128)(l.shape[d] - 1) * (__int128)l.strides[d];
        if (span < 0) lo += span;
        else hi += span;
    }
    if (lo < 0) {
        *why = "shape " + shape_debug(l) + " with offset " + std::to_string(l.offset) +
               " reaches below storage index 0";
        return false;
    }
    if (hi >= (__int128)buffer_len) {
        *why = "shape " + shape_debug(l) + " with offset " + std::to_string(l.offset) +
               " needs storage index " + std::to_string((unsigned long long)hi) +
               " but the buffer holds " + std::to_string(buffer_len) + " elements";
        return false;
    }
    return true;
}

heph_status validate_layout(const heph_layout &l, uint64_t buffer_len) {
    std::string why;
    if (!layout_fits(l, buffer_len, &why)) return fail(HEPH_DISPATCH_FAILED, "layout rejected: " + why);
    return HEPH_OK;
}

bool has_zero_stride_aliasing(const heph_layout &l) {
    for (uint32_t d = 0; d < l.rank; ++d)
        if (l.shape[d] > 1 && l.strides[d] == 0) return true;
    return false;
}

bool layout_is_dense(const heph_layout &l) {
    int64_t expect = 1;
    for (int d = (int)l.rank - 1; d >= 0; --d) {
        if (l.shape[d] != 1 && l.strides[d] != expect) return false;
        expect *= (int64_t)l.shape[d];
    }
    return true;
}

bool layout_covers_dense_block(const heph_layout &l, int64_t *first) {
    struct Dim {
        uint64_t extent;
        int64_t stride;
    } dims[HEPH_MAX_RANK];
    int k = 0;
    int64_t lo = (int64_t)l.offset;
    for (uint32_t d = 0; d < l.rank && d < HEPH_MAX_RANK; ++d) {
        if (l.shape[d] == 0) return false;
        if (l.shape[d] == 1) continue;
        dims[k++] = {l.shape[d], l.strides[d]};
        if (l.strides[d] < 0) lo += (int64_t)(l.shape[d] - 1) * l.strides[d];
    }
    // insertion sort by |stride|
    for (int i = 1; i < k; ++i)
        for (int j = i; j > 0 && std::llabs(dims[j].stride) < std::llabs(dims[j - 1].stride); --j) std::swap(dims[j], dims[j - 1]);
    int64_t expect = 1;
    for (int i = 0; i < k; ++i) {
        if (std::llabs(dims[i].stride) != expect) return false;
        expect *= (int64_t)dims[i].extent;
    }
    *first = lo;
    return true;
}

static bool same_shape(const heph_layout &a, const heph_layout &b) {
    if (a.rank != b.rank) return false;
    for (uint32_t d = 0; d < a.rank; ++d)
        if (a.shape[d] != b.shape[d]) return false;
    return true;
}

heph_status plan_axis_reduction(const heph_layout &in, uint64_t in_len, const heph_layout &out,
                                uint64_t out_len, uint32_t axis, bool alias, bool *noop,
                                AxisProblem *p) {
    *noop = false;
    if (axis >= 2)
        return fail(HEPH_DISPATCH_FAILED,
                    "axis " + std::to_string(axis) + " is out of bounds for rank-2 reduction");
    if (in.rank != 2 || out.rank != 2)
        return fail(HEPH_DISPATCH_FAILED, "axis reduction operands must be rank 2, got input rank " +
                                              std::to_string(in.rank) + " and output rank " +
                                              std::to_string(out.rank));
    heph_layout expected = in;
    expected.shape[axis] = 1;
    if (!same_shape(expected, out))
        return fail(HEPH_DISPATCH_FAILED, "axis reduction output shape mismatch: input " +
                                              shape_debug(in) + ", axis " + std::to_string(axis) +
                                              ", out " + shape_debug(out));
    if (alias)
        return fail(HEPH_DISPATCH_FAILED, "axis reduction output buffer must not alias input buffer");
    if (has_zero_stride_aliasing(out))
        return fail(HEPH_DISPATCH_FAILED,
                    "axis reduction output layout must not contain zero-stride aliasing");
    heph_status st = validate_layout(in, in_len);
    if (st != HEPH_OK) return st;
    st = validate_layout(out, out_len);
    if (st != HEPH_OK) return st;
    uint64_t out_size = 0;
    layout_size(out, &out_size);
    if (out_size == 0) {
        *noop = true;
        return HEPH_OK;
    }
    uint32_t other = 1 - axis;
    p->outer = in.shape[other];
    p->len = in.shape[axis];
    p->in_base = (int64_t)in.offset;
    p->in_o = in.strides[other];
    p->in_r = in.strides[axis];
    p->out_base = (int64_t)out.offset;
    p->out_o = out.strides[other];
    p->out_r = 0;
    return HEPH_OK;
}

heph_status plan_axis_scan(const heph_layout &in, uint64_t in_len, const heph_layout &out,
                           uint64_t out_len, uint32_t axis, bool alias, bool *noop,
                           AxisProblem *p) {
    *noop = false;
    // The reference accepts rank 2 only (core accelerator/scan.rs:519-523);
    // rank 1 (one line, the 1-D case) is accepted here as an extension.  Any
    // other rank is rejected with the reference's wording.
    if (in.rank != 1 && in.rank != 2)
        return fail(HEPH_DISPATCH_FAILED,
                    "cuda-sm100a scan supports rank 2 only, got rank " + std::to_string(in.rank));
    if (axis >= in.rank)
        return fail(HEPH_DISPATCH_FAILED, "scan axis " + std::to_string(axis) +
                                              " is out of bounds for rank-" +
                                              std::to_string(in.rank) + " scan");
    if (!same_shape(in, out))
        return fail(HEPH_DISPATCH_FAILED, "scan output shape mismatch: input " + shape_debug(in) +
                                              ", out " + shape_debug(out));
    if (alias) return fail(HEPH_DISPATCH_FAILED, "scan output buffer must not alias input buffer");
    if (has_zero_stride_aliasing(out))
        return fail(HEPH_DISPATCH_FAILED, "scan output layout must not contain zero-stride aliasing");
    heph_status st = validate_layout(in, in_len);
    if (st != HEPH_OK) return st;
    st = validate_layout(out, out_len);
    if (st != HEPH_OK) return st;
    uint64_t size = 0;
    layout_size(out, &size);
    if (size == 0) {
        *noop = true;
        return HEPH_OK;
    }
    p->in_base = (int64_t)in.offset;
    p->out_base = (int64_t)out.offset;
    p->len = in.shape[axis];
    p->in_r = in.strides[axis];
    p->out_r = out.strides[axis];
    if (in.rank == 1) {
        p->outer = 1;
        p->in_o = 0;
        p->out_o = 0;
    } else {
        uint32_t other = 1 - axis;
        p->outer = in.shape[other];
        p->in_o = in.strides[other];
        p->out_o = out.strides[other];
    }
    return HEPH_OK;
}

heph_status plan_full_reduction(const heph_layout &in, uint64_t in_len, const heph_layout &out,
                                uint64_t out_len, uint64_t *count) {
    heph_status st = validate_layout(out, out_len);
    if (st != HEPH_OK) return st;
    uint64_t out_size = 0;
    layout_size(out, &out_size);
    if (out_size != 1)
        return fail(HEPH_DISPATCH_FAILED, "full reduction output must have exactly 1 element");
    if (!layout_size(in, count))
        return fail(HEPH_DISPATCH_FAILED, "layout rejected: element count of shape " +
                                              shape_debug(in) + " overflows");
    return validate_layout(in, in_len);
}

}  // namespace heph

// ------------------------------------------------------------------ C ABI

using namespace heph;

extern "C" heph_status heph_validate_reduction_width(uint32_t width) {
    if (width == 0 || (width & (width - 1)) != 0)
        return fail(HEPH_DISPATCH_FAILED,
                    "reduction block width " + std::to_string(width) + " must be a power of two");
    return HEPH_OK;
}

extern "C" heph_status heph_validate_scan_width(uint32_t width) {
    if (width == 0 || (width & (width - 1)) != 0)
        return fail(HEPH_DISPATCH_FAILED,
                    "scan block width " + std::to_string(width) + " must be a power of two");
    return HEPH_OK;
}

extern "C" uint64_t heph_reduction_pass_count(uint64_t len, uint32_t width) {
    if (width < 2) return 0;
    uint64_t passes = 0;
    while (len > 1) {
        len = (len + width - 1) / width;
        ++passes;
    }
    return passes;
}

extern "C" heph_status heph_layout_validate(const heph_layout *layout, uint64_t buffer_len) {
    if (!layout) return fail(HEPH_INVALID_CONFIGURATION, "layout is null");
    return validate_layout(*layout, buffer_len);
}

extern "C" heph_status heph_plan_axis_reduction(const heph_layout *input, uint64_t input_len,
                                                const heph_layout *output, uint64_t output_len,
                                                uint32_t axis, int buffers_alias, int *out_noop) {
    if (!input || !output) return fail(HEPH_INVALID_CONFIGURATION, "layout is null");
    bool noop = false;
    AxisProblem p;
    heph_status st = plan_axis_reduction(*input, input_len, *output, output_len, axis,
                                         buffers_alias != 0, &noop, &p);
    if (out_noop) *out_noop = noop ? 1 : 0;
    return st;
}

extern "C" heph_status heph_plan_axis_scan(const heph_layout *input, uint64_t input_len,
                                           const heph_layout *output, uint64_t output_len,
                                           uint32_t axis, int buffers_alias, int *out_noop) {
    if (!input || !output) return fail(HEPH_INVALID_CONFIGURATION, "layout is null");
    bool noop = false;
    AxisProblem p;
    heph_status st = plan_axis_scan(*input, input_len, *output, output_len, axis,
                                    buffers_alias != 0, &noop, &p);
    if (out_noop) *out_noop = noop ? 1 : 0;
    return st;
}

extern "C" heph_status heph_plan_full_reduction(const heph_layout *input, uint64_t input_len,
                                                const heph_layout *output, uint64_t output_len) {
    if (!input || !output) return fail(HEPH_INVALID_CONFIGURATION, "layout is null");
    uint64_t count = 0;
    return plan_full_reduction(*input, input_len, *output, output_len, &count);
}

namespace heph {

void stream_view(const heph_layout *const *ls, int nops, StreamView *v) {
    struct Dim {
        uint64_t extent;
        int64_t stride[2];
    } dims[HEPH_MAX_RANK];
    int k = 0;
    int64_t off[2] = {0, 0};
    for (int o = 0; o < nops; ++o) off[o] = (int64_t)ls[o]->offset;
    const heph_layout &l0 = *ls[0];
    for (uint32_t d = 0; d < l0.rank && d < HEPH_MAX_RANK; ++d) {
        if (l0.shape[d] == 1) continue;
        Dim x{l0.shape[d], {0, 0}};
        const bool flip = l0.strides[d] < 0;
        for (int o = 0; o < nops; ++o) {
            int64_t s = ls[o]->strides[d];
            if (flip) {
                off[o] += (int64_t)(l0.shape[d] - 1) * s;
                s = -s;
            }
            x.stride[o] = s;
        }
        dims[k++] = x;
    }
    // Stable insertion sort, largest first-operand stride outermost.
    for (int i = 1; i < k; ++i)
        for (int j = i; j > 0 && dims[j].stride[0] > dims[j - 1].stride[0]; --j) std::swap(dims[j], dims[j - 1]);
    // Merge an outer dim into the inner one when, for every operand, stepping
    // the outer dim equals stepping past the whole inner dim.
    int r = 0;
    for (int i = 0; i < k; ++i) {
        if (r > 0) {
            Dim &in = dims[i];
            Dim &out = dims[r - 1];
            bool ok = true;
            for (int o = 0; o < nops; ++o) ok = ok && out.stride[o] == (int64_t)in.extent * in.stride[o];
            if (ok) {
                out.extent *= in.extent;
                for (int o = 0; o < nops; ++o) out.stride[o] = in.stride[o];
                continue;
            }
        }
        dims[r++] = dims[i];
    }
    if (r == 0) dims[r++] = Dim{1, {1, 1}};
    v->rank = (uint32_t)r;
    for (int d = 0; d < r; ++d) {
        v->shape[d] = dims[d].extent;
        for (int o = 0; o < nops; ++o) v->strides[o][d] = dims[d].stride[o];
    }
    for (int o = 0; o < nops; ++o) v->offset[o] = off[o];
}

bool stream_view_vectorize(StreamView *v, int nops, uint32_t elems, const void *const *bases, size_t elem_size) {
    const int in = (int)v->rank - 1;
    const int64_t e = (int64_t)elems;
    if (v->shape[in] % elems) return false;
    for (int o = 0; o < nops; ++o) {
        if (v->strides[o][in] != 1 || v->offset[o] % e) return false;
        for (int d = 0; d < in; ++d)
            if (v->strides[o][d] % e) return false;
        const uintptr_t a = reinterpret_cast<uintptr_t>(bases[o]) + (uintptr_t)(v->offset[o] * (int64_t)elem_size);
        if (a & 15u) return false;
    }
    v->shape[in] /= elems;
    for (int o = 0; o < nops; ++o) {
        for (int d = 0; d < in; ++d) v->strides[o][d] /= e;
        v->offset[o] /= e;
    }
    return true;
}

}  // namespace heph
