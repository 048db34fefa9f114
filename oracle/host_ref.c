/*
 * host_ref.c — CPU oracle for the reduce/scan path (TEST INFRASTRUCTURE ONLY;
 * see host_ref.h for what it restates and where from).  Plain sequential
 * loops: clarity over speed, except the *_mt baseline variants at the end.
 */
#include "host_ref.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------ view walking */

static uint64_t layout_size(const href_layout *l) {
    uint64_t n = 1;
    for (uint32_t d = 0; d < l->rank; ++d) n *= l->shape[d];
    return n;
}

/* Element offset of the logical (row-major) position `linear`. */
static int64_t layout_offset_of(const href_layout *l, uint64_t linear) {
    int64_t off = (int64_t)l->offset;
    for (int d = (int)l->rank - 1; d >= 0; --d) {
        uint64_t extent = l->shape[d];
        uint64_t c = linear % extent;
        linear /= extent;
        off += (int64_t)c * l->strides[d];
    }
    return off;
}

/* Rank-2 element offset of (row, col). */
static int64_t at2(const href_layout *l, uint64_t r, uint64_t c) {
    return (int64_t)l->offset + (int64_t)r * l->strides[0] + (int64_t)c * l->strides[1];
}

/* ------------------------------------------------------- typed operations */
/* Identities: crates/hephaestus-core/src/domain/ops.rs:926-984 (f32/u32/i32);
 * f64/i64 use the analogous extremes. Integer arithmetic wraps (computed in
 * the unsigned type of the same width). */

#define DEFINE_TYPE(SUF, T, UT, IS_FLOAT, MINV, MAXV)                                      \
    static T SUF##_identity(int op) {                                                      \
        switch (op) {                                                                      \
            case HREF_PROD: return (T)1;                                                   \
            case HREF_MIN: return (T)(MAXV);                                               \
            case HREF_MAX: return (T)(MINV);                                               \
            default: return (T)0;                                                          \
        }                                                                                  \
    }                                                                                      \
    static T SUF##_combine(int op, T lhs, T rhs) {                                         \
        switch (op) {                                                                      \
            case HREF_PROD:                                                                \
                if (IS_FLOAT) return (T)(lhs * rhs);                                       \
                return (T)((UT)lhs * (UT)rhs);                                             \
            case HREF_MIN: return (lhs < rhs) ? lhs : rhs;                                 \
            case HREF_MAX: return (lhs > rhs) ? lhs : rhs;                                 \
            default:                                                                       \
                if (IS_FLOAT) return (T)(lhs + rhs);                                       \
                return (T)((UT)lhs + (UT)rhs);                                             \
        }                                                                                  \
    }                                                                                      \
    static T SUF##_div_len(T sum, uint64_t len) { return (T)(sum / (T)len); }

DEFINE_TYPE(f32, float, float, 1, -FLT_MAX, FLT_MAX)
DEFINE_TYPE(f64, double, double, 1, -DBL_MAX, DBL_MAX)
DEFINE_TYPE(u32, uint32_t, uint32_t, 0, 0u, UINT32_MAX)
DEFINE_TYPE(i32, int32_t, uint32_t, 0, INT32_MIN, INT32_MAX)
DEFINE_TYPE(i64, int64_t, uint64_t, 0, INT64_MIN, INT64_MAX)

/* ---------------------------------------------------------- full reduction */
/* FullReductionOps::reduce_full_into (core reduction.rs:267): one element out,
 * identity for an empty view. */

#define DEFINE_FULL(SUF, T, IN_T)                                                          \
    static void SUF##_full_from_##IN_T(int op, const IN_T *base, const href_layout *l,     \
                                       T *out) {                                           \
        uint64_t n = layout_size(l);                                                       \
        T acc = SUF##_identity(op);                                                        \
        for (uint64_t i = 0; i < n; ++i)                                                   \
            acc = SUF##_combine(op, acc, (T)base[layout_offset_of(l, i)]);                 \
        *out = acc;                                                                        \
    }

DEFINE_FULL(f32, float, float)
DEFINE_FULL(f64, double, double)
DEFINE_FULL(f64, double, float)
DEFINE_FULL(u32, uint32_t, uint32_t)
DEFINE_FULL(i32, int32_t, int32_t)
DEFINE_FULL(i64, int64_t, int64_t)
DEFINE_FULL(i64, int64_t, int32_t)

int href_reduce_full(int dtype, int out_dtype, int op, const void *base, const href_layout *l,
                     void *out) {
    if (op < HREF_SUM || op > HREF_MAX) return -1;
    if (dtype == out_dtype) {
        switch (dtype) {
            case HREF_F32: f32_full_from_float(op, base, l, out); return 0;
            case HREF_F64: f64_full_from_double(op, base, l, out); return 0;
            case HREF_U32: u32_full_from_uint32_t(op, base, l, out); return 0;
            case HREF_I32: i32_full_from_int32_t(op, base, l, out); return 0;
            case HREF_I64: i64_full_from_int64_t(op, base, l, out); return 0;
            default: return -1;
        }
    }
    if (dtype == HREF_I32 && out_dtype == HREF_I64) {
        i64_full_from_int32_t(op, base, l, out);
        return 0;
    }
    if (dtype == HREF_F32 && out_dtype == HREF_F64) {
        f64_full_from_float(op, base, l, out);
        return 0;
    }
    return -1;
}

/* ----------------------------------------------------------- axis reduction */
/* axis_reduction_kernel / mean_axis_kernel semantics
 * (hephaestus-cuda application/reduction.rs:218-297): for each output
 * position, fold the reduced axis in increasing order from the identity. */

#define DEFINE_AXIS(SUF, T)                                                                \
    static void SUF##_axis(int op, const T *in, const href_layout *il, uint32_t axis,      \
                           T *out, const href_layout *ol) {                                \
        uint64_t len = il->shape[axis];                                                    \
        uint64_t outer = il->shape[1 - axis];                                              \
        int fold = (op == HREF_MEAN) ? HREF_SUM : op;                                      \
        for (uint64_t o = 0; o < outer; ++o) {                                             \
            T acc = SUF##_identity(fold);                                                  \
            for (uint64_t r = 0; r < len; ++r) {                                           \
                uint64_t row = axis == 0 ? r : o, col = axis == 0 ? o : r;                 \
                acc = SUF##_combine(fold, acc, in[at2(il, row, col)]);                     \
            }                                                                              \
            if (op == HREF_MEAN) acc = SUF##_div_len(acc, len);                            \
            uint64_t orow = axis == 0 ? 0 : o, ocol = axis == 0 ? o : 0;                   \
            out[at2(ol, orow, ocol)] = acc;                                                \
        }                                                                                  \
    }

DEFINE_AXIS(f32, float)
DEFINE_AXIS(f64, double)
DEFINE_AXIS(u32, uint32_t)
DEFINE_AXIS(i32, int32_t)
DEFINE_AXIS(i64, int64_t)

int href_reduce_axis(int dtype, int op, const void *in, const href_layout *il, uint32_t axis,
                     void *out, const href_layout *ol) {
    if (il->rank != 2 || ol->rank != 2 || axis > 1 || op < HREF_SUM || op > HREF_MEAN)
        return -1;
    if ((op == HREF_MIN || op == HREF_MAX || op == HREF_MEAN) && il->shape[axis] == 0)
        return -1;
    switch (dtype) {
        case HREF_F32: f32_axis(op, in, il, axis, out, ol); return 0;
        case HREF_F64: f64_axis(op, in, il, axis, out, ol); return 0;
        case HREF_U32: u32_axis(op, in, il, axis, out, ol); return 0;
        case HREF_I32: i32_axis(op, in, il, axis, out, ol); return 0;
        case HREF_I64: i64_axis(op, in, il, axis, out, ol); return 0;
        default: return -1;
    }
}

/* ------------------------------------------------------------ arg-reduction */
/* [EXT] The first position holding the extreme wins (strict comparison while
 * walking positions in increasing order). */

#define DEFINE_ARG(SUF, T)                                                                 \
    static void SUF##_arg(int op, const T *in, const href_layout *il, uint32_t axis,       \
                          T *vals, const href_layout *vl, uint32_t *idx,                   \
                          const href_layout *xl) {                                         \
        uint64_t len = il->shape[axis];                                                    \
        uint64_t outer = il->shape[1 - axis];                                              \
        for (uint64_t o = 0; o < outer; ++o) {                                             \
            T best = 0;                                                                    \
            uint32_t best_i = 0;                                                           \
            for (uint64_t r = 0; r < len; ++r) {                                           \
                uint64_t row = axis == 0 ? r : o, col = axis == 0 ? o : r;                 \
                T v = in[at2(il, row, col)];                                               \
                if (r == 0 || (op == HREF_MAX ? (v > best) : (v < best))) {                \
                    best = v;                                                              \
                    best_i = (uint32_t)r;                                                  \
                }                                                                          \
            }                                                                              \
            uint64_t orow = axis == 0 ? 0 : o, ocol = axis == 0 ? o : 0;                   \
            vals[at2(vl, orow, ocol)] = best;                                              \
            idx[at2(xl, orow, ocol)] = best_i;                                             \
        }                                                                                  \
    }

DEFINE_ARG(f32, float)
DEFINE_ARG(f64, double)
DEFINE_ARG(u32, uint32_t)
DEFINE_ARG(i32, int32_t)
DEFINE_ARG(i64, int64_t)

int href_arg_reduce_axis(int dtype, int op, const void *in, const href_layout *il,
                         uint32_t axis, void *values, const href_layout *vl, uint32_t *indices,
                         const href_layout *xl) {
    if (il->rank != 2 || axis > 1 || (op != HREF_MIN && op != HREF_MAX)) return -1;
    if (il->shape[axis] == 0) return -1;
    switch (dtype) {
        case HREF_F32: f32_arg(op, in, il, axis, values, vl, indices, xl); return 0;
        case HREF_F64: f64_arg(op, in, il, axis, values, vl, indices, xl); return 0;
        case HREF_U32: u32_arg(op, in, il, axis, values, vl, indices, xl); return 0;
        case HREF_I32: i32_arg(op, in, il, axis, values, vl, indices, xl); return 0;
        case HREF_I64: i64_arg(op, in, il, axis, values, vl, indices, xl); return 0;
        default: return -1;
    }
}

/* --------------------------------------------------------------------- scan */
/* scan_kernel semantics (core accelerator/scan.rs:94-147): along each line,
 * Forward accumulates from index 0 upward, Reverse from the last index
 * downward; acc = combine(acc, x).  Exclusive [EXT] writes acc before the
 * combine. */

#define DEFINE_SCAN(SUF, T)                                                                \
    static void SUF##_scan(int op, int reverse, int exclusive, const T *in,                \
                           const href_layout *il, uint32_t axis, T *out,                   \
                           const href_layout *ol) {                                        \
        uint64_t len = il->shape[axis];                                                    \
        uint64_t lines = il->rank == 1 ? 1 : il->shape[1 - axis];                          \
        for (uint64_t line = 0; line < lines; ++line) {                                    \
            T acc = SUF##_identity(op);                                                    \
            for (uint64_t s = 0; s < len; ++s) {                                           \
                uint64_t idx = reverse ? len - 1 - s : s;                                  \
                int64_t src, dst;                                                          \
                if (il->rank == 1) {                                                       \
                    src = (int64_t)il->offset + (int64_t)idx * il->strides[0];             \
                    dst = (int64_t)ol->offset + (int64_t)idx * ol->strides[0];             \
                } else {                                                                   \
                    uint64_t row = axis == 0 ? idx : line, col = axis == 0 ? line : idx;   \
                    src = at2(il, row, col);                                               \
                    dst = at2(ol, row, col);                                               \
                }                                                                          \
                T x = in[src];                                                             \
                if (exclusive) {                                                           \
                    out[dst] = acc;                                                        \
                    acc = SUF##_combine(op, acc, x);                                       \
                } else {                                                                   \
                    acc = SUF##_combine(op, acc, x);                                       \
                    out[dst] = acc;                                                        \
                }                                                                          \
            }                                                                              \
        }                                                                                  \
    }

DEFINE_SCAN(f32, float)
DEFINE_SCAN(f64, double)
DEFINE_SCAN(u32, uint32_t)
DEFINE_SCAN(i32, int32_t)
DEFINE_SCAN(i64, int64_t)

int href_scan_axis(int dtype, int op, int reverse, int exclusive, const void *in,
                   const href_layout *il, uint32_t axis, void *out, const href_layout *ol) {
    if (op != HREF_SUM && op != HREF_PROD) return -1;
    if (il->rank == 1 ? axis != 0 : (il->rank != 2 || axis > 1)) return -1;
    switch (dtype) {
        case HREF_F32: f32_scan(op, reverse, exclusive, in, il, axis, out, ol); return 0;
        case HREF_F64: f64_scan(op, reverse, exclusive, in, il, axis, out, ol); return 0;
        case HREF_U32: u32_scan(op, reverse, exclusive, in, il, axis, out, ol); return 0;
        case HREF_I32: i32_scan(op, reverse, exclusive, in, il, axis, out, ol); return 0;
        case HREF_I64: i64_scan(op, reverse, exclusive, in, il, axis, out, ol); return 0;
        default: return -1;
    }
}

/* ------------------------------------------------------ map reductions */

#define DEFINE_MAP(SUF, T, UT, IS_FLOAT, IS_SIGNED)                                         \
    static T SUF##_abs(T v) {                                                              \
        if (IS_FLOAT) return v < (T)0 ? -v : (v == (T)0 ? (T)0 : v);                        \
        if (IS_SIGNED) return v < (T)0 ? (T)((UT)0 - (UT)v) : v;                            \
        return v;                                                                          \
    }                                                                                      \
    static void SUF##_map(int map, const T *a, const href_layout *la, const T *b,         \
                          const href_layout *lb, T *out) {                                 \
        uint64_t n = layout_size(la);                                                      \
        int red = map == 4 ? HREF_MAX : HREF_SUM;                                          \
        T acc = SUF##_identity(red);                                                       \
        for (uint64_t i = 0; i < n; ++i) {                                                 \
            T x = a[layout_offset_of(la, i)];                                              \
            T m;                                                                           \
            if (map == 0) m = SUF##_combine(HREF_PROD, x, b[layout_offset_of(lb, i)]);     \
            else if (map == 1) m = x;                                                      \
            else if (map == 3) m = SUF##_combine(HREF_PROD, x, x);                         \
            else m = SUF##_abs(x);                                                         \
            acc = SUF##_combine(red, acc, m);                                              \
        }                                                                                  \
        *out = acc;                                                                        \
    }

DEFINE_MAP(f32, float, float, 1, 1)
DEFINE_MAP(f64, double, double, 1, 1)
DEFINE_MAP(u32, uint32_t, uint32_t, 0, 0)
DEFINE_MAP(i32, int32_t, uint32_t, 0, 1)
DEFINE_MAP(i64, int64_t, uint64_t, 0, 1)

int href_map_reduce(int dtype, int map, const void *a, const href_layout *la, const void *b,
                    const href_layout *lb, void *out) {
    if (map < 0 || map > 4) return -1;
    if (map != 0) { b = a; lb = la; }
    switch (dtype) {
        case HREF_F32:
            f32_map(map, a, la, b, lb, out);
            if (map == 3) *(float *)out = sqrtf(*(float *)out);
            return 0;
        case HREF_F64:
            f64_map(map, a, la, b, lb, out);
            if (map == 3) *(double *)out = sqrt(*(double *)out);
            return 0;
        case HREF_U32: if (map == 3) return -1; u32_map(map, a, la, b, lb, out); return 0;
        case HREF_I32: if (map == 3) return -1; i32_map(map, a, la, b, lb, out); return 0;
        case HREF_I64: if (map == 3) return -1; i64_map(map, a, la, b, lb, out); return 0;
        default: return -1;
    }
}

/* -------------------------------------------------------------- generators */

/* SplitMix64 output function (Steele, Lea & Flood, OOPSLA 2014), applied to
 * the counter advanced by the golden-ratio increment. */
static uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t href_hash(uint64_t seed, uint64_t index) { return splitmix64((seed << 32) ^ index); }

void href_generate(int kind, uint64_t seed, uint64_t base, uint64_t count, void *out) {
    for (uint64_t k = 0; k < count; ++k) {
        uint64_t i = base + k;
        switch (kind) {
            case HREF_GEN_F32_UNIFORM_PM1: {
                uint64_t h = href_hash(seed, i);
                ((float *)out)[k] = -1.0f + 2.0f * ((float)(h >> 40) * 0x1p-24f);
                break;
            }
            case HREF_GEN_U32_LOW4:
                ((uint32_t *)out)[k] = (uint32_t)(href_hash(seed, i) & 15u);
                break;
            case HREF_GEN_F32_NORMAL: {
                /* Box & Muller (1958): u1 in (0,1], u2 in [0,1). */
                double u1 = (double)((href_hash(seed, 2 * i) >> 11) + 1) * 0x1p-53;
                double u2 = (double)(href_hash(seed, 2 * i + 1) >> 11) * 0x1p-53;
                double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
                ((float *)out)[k] = (float)z;
                break;
            }
            case HREF_GEN_F64_UNIT:
                ((double *)out)[k] = (double)(href_hash(seed, i) >> 11) * 0x1p-53;
                break;
            case HREF_GEN_I32_PM1000:
                ((int32_t *)out)[k] = (int32_t)(href_hash(seed, i) % 2001u) - 1000;
                break;
            default: break;
        }
    }
}

/* ---------------------------------------------------- CPU baseline (OpenMP) */

int href_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int pick_threads(int threads) { return threads > 0 ? threads : href_max_threads(); }

/* Two-pass chunked scan: per-chunk totals, serial carry, per-chunk scan. */
#define DEFINE_MT_SCAN(NAME, T, UT, EXCL)                                                  \
    void NAME(const T *in, T *out, uint64_t n, T carry, int threads) {                     \
        int nt = pick_threads(threads);                                                    \
        UT *totals = (UT *)calloc((size_t)nt + 1, sizeof(UT));                             \
        _Pragma("omp parallel num_threads(nt)") {                                          \
            int t = 0, tn = 1;                                                             \
            PAR_IDS(t, tn);                                                                \
            uint64_t lo = n * (uint64_t)t / (uint64_t)tn, hi = n * (uint64_t)(t + 1) / (uint64_t)tn; \
            UT s = 0;                                                                      \
            for (uint64_t i = lo; i < hi; ++i) s += (UT)in[i];                             \
            totals[t + 1] = s;                                                             \
            _Pragma("omp barrier");                                                        \
            UT acc = (UT)carry;                                                            \
            for (int q = 0; q <= t; ++q) acc += totals[q];                                 \
            for (uint64_t i = lo; i < hi; ++i) {                                           \
                if (EXCL) {                                                                \
                    out[i] = (T)acc;                                                       \
                    acc += (UT)in[i];                                                      \
                } else {                                                                   \
                    acc += (UT)in[i];                                                      \
                    out[i] = (T)acc;                                                       \
                }                                                                          \
            }                                                                              \
        }                                                                                  \
        free(totals);                                                                      \
    }

#ifdef _OPENMP
#define PAR_IDS(t, tn) do { t = omp_get_thread_num(); tn = omp_get_num_threads(); } while (0)
#else
#define PAR_IDS(t, tn) do { t = 0; tn = 1; } while (0)
#endif

DEFINE_MT_SCAN(href_exclusive_scan_u32_mt, uint32_t, uint32_t, 1)
DEFINE_MT_SCAN(href_inclusive_scan_i32_mt, int32_t, uint32_t, 0)

int64_t href_sum_i32_to_i64_mt(const int32_t *in, uint64_t n, int threads) {
    int nt = pick_threads(threads);
    uint64_t total = 0;
#pragma omp parallel for num_threads(nt) reduction(+ : total) schedule(static)
    for (uint64_t i = 0; i < n; ++i) total += (uint64_t)(int64_t)in[i];
    return (int64_t)total;
}

float href_sum_f32_mt(const float *in, uint64_t n, int threads) {
    int nt = pick_threads(threads);
    float total = 0.0f;
#pragma omp parallel for num_threads(nt) reduction(+ : total) schedule(static)
    for (uint64_t i = 0; i < n; ++i) total += in[i];
    return total;
}

void href_row_argmax_f32_mt(const float *in, uint64_t rows, uint64_t cols, float *values,
                            uint32_t *indices, int threads) {
    int nt = pick_threads(threads);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (uint64_t r = 0; r < rows; ++r) {
        const float *row = in + r * cols;
        float best = row[0];
        uint32_t bi = 0;
        for (uint64_t c = 1; c < cols; ++c)
            if (row[c] > best) {
                best = row[c];
                bi = (uint32_t)c;
            }
        values[r] = best;
        indices[r] = bi;
    }
}

void href_col_sum_f64_mt(const double *in, uint64_t rows, uint64_t cols, double *out,
                         int threads) {
    int nt = pick_threads(threads);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (uint64_t c0 = 0; c0 < cols; c0 += 256) {
        uint64_t c1 = c0 + 256 < cols ? c0 + 256 : cols;
        for (uint64_t c = c0; c < c1; ++c) out[c] = 0.0;
        for (uint64_t r = 0; r < rows; ++r)
            for (uint64_t c = c0; c < c1; ++c) out[c] += in[r * cols + c];
    }
}
