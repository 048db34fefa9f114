/*
 * host_ref.h — CPU oracle for the reduce/scan path.  TEST INFRASTRUCTURE ONLY:
 * used by tests/, __graft_entry__.smoke() and bench.py's CPU baseline as the
 * checker; the product library never links or calls it.
 *
 * It restates, in plain C, the semantics hephaestus defines for this path:
 *  - sequential left folds in the element type, wrapping two's-complement
 *    integers (the host reference device's contract,
 *    crates/hephaestus-host/src/lib.rs:1-9 and docs/adr/0046-host-reference-device.md);
 *  - identities of crates/hephaestus-core/src/domain/ops.rs:926-984
 *    (f32 min/max identities are +/-3.402823466e+38, not infinities),
 *    extended to f64/i64 with the analogous values;
 *  - combine expressions of the CUDA dialect: min(a,b) = a<b?a:b and
 *    max(a,b) = a>b?a:b (crates/hephaestus-cuda/src/application/reduction.rs:24-25),
 *    lhs the accumulator, rhs the element;
 *  - keepdims rank-2 axis reductions, mean = sum / axis length in the element
 *    type (reduction.rs:268-297);
 *  - inclusive forward/reverse axis scans (core accelerator/scan.rs:94-147),
 *    plus exclusive scans: out[i] = fold of the elements strictly before i in
 *    scan order, the identity first;
 *  - arg-reductions with the lowest index among equal extrema.
 *
 * Parity status: pinned against the reference's conformance and contract
 * fixtures (tests/golden/reference_fixtures.json, transcribed from the
 * reference's test sources with file:line).  The reference itself (Rust) cannot
 * be built here, and its RNG (leto, not vendored) cannot be reproduced, so
 * large seeded cases are checked against this restatement only.
 */
#ifndef HEPH_ORACLE_HOST_REF_H
#define HEPH_ORACLE_HOST_REF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { HREF_F32 = 0, HREF_F64 = 1, HREF_U32 = 2, HREF_I32 = 3, HREF_I64 = 4 };
enum { HREF_SUM = 0, HREF_PROD = 1, HREF_MIN = 2, HREF_MAX = 3, HREF_MEAN = 4 };

typedef struct href_layout {
    uint32_t rank;
    uint32_t _pad;
    uint64_t shape[4];
    int64_t strides[4];
    uint64_t offset;
} href_layout;

/* Full reduction of the view (row-major logical order) into *out of
 * out_dtype (== dtype, or I32->I64 / F32->F64 widening).  Returns 0, or -1 on
 * an unsupported combination. */
int href_reduce_full(int dtype, int out_dtype, int op, const void *base,
                     const href_layout *layout, void *out);

/* Rank-2 keepdims axis reduction; out written through out_layout. */
int href_reduce_axis(int dtype, int op, const void *in, const href_layout *in_layout,
                     uint32_t axis, void *out, const href_layout *out_layout);

/* Rank-2 arg-reduction (op MIN or MAX): value and u32 position along axis. */
int href_arg_reduce_axis(int dtype, int op, const void *in, const href_layout *in_layout,
                         uint32_t axis, void *values, const href_layout *values_layout,
                         uint32_t *indices, const href_layout *indices_layout);

/* Rank-1 or rank-2 axis scan (op SUM or PROD). */
int href_scan_axis(int dtype, int op, int reverse, int exclusive, const void *in,
                   const href_layout *in_layout, uint32_t axis, void *out,
                   const href_layout *out_layout);

/* Fused map-reduction (map: 0 dot, 1 identity-sum, 2 |x| sum, 3 sqrt(sum x^2),
 * 4 max |x|) of same-shape views a and b (b ignored unless map == 0):
 * sequential left fold of map(a_i, b_i) from the reduce identity
 * (hephaestus-cuda application/linalg/norms.rs:55-89, 357-450). */
int href_map_reduce(int dtype, int map, const void *a, const href_layout *la, const void *b,
                    const href_layout *lb, void *out);

/* SplitMix64 (Steele, Lea & Flood 2014) counter stream:
 * h(seed, i) = splitmix64_mix(seed * 2^32 XOR i). */
uint64_t href_hash(uint64_t seed, uint64_t index);

/* Synthetic generators (kind: see HREF_GEN_*), elements index_base..+count. */
enum {
    HREF_GEN_F32_UNIFORM_PM1 = 0, /* -1 + 2*((h>>40)*2^-24)          */
    HREF_GEN_U32_LOW4 = 1,        /* h & 15                          */
    HREF_GEN_F32_NORMAL = 2,      /* Box-Muller in f64, rounded      */
    HREF_GEN_F64_UNIT = 3,        /* (h>>11)*2^-53                   */
    HREF_GEN_I32_PM1000 = 4       /* (h mod 2001) - 1000             */
};
void href_generate(int kind, uint64_t seed, uint64_t index_base, uint64_t count, void *out);

/* --- CPU baseline variants (OpenMP over `threads`, 0 = all cores). ---
 * Integer results are identical to the sequential folds; float sums are
 * chunked (within tolerance). */
int href_max_threads(void);
void href_exclusive_scan_u32_mt(const uint32_t *in, uint32_t *out, uint64_t n, uint32_t carry,
                                int threads);
void href_inclusive_scan_i32_mt(const int32_t *in, int32_t *out, uint64_t n, int32_t carry,
                                int threads);
int64_t href_sum_i32_to_i64_mt(const int32_t *in, uint64_t n, int threads);
float href_sum_f32_mt(const float *in, uint64_t n, int threads);
void href_row_argmax_f32_mt(const float *in, uint64_t rows, uint64_t cols, float *values,
                            uint32_t *indices, int threads);
void href_col_sum_f64_mt(const double *in, uint64_t rows, uint64_t cols, double *out,
                         int threads);

#ifdef __cplusplus
}
#endif

#endif
