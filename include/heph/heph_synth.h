/*
 * heph_synth.h — seeded synthetic inputs generated on the device, for tests
 * and benchmarks of the reduce/scan path.  Not part of the reference-facing
 * surface (hephaestus generates inputs through leto on the host,
 * crates/hephaestus-cuda/src/application/random.rs:11-41; leto is not
 * available, so this project defines its own counter-based stream).
 *
 * h(seed, i) = splitmix64(seed * 2^32 XOR i), SplitMix64 of Steele, Lea &
 * Flood (2014).  The integer generators are bit-identical to the host oracle
 * (oracle/host_ref.c, href_generate); the normal generator uses the device's
 * double-precision log/cos and can differ from the host in the last bit.
 */
#ifndef HEPH_HEPH_SYNTH_H
#define HEPH_HEPH_SYNTH_H

#include "heph/heph.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum heph_synth_kind {
    HEPH_SYNTH_F32_UNIFORM_PM1 = 0, /* -1 + 2*((h>>40)*2^-24), exact f32 in [-1,1) */
    HEPH_SYNTH_U32_LOW4 = 1,        /* h & 15                                     */
    HEPH_SYNTH_F32_NORMAL = 2,      /* Box-Muller in f64 from h(2i), h(2i+1)       */
    HEPH_SYNTH_F64_UNIT = 3,        /* (h>>11)*2^-53 in [0,1)                      */
    HEPH_SYNTH_I32_PM1000 = 4       /* (h mod 2001) - 1000                         */
} heph_synth_kind;

/* Fills elements [offset, offset+count) of `buffer` with stream elements
 * index_base .. index_base+count-1. */
heph_status heph_synth_fill(heph_device *device, heph_buffer *buffer, uint64_t offset,
                            uint64_t count, heph_synth_kind kind, uint64_t seed,
                            uint64_t index_base, heph_stream stream);

/* Injects exact ties into a row-major f32 [rows x cols] matrix: a row with
 * h(seed, 2^32+row) % 100 == 0 gets x[row][j] = max(row) at
 * j = h(seed, 2^33+row) % cols (or (j+1) % cols when j is the row's first
 * argmax), so its expected argmax is min(j, first argmax). */
heph_status heph_synth_inject_row_ties(heph_device *device, heph_buffer *matrix, uint64_t rows,
                                       uint64_t cols, uint64_t seed, heph_stream stream);

#ifdef __cplusplus
}
#endif

#endif
