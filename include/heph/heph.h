/*
 * heph.h — C ABI of the B200-native (sm_100a) reduce/scan path.
 *
 * This library is a drop-in for the reduce/scan hot path of hephaestus
 * (github.com/ryancinsight/hephaestus, workspace 0.19.0): the seams
 * `ComputeDevice`, `FullReductionOps`, `AxisReductionOps` and `ScanOps`
 * together with the `HephaestusError` vocabulary.  Every entry point below
 * names the reference interface it replaces as `path:line` within that
 * project.  A Rust backend crate binds these symbols 1:1 through an
 * `extern "C"` block of the same names and argument types.
 *
 * Conventions
 *  - Every fallible call returns a heph_status.  On failure a thread-local
 *    message (the reference's wording where the reference has one) is
 *    available from heph_last_error().
 *  - A call that fails validation writes nothing to any output buffer.
 *  - Compute entry points are asynchronous and stream-ordered.  A NULL
 *    heph_stream means the device's own stream.  Transfers (upload, download,
 *    write) are synchronous, as the reference's are.
 *  - Extensions beyond the reference's vocabulary are marked [EXT]: f64/i64
 *    element types, 64-bit extents and offsets, the i32->i64 / f32->f64
 *    widening accumulator, exclusive scans, arg-reductions and the
 *    partitioned multi-GPU drivers.
 */
#ifndef HEPH_HEPH_H
#define HEPH_HEPH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* HephaestusError — crates/hephaestus-core/src/domain/error.rs:8-58.
 * HEPH_OK has no counterpart (it is Rust's Ok(())). */
typedef enum heph_status {
    HEPH_OK = 0,
    HEPH_ADAPTER_UNAVAILABLE = 1,    /* AdapterUnavailable   error.rs:10  */
    HEPH_DEVICE_UNAVAILABLE = 2,     /* DeviceUnavailable    error.rs:16  */
    HEPH_ALLOCATION_FAILED = 3,      /* AllocationFailed     error.rs:23  */
    HEPH_LENGTH_MISMATCH = 4,        /* LengthMismatch       error.rs:29  */
    HEPH_DISPATCH_FAILED = 5,        /* DispatchFailed       error.rs:37  */
    HEPH_INVALID_CONFIGURATION = 6,  /* InvalidConfiguration error.rs:44  */
    HEPH_TRANSFER_FAILED = 7         /* TransferFailed       error.rs:50  */
} heph_status;

/* Element types: the reference's `Pod` scalars with reduction identities
 * (f32/u32/i32, crates/hephaestus-core/src/domain/ops.rs:926-984) plus
 * f64 and i64 [EXT]. */
typedef enum heph_dtype {
    HEPH_F32 = 0,
    HEPH_F64 = 1, /* [EXT] */
    HEPH_U32 = 2,
    HEPH_I32 = 3,
    HEPH_I64 = 4  /* [EXT] */
} heph_dtype;

/* Combining operators — SumOp/ProdOp/MinOp/MaxOp markers
 * (crates/hephaestus-core/src/domain/ops.rs:736-804).  HEPH_MEAN is the
 * `mean_axis_into` form (reduction.rs:143).  Scans take HEPH_SUM (CumSumOp)
 * or HEPH_PROD (CumProdOp). */
typedef enum heph_op {
    HEPH_SUM = 0,
    HEPH_PROD = 1,
    HEPH_MIN = 2,
    HEPH_MAX = 3,
    HEPH_MEAN = 4
} heph_op;

/* Map of a fused map-reduction — the MapReductionOp markers of
 * hephaestus-cuda application/linalg/norms.rs:55-89: DotMap (lhs*rhs, sum),
 * IdentityMap (lhs, sum; trace over a diagonal view), AbsMap (|lhs|, sum; L1),
 * SquareMap (lhs*lhs, sum, then sqrt; L2), MaxAbsMap (|lhs|, max; max norm). */
typedef enum heph_map {
    HEPH_MAP_DOT = 0,
    HEPH_MAP_SUM = 1,
    HEPH_MAP_NORM_L1 = 2,
    HEPH_MAP_NORM_L2 = 3,
    HEPH_MAP_NORM_MAX = 4
} heph_map;

/* ScanDirection — crates/hephaestus-core/src/domain/scan.rs:38. */
typedef enum heph_scan_direction {
    HEPH_FORWARD = 0,
    HEPH_REVERSE = 1
} heph_scan_direction;

#define HEPH_MAX_RANK 4

/* A strided view's layout: leto::Layout<N> (shape, element strides, element
 * offset) as carried by StridedView (crates/hephaestus-core/src/domain/view.rs:27).
 * 64-bit extents, strides and offset [EXT]; the reference narrows them to
 * u32/i32 (crates/hephaestus-core/src/domain/planning.rs:17-28). */
typedef struct heph_layout {
    uint32_t rank;
    uint32_t _pad;
    uint64_t shape[HEPH_MAX_RANK];
    int64_t strides[HEPH_MAX_RANK];
    uint64_t offset;
} heph_layout;

typedef struct heph_device heph_device;     /* CudaDevice  (hephaestus-cuda infrastructure/device.rs:91) */
typedef struct heph_buffer heph_buffer;     /* CudaBuffer<T> (hephaestus-cuda infrastructure/buffer.rs:22) */
typedef struct heph_prepared heph_prepared; /* Prepared<'op> handles of the three seams */
typedef struct heph_comm heph_comm;         /* [EXT] NCCL communicator of a partitioned job */
typedef void *heph_stream;                  /* a cudaStream_t; NULL = the device's stream */

/* ---------------------------------------------------------------- errors */

/* Thread-local message of the last failed call on this thread ("" if none). */
const char *heph_last_error(void);
/* Display prefix of each HephaestusError variant, e.g. "kernel dispatch failed". */
const char *heph_status_name(heph_status status);
/* sizeof the element type, 0 for an unknown value. */
size_t heph_dtype_size(heph_dtype dtype);
/* Library version string. */
const char *heph_version(void);

/* ----------------------------------------- device — ComputeDevice seam */

/* Number of CUDA devices visible (0 when no driver / no GPU; never fails). */
heph_status heph_device_count(int *out_count);
/* CudaDevice::try_with_ordinal — hephaestus-cuda infrastructure/device.rs:145-204.
 * Creates the device's stream and stream-ordered pool and runs the same
 * one-element round trip sanity check.  AdapterUnavailable without a GPU. */
heph_status heph_device_open(int ordinal, heph_device **out);
heph_status heph_device_close(heph_device *device);
/* ComputeDevice::backend_name — core device.rs:94.  Returns "cuda-sm100a". */
const char *heph_device_backend_name(const heph_device *device);
/* ComputeDevice::synchronize — core device.rs:223.  Waits for the device
 * stream and reports a device-side failure (e.g. a bounded look-back wait
 * that ran out) as DispatchFailed. */
heph_status heph_device_synchronize(heph_device *device);
/* Self-test of the failure path of the bounded device waits (no counterpart
 * in the reference): enqueues the look-back wait (which = 0) or the
 * staged-part mbarrier wait (which = 1) against a partner that never
 * arrives.  The wait gives up after its bound (about a second for the
 * look-back, two seconds for the mbarrier), raises the device error bit and
 * returns; the next synchronize reports DispatchFailed and the device stays
 * usable.  No GPU fault is involved. */
heph_status heph_selftest_wait_timeout(heph_device *device, int which, heph_stream stream);
/* Waits for `stream` and reports device-side failures like synchronize. */
heph_status heph_stream_synchronize(heph_device *device, heph_stream stream);
/* The device's own stream (a cudaStream_t). */
heph_status heph_device_stream(heph_device *device, heph_stream *out);
heph_status heph_device_ordinal(const heph_device *device, int *out);
/* Streaming-multiprocessor count (148 on B200). */
heph_status heph_device_sm_count(const heph_device *device, int *out);

/* ---------------------------------------- buffers — DeviceBuffer<T> seam */

/* alloc_zeroed_with_hint / alloc_uninitialized_with_hint — core device.rs:104,116.
 * Memory comes from the device's stream-ordered pool. */
heph_status heph_buffer_alloc(heph_device *device, heph_dtype dtype, uint64_t len,
                              int zeroed, heph_buffer **out);
/* upload_with_hint — core device.rs:135 (allocate + host->device copy). */
heph_status heph_buffer_upload(heph_device *device, heph_dtype dtype, const void *host,
                               uint64_t len, heph_buffer **out);
/* download — core device.rs:147.  LengthMismatch unless host_len == len(buffer). */
heph_status heph_buffer_download(heph_device *device, const heph_buffer *buffer,
                                 void *host, uint64_t host_len);
/* download_sub_buffer — hephaestus-cuda infrastructure/device.rs:349. */
heph_status heph_buffer_download_sub(heph_device *device, const heph_buffer *buffer,
                                     uint64_t offset, void *host, uint64_t count);
/* write_buffer — core device.rs:181.  LengthMismatch unless lengths agree. */
heph_status heph_buffer_write(heph_device *device, heph_buffer *buffer, const void *host,
                              uint64_t host_len);
/* write_sub_buffer — core device.rs:187. */
heph_status heph_buffer_write_sub(heph_device *device, heph_buffer *buffer, uint64_t offset,
                                  const void *host, uint64_t count);
/* copy_buffer — core device.rs:206 (device-to-device, complete on return). */
heph_status heph_buffer_copy(heph_device *device, const heph_buffer *src, heph_buffer *dst);
/* Drop for CudaBuffer — hephaestus-cuda infrastructure/buffer.rs:82-97. */
heph_status heph_buffer_free(heph_buffer *buffer);
uint64_t heph_buffer_len(const heph_buffer *buffer);
heph_dtype heph_buffer_dtype(const heph_buffer *buffer);
/* Raw device address (DeviceApi::device_ptr — core accelerator/device_api.rs:96). */
void *heph_buffer_device_ptr(const heph_buffer *buffer);
/* Wrap caller-owned device memory (not freed by heph_buffer_free). [EXT] */
heph_status heph_buffer_wrap(heph_device *device, heph_dtype dtype, void *device_ptr,
                             uint64_t len, heph_buffer **out);

/* [EXT] Asynchronous stream-ordered transfers for pinned host memory. */
heph_status heph_buffer_upload_async(heph_device *device, heph_buffer *buffer, uint64_t offset,
                                     const void *host, uint64_t count, heph_stream stream);
heph_status heph_buffer_download_async(heph_device *device, const heph_buffer *buffer,
                                       uint64_t offset, void *host, uint64_t count,
                                       heph_stream stream);
heph_status heph_host_alloc_pinned(uint64_t bytes, void **out);
heph_status heph_host_free_pinned(void *ptr);

/* ------------------------------------------------ host-only planners */

/* validate_reduction_width — core reduction.rs:339.  Message:
 * "reduction block width {w} must be a power of two". */
heph_status heph_validate_reduction_width(uint32_t width);
/* The scan planner's width check — core scan.rs:98-102.  Message:
 * "scan block width {w} must be a power of two". */
heph_status heph_validate_scan_width(uint32_t width);
/* reduction_pass_count — core reduction.rs:356 (tree depth of the
 * reference's multi-pass plan; kept for contract tests). */
uint64_t heph_reduction_pass_count(uint64_t len, uint32_t width);

/* Layout::validate_storage_len / checked_size semantics (leto).  Failure is
 * DispatchFailed with the prefix "layout rejected:"
 * (core planning.rs:10-14). */
heph_status heph_layout_validate(const heph_layout *layout, uint64_t buffer_len);

/* Validation half of plan_axis_reduction — core reduction.rs:410-500 — with
 * 64-bit extents.  Sets *out_noop = 1 when the output is empty. */
heph_status heph_plan_axis_reduction(const heph_layout *input, uint64_t input_len,
                                     const heph_layout *output, uint64_t output_len,
                                     uint32_t axis, int buffers_alias, int *out_noop);
/* Validation half of plan_axis_scan — core scan.rs:87-178 — with 64-bit
 * extents.  Rank 2 as in the reference; [EXT] rank 1 (a single line) is also
 * accepted; every other rank is rejected with the reference's message
 * "cuda-sm100a scan supports rank 2 only, got rank N"
 * (core accelerator/scan.rs:519-523).  Sets *out_noop = 1 when empty. */
heph_status heph_plan_axis_scan(const heph_layout *input, uint64_t input_len,
                                const heph_layout *output, uint64_t output_len,
                                uint32_t axis, int buffers_alias, int *out_noop);
/* Validation of prepare_reduce_full — hephaestus-cuda
 * application/full_reduction_seam.rs:59-72. */
heph_status heph_plan_full_reduction(const heph_layout *input, uint64_t input_len,
                                     const heph_layout *output, uint64_t output_len);

/* -------------------------------------------- FullReductionOps seam */

/* FullReductionOps::reduce_full_into — core reduction.rs:267; CUDA
 * full_reduction_seam.rs:49-114.  `out` must view exactly one element.
 * Element type of `out` may differ from `in` only as a widening
 * accumulator [EXT]: I32->I64, F32->F64.  op: SUM, PROD, MIN, MAX
 * (an empty input writes the identity, ops.rs:926-984). */
heph_status heph_reduce_full(heph_device *device, heph_op op,
                             const heph_buffer *in, const heph_layout *in_layout,
                             heph_buffer *out, const heph_layout *out_layout,
                             heph_stream stream);

/* -------------------------------------------- AxisReductionOps seam */

/* AxisReductionOps::reduce_axis_into / prod_axis_into / mean_axis_into /
 * min_axis_into / max_axis_into — core reduction.rs:74-223; CUDA
 * application/reduction.rs:333-575.  Rank-2 keepdims reduction along `axis`.
 * min/max/mean reject an empty reduced axis with
 * "{op}_axis is undefined for empty axis {axis}". */
heph_status heph_reduce_axis(heph_device *device, heph_op op,
                             const heph_buffer *in, const heph_layout *in_layout, uint32_t axis,
                             heph_buffer *out, const heph_layout *out_layout,
                             heph_stream stream);

/* [EXT] Arg-reduction along `axis`: `values` receives the max (op=HEPH_MAX)
 * or min (op=HEPH_MIN) like heph_reduce_axis, `indices` (a U32 buffer with
 * the same keepdims layout) receives the position along `axis` of that
 * value; among equal values the lowest position wins.  No reference
 * counterpart (hephaestus has no argmax); output conventions follow
 * max_axis_into (core reduction.rs:186). */
heph_status heph_arg_reduce_axis(heph_device *device, heph_op op,
                                 const heph_buffer *in, const heph_layout *in_layout,
                                 uint32_t axis,
                                 heph_buffer *values, const heph_layout *values_layout,
                                 heph_buffer *indices, const heph_layout *indices_layout,
                                 heph_stream stream);

/* ------------------------------------------ fused map-reductions (vector) */

/* dot / trace / norm_l1 / norm_l2 / norm_max — hephaestus-cuda
 * application/linalg/norms.rs:357-450, DenseVectorOps::dot/norm_l1/norm_l2/
 * norm_max (crates/hephaestus-core/src/domain/vector.rs:57-229).  `a` (and
 * `b` for HEPH_MAP_DOT, NULL otherwise) are strided views of the same shape
 * (rank <= 4); `out` views one element of the same element type.  The map is
 * fused into a single-launch reduction; HEPH_MAP_NORM_L2 needs f32/f64.
 * Shape mismatch: "dot product shape mismatch: lhs [..], rhs [..]". */
heph_status heph_map_reduce_full(heph_device *device, heph_map map,
                                 const heph_buffer *a, const heph_layout *a_layout,
                                 const heph_buffer *b, const heph_layout *b_layout,
                                 heph_buffer *out, const heph_layout *out_layout,
                                 heph_stream stream);
/* prepare_dot / prepare_norm_l2 — hephaestus-cuda application/prepared_map_reduction.rs
 * (any map here); dispatched with heph_dispatch_prepared, batchable. */
heph_status heph_prepare_map_reduce_full(heph_device *device, heph_map map,
                                         const heph_buffer *a, const heph_layout *a_layout,
                                         const heph_buffer *b, const heph_layout *b_layout,
                                         heph_buffer *out, const heph_layout *out_layout,
                                         heph_prepared **out_prepared);

/* -------------------------------------------------------- ScanOps seam */

/* ScanOps::scan_axis_into — core scan.rs:219; AxisScanOps
 * accelerator/scan.rs:492-572.  op: HEPH_SUM (CumSumOp) or HEPH_PROD
 * (CumProdOp).  Inclusive unless `exclusive` [EXT].  Rank 2 (as the
 * reference) or rank 1 [EXT]. */
heph_status heph_scan_axis(heph_device *device, heph_op op, heph_scan_direction direction,
                           int exclusive,
                           const heph_buffer *in, const heph_layout *in_layout, uint32_t axis,
                           heph_buffer *out, const heph_layout *out_layout,
                           heph_stream stream);

/* ------------------------------------------------ prepared (rebind) forms */

/* prepare_reduce_full — core reduction.rs:287. */
heph_status heph_prepare_reduce_full(heph_device *device, heph_op op,
                                     const heph_buffer *in, const heph_layout *in_layout,
                                     heph_buffer *out, const heph_layout *out_layout,
                                     heph_prepared **out_prepared);
/* prepare_reduce_axis_into — core reduction.rs:202. */
heph_status heph_prepare_reduce_axis(heph_device *device, heph_op op,
                                     const heph_buffer *in, const heph_layout *in_layout,
                                     uint32_t axis,
                                     heph_buffer *out, const heph_layout *out_layout,
                                     heph_prepared **out_prepared);
/* prepare_scan_axis — core scan.rs:237. */
heph_status heph_prepare_scan_axis(heph_device *device, heph_op op,
                                   heph_scan_direction direction, int exclusive,
                                   const heph_buffer *in, const heph_layout *in_layout,
                                   uint32_t axis,
                                   heph_buffer *out, const heph_layout *out_layout,
                                   heph_prepared **out_prepared);
/* dispatch_full / dispatch_prepared / dispatch_scan — core reduction.rs:222,
 * :305, scan.rs:259.  Re-reads the bound buffers: later writes are observed. */
heph_status heph_dispatch_prepared(heph_device *device, const heph_prepared *prepared,
                                   heph_stream stream);
heph_status heph_prepared_free(heph_prepared *prepared);

/* Batch submission — submit_prepared_reduction_batch (hephaestus-cuda
 * application/prepared_reduction.rs:165) and submit_prepared_axis_reduction_batch
 * (prepared_axis_reduction.rs:84): a fixed list of prepared full / axis
 * reductions recorded once as a CUDA graph and replayed with one launch per
 * heph_batch_launch.  Consecutive dense full reductions of one operator and
 * element type whose outputs overlap none of the run's inputs or other
 * outputs are fused into one kernel (same results as running them in order).
 * Creation dispatches every item once (setting up the workspace the graph
 * uses).  Replays of one batch must not overlap on the GPU.
 * Prepared scans are rejected (InvalidConfiguration). */
typedef struct heph_batch heph_batch;
heph_status heph_batch_create(heph_device *device, const heph_prepared *const *items, uint32_t count,
                              heph_batch **out);
heph_status heph_batch_launch(heph_batch *batch, heph_stream stream);
heph_status heph_batch_free(heph_batch *batch);

/* ---------------------------------- [EXT] partitioned 1-D multi-GPU path */

/* One process per GPU.  Rank 0 creates the id, the caller ships it to the
 * other ranks (e.g. over a torch.distributed store), every rank calls
 * heph_comm_init.  NCCL is loaded at run time (libnccl.so.2). */
#define HEPH_COMM_ID_BYTES 128
heph_status heph_comm_unique_id(uint8_t id[HEPH_COMM_ID_BYTES]);
heph_status heph_comm_init(heph_device *device, const uint8_t id[HEPH_COMM_ID_BYTES],
                           int nranks, int rank, heph_comm **out);
heph_status heph_comm_destroy(heph_comm *comm);
/* Aborts in-flight NCCL work (failure path: a peer is gone). */
heph_status heph_comm_abort(heph_comm *comm);
/* [EXT] *out = 1 when the partitioned calls exchange the ranks' totals /
 * partials over peer memory (every rank mapped every other
 * rank's mailbox through CUDA IPC at heph_comm_init; one kernel stores and
 * waits, bounded by a 2 s device deadline that reports DispatchFailed
 * "exchange timeout…"), 0 when it uses ncclAllGather (mapping failed on some
 * rank, more than 32 ranks, or HEPH_DIST_EXCHANGE=nccl).  All ranks agree. */
heph_status heph_comm_peer_exchange(const heph_comm *comm, int *out);

/* [EXT] Host-side deadline on a partitioned call: waits until `stream` (NULL
 * = the device's stream) has finished the work queued on it, polling NCCL's
 * asynchronous error (ncclCommGetAsyncError) meanwhile.  When NCCL reports an
 * error, or `timeout_ms` passes first (a peer rank died or never arrived),
 * the communicator is aborted (ncclCommAbort: its kernels exit) and
 * DispatchFailed is returned with the reason; the communicator then only
 * accepts heph_comm_destroy.  The reference has no multi-GPU path and no
 * counterpart. */
heph_status heph_comm_wait(heph_comm *comm, heph_stream stream, uint32_t timeout_ms);

/* [EXT] Runs the wait policy of heph_comm_wait against scripted fakes, with
 * no GPU and no NCCL (0: the stream completes; 1: NCCL reports an error;
 * 2: the deadline passes; 3: the stream fails); *out_aborted = how many
 * times the policy aborted the fake communicator.  For tests and health
 * checks; no counterpart in the reference. */
heph_status heph_selftest_comm_wait_policy(int scenario, uint32_t timeout_ms, int *out_aborted);

/* Each rank holds one contiguous slice of a global 1-D buffer (rank order =
 * slice order).  `out` (one element, dtype may widen I32->I64 / F32->F64)
 * receives the reduction of the WHOLE global buffer on every rank: local
 * single-pass reduction, then the exchange of the per-rank partials (over
 * peer memory, or one NCCL all-gather: heph_comm_peer_exchange), then a
 * fixed-order combine on the device.  op: SUM, PROD, MIN, MAX. */
heph_status heph_partitioned_reduce_full(heph_comm *comm, heph_op op,
                                         const heph_buffer *in, const heph_layout *in_layout,
                                         heph_buffer *out, const heph_layout *out_layout,
                                         heph_stream stream);
/* Forward scan of the global buffer: each rank writes its slice of the
 * global (inclusive or exclusive) prefix.  Reduce-then-scan: local total,
 * exchange of the totals (peer memory or NCCL all-gather), carry = fold of
 * the lower ranks' totals, then the slice's scan seeded with that carry. */
heph_status heph_partitioned_scan(heph_comm *comm, heph_op op, int exclusive,
                                  const heph_buffer *in, const heph_layout *in_layout,
                                  heph_buffer *out, const heph_layout *out_layout,
                                  heph_stream stream);
/* heph_partitioned_scan and heph_partitioned_reduce_full of the SAME global
 * buffer in one call (no counterpart in the reference): one local pass
 * computes the slice's scan total (scan_op: SUM, PROD) and its reduction
 * partial (reduce_op: SUM, PROD, MIN, MAX; reduce_out may widen I32->I64 /
 * F32->F64), one exchange carries both, then the seeded scan.  Each rank
 * reads its slice twice and writes it once - the traffic of the same pair of
 * calls on one GPU - instead of three reads.  Outputs must not alias the
 * input. */
heph_status heph_partitioned_scan_reduce(heph_comm *comm, heph_op scan_op, int exclusive,
                                         const heph_buffer *in, const heph_layout *in_layout,
                                         heph_buffer *scan_out, const heph_layout *scan_layout,
                                         heph_op reduce_op, heph_buffer *reduce_out,
                                         const heph_layout *reduce_layout, heph_stream stream);

/* ------------------------------------------ [EXT] seeded scan building block */

/* Single-pass forward scan of a contiguous rank-1 view whose first element is
 * preceded by the carry stored in `carry` (one element of the same dtype,
 * device memory).  This is the local step of the partitioned scan. */
heph_status heph_scan_seeded(heph_device *device, heph_op op, int exclusive,
                             const heph_buffer *in, const heph_layout *in_layout,
                             heph_buffer *out, const heph_layout *out_layout,
                             const heph_buffer *carry, uint64_t carry_offset,
                             heph_stream stream);

/* ------------------------------------------- [EXT] host-buffer scan pipeline */

/* Forward scan (op SUM/PROD, inclusive or exclusive) of `count` contiguous
 * elements in HOST memory into host memory — the composition upload ->
 * scan_axis_into -> download of the reference (core device.rs:135, scan.rs:219,
 * device.rs:147) with the three phases overlapped: chunks of `chunk_elems`
 * (0 = 64 MiB worth) flow through three device slots, host->device copies,
 * seeded device scans and device->host copies running concurrently on two
 * copy engines and the device's stream.  Returns when host_out is complete.
 * Staging comes from the device's stream-ordered pool.  Pinned host memory
 * (heph_host_alloc_pinned) is needed for the copies to overlap. */
heph_status heph_scan_host(heph_device *device, heph_op op, int exclusive, heph_dtype dtype,
                           const void *host_in, void *host_out, uint64_t count, uint64_t chunk_elems);

/* [EXT] heph_scan_host plus a full reduction of the same host input (the
 * scan + sum pair of the partitioned 1-D case on one device): every chunk is
 * also reduced on the device while it is staged, the chunks' results folded
 * in order, and the single result (acc_dtype: the input type or its widening
 * I32->I64 / F32->F64; op SUM/PROD/MIN/MAX; the identity when count == 0)
 * written to *host_reduce_out.  Replaces upload + ScanOps::scan_axis_into +
 * FullReductionOps::reduce_full_into + download (core scan.rs:219,
 * reduction.rs:243, device.rs:135,147) for host data. */
heph_status heph_scan_reduce_host(heph_device *device, heph_op scan_op, int exclusive, heph_dtype dtype,
                                  const void *host_in, void *host_out, uint64_t count, heph_op reduce_op,
                                  heph_dtype acc_dtype, void *host_reduce_out, uint64_t chunk_elems);

/* ------------------------------------------ allocation-free full reduction */

/* No counterpart in the reference: an extra entry point for callers that
 * cannot allocate device memory when they call in (a host that runs inside a
 * fixed memory budget or owns every device buffer itself, or code that must
 * not re-enter an allocator from the call site).  heph_reduce_full may
 * allocate its workspace from the stream-ordered pool on first use per
 * stream; this variant allocates nothing and needs no heph_device.
 *
 * Reduces `count` contiguous elements at the device pointer `in` (dtype
 * in_dtype, current CUDA device) into the single element `*out` (out_dtype ==
 * in_dtype, or the widening pairs I32->I64, F32->F64), op SUM/PROD/MIN/MAX,
 * enqueued on `stream` (NULL = the legacy default stream).  Result identical
 * in algorithm to heph_reduce_full on a dense view.
 *
 * Scratch: a static 16 KiB + 256 B device array inside the library (every GPU
 * that loads the library keeps it until the process exits) that holds one
 * partial per CTA for at most 2048 CTAs; a launch that would need more is
 * rejected with HEPH_INVALID_CONFIGURATION.  Every call looks up that
 * array's device address in the calling thread's current context (no
 * allocation), so non-primary driver-API contexts are served too; the first
 * call in a context loads the library's kernels there, so make that first
 * call before any stream capture.  All calls share the one array, so calls whose
 * kernels overlap on the GPU (different streams, or several host threads)
 * race and must be serialised by the caller. */
heph_status heph_reduce_full_noalloc(heph_op op, heph_dtype in_dtype, heph_dtype out_dtype,
                                     const void *in, uint64_t count, void *out, heph_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* HEPH_HEPH_H */
