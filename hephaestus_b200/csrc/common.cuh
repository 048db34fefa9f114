// common.cuh — shared definitions of the sm_100a reduce/scan library:
// error plumbing, element-type traits, combine operators and their
// identities, the device / buffer / workspace objects behind the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cfloat>
#include <climits>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <type_traits>

#include "heph/heph.h"

namespace heph {

// ------------------------------------------------------------------ errors

void set_last_error(const std::string &msg);
heph_status fail(heph_status status, const std::string &msg);
heph_status cuda_fail(heph_status status, cudaError_t err, const char *what);

#define HEPH_CUDA_TRY(expr, status, what)                                   \
    do {                                                                    \
        cudaError_t heph_err_ = (expr);                                     \
        if (heph_err_ != cudaSuccess) return ::heph::cuda_fail(status, heph_err_, what); \
    } while (0)

// Bit-level reinterpretation between equally sized trivially copyable types.
template <typename To, typename From> __host__ __device__ __forceinline__ To bitcast(const From &f) {
    static_assert(sizeof(To) == sizeof(From), "bitcast between types of different size");
    To t;
    memcpy(&t, &f, sizeof(To));
    return t;
}

// ------------------------------------------------------------- operators

enum Op : int { OP_SUM = 0, OP_PROD = 1, OP_MIN = 2, OP_MAX = 3 };

// Identities of crates/hephaestus-core/src/domain/ops.rs:926-984 (f32, u32,
// i32); f64 and i64 take the analogous extremes.
template <typename T> struct Limits;
template <> struct Limits<float> {
    static constexpr float lowest() { return -FLT_MAX; }
    static constexpr float highest() { return FLT_MAX; }
};
template <> struct Limits<double> {
    static constexpr double lowest() { return -DBL_MAX; }
    static constexpr double highest() { return DBL_MAX; }
};
template <> struct Limits<uint32_t> {
    static constexpr uint32_t lowest() { return 0u; }
    static constexpr uint32_t highest() { return UINT32_MAX; }
};
template <> struct Limits<int32_t> {
    static constexpr int32_t lowest() { return INT32_MIN; }
    static constexpr int32_t highest() { return INT32_MAX; }
};
template <> struct Limits<int64_t> {
    static constexpr int64_t lowest() { return INT64_MIN; }
    static constexpr int64_t highest() { return INT64_MAX; }
};

template <typename T> struct Unsigned { using type = T; };
template <> struct Unsigned<int32_t> { using type = uint32_t; };
template <> struct Unsigned<int64_t> { using type = uint64_t; };

template <typename T> constexpr bool is_float_v = false;
template <> constexpr bool is_float_v<float> = true;
template <> constexpr bool is_float_v<double> = true;

template <typename T, int OP> __host__ __device__ __forceinline__ T identity() {
    if constexpr (OP == OP_PROD) return T(1);
    else if constexpr (OP == OP_MIN) return Limits<T>::highest();
    else if constexpr (OP == OP_MAX) return Limits<T>::lowest();
    else return T(0);
}

// Combine expressions of the CUDA dialect (lhs = accumulator, rhs = element):
// "lhs + rhs", "lhs * rhs", min(a,b) = a<b?a:b, max(a,b) = a>b?a:b
// (hephaestus-cuda application/reduction.rs:24-25, core ops.rs:912-919).
// Integer arithmetic wraps (two's complement), computed in the unsigned type.
template <typename T, int OP> __host__ __device__ __forceinline__ T combine(T lhs, T rhs) {
    if constexpr (OP == OP_SUM) {
        if constexpr (is_float_v<T>) return lhs + rhs;
        else {
            using U = typename Unsigned<T>::type;
            return T(U(lhs) + U(rhs));
        }
    } else if constexpr (OP == OP_PROD) {
        if constexpr (is_float_v<T>) return lhs * rhs;
        else {
            using U = typename Unsigned<T>::type;
            return T(U(lhs) * U(rhs));
        }
    } else if constexpr (OP == OP_MIN) {
        return (lhs < rhs) ? lhs : rhs;
    } else {
        return (lhs > rhs) ? lhs : rhs;
    }
}

// ------------------------------------------------------------ dtype maps

template <typename T> struct DtypeOf;
template <> struct DtypeOf<float> { static constexpr heph_dtype value = HEPH_F32; };
template <> struct DtypeOf<double> { static constexpr heph_dtype value = HEPH_F64; };
template <> struct DtypeOf<uint32_t> { static constexpr heph_dtype value = HEPH_U32; };
template <> struct DtypeOf<int32_t> { static constexpr heph_dtype value = HEPH_I32; };
template <> struct DtypeOf<int64_t> { static constexpr heph_dtype value = HEPH_I64; };

size_t dtype_size(heph_dtype dt);
bool dtype_valid(heph_dtype dt);

// Calls F.template operator()<T>() with the C++ type of `dt`.
template <typename F> heph_status dispatch_dtype(heph_dtype dt, F &&f) {
    switch (dt) {
        case HEPH_F32: return f.template operator()<float>();
        case HEPH_F64: return f.template operator()<double>();
        case HEPH_U32: return f.template operator()<uint32_t>();
        case HEPH_I32: return f.template operator()<int32_t>();
        case HEPH_I64: return f.template operator()<int64_t>();
    }
    return fail(HEPH_INVALID_CONFIGURATION, "unknown element type");
}

// ---------------------------------------------------------- device state

// Per-(device, stream) scratch: reduction partials and the decoupled
// look-back tile status.  Kernels on one stream run in order, so one
// workspace per stream is never used by two kernels at once.
struct Workspace {
    cudaStream_t stream = nullptr;
    void *partials = nullptr;  // per-CTA / per-split partial results
    size_t partials_bytes = 0;
    unsigned int *tickets = nullptr;  // last-block tickets, zero at rest
    static constexpr int kTickets = 64;
    // Look-back status: flags (epoch-tagged) + aggregate / inclusive values.
    void *scan_status = nullptr;
    size_t scan_status_bytes = 0;
    unsigned long long *tile_counter = nullptr;  // reserved; zero at rest
    uint32_t epoch = 0;                           // tags this call's flags
    void *small = nullptr;                        // 256 bytes of per-call scalars
};

struct Device {
    int ordinal = 0;
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    cudaMemPool_t pool = nullptr;
    // Device-side failure word in mapped pinned host memory: kernels set it
    // when a bounded wait runs out; synchronize reports and clears it.
    unsigned int *error_host = nullptr;
    unsigned int *error_dev = nullptr;
    std::mutex mu;
    std::map<cudaStream_t, Workspace *> workspaces;
};

struct Buffer {
    Device *device = nullptr;
    heph_dtype dtype = HEPH_F32;
    uint64_t len = 0;
    void *ptr = nullptr;
    bool owned = true;
};

// Makes `device` current on the calling thread.
heph_status bind(Device *device);
cudaStream_t resolve_stream(Device *device, heph_stream stream);
// Workspace of `stream`, grown so that partials >= partial_bytes and the scan
// status holds >= scan_tiles tiles of `status_stride` bytes.  Caller holds mu.
heph_status workspace_for(Device *device, cudaStream_t stream, size_t partial_bytes,
                          size_t scan_status_bytes, Workspace **out);

// Device-side error codes written to Device::error_dev.
enum DeviceError : unsigned int { DEVERR_LOOKBACK_TIMEOUT = 1u, DEVERR_BULK_TIMEOUT = 2u, DEVERR_EXCHANGE_TIMEOUT = 4u };

}  // namespace heph

// The opaque C ABI handles are the device and buffer objects themselves.
struct heph_device : heph::Device {};
struct heph_buffer : heph::Buffer {};
