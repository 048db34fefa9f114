// dist.cu — partitioned 1-D reduce and scan across the GPUs of one node, one
// process per GPU, NCCL over NVLink/NVSwitch for the exchange.
//
// The reference has no multi-device path (hephaestus-cuda opens independent
// contexts per ordinal, infrastructure/device.rs:657-672).  The exchange here
// is a few bytes per rank, so the whole call stays stream-ordered with no host
// synchronisation:
//   reduce: local single-pass reduction -> ncclAllGather of the per-rank
//           partials -> one thread folds them in rank order into `out`;
//   scan:   local reduction of the slice (its total) -> ncclAllGather of the
//           totals -> carry = fold of the lower ranks' totals -> look-back
//           scan of the slice seeded with the carry.
//   scan + reduce of the same slice (heph_partitioned_scan_reduce): ONE
//           local pass computes the slice's scan total and its reduction
//           partial, one ncclAllGather carries both (16 bytes per rank), one
//           thread folds the carry and the global reduction, then the seeded
//           scan: every rank moves 3 bytes-units per element, as one GPU does
//           for the same pair, so the pair scales with the rank count.
//           The exchange of this pair runs over peer memory instead of
//           NCCL when every rank could map every other rank's mailbox: ONE
//           32-thread kernel stores the rank's 16-byte pair into each peer's
//           mailbox over NVLink (data, then a release store of the call's
//           epoch as the flag), waits (bounded by the global timer) for every
//           rank's flag in its own mailbox, and folds the carry and the
//           global reduction — one launch in place of ncclAllGather plus the
//           fold kernel.
// NCCL is resolved at run time from the libnccl.so.2 already loaded into the
// process (torch's), else from the loader path, so this library carries no
// link-time NCCL dependency.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "comm_wait.h"
#include "common.cuh"
#include "device_utils.cuh"
#include "kernels.h"
#include "plan.h"

namespace heph {
namespace {

struct NcclApi {
    bool loaded = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char *e = dlerror();
            api.why = std::string("libnccl.so.2 could not be loaded: ") + (e ? e : "unknown");
            return;
        }
        auto sym = [&](const char *name) { return dlsym(h, name); };
        api.GetUniqueId = (decltype(api.GetUniqueId))sym("ncclGetUniqueId");
        api.CommInitRank = (decltype(api.CommInitRank))sym("ncclCommInitRank");
        api.AllGather = (decltype(api.AllGather))sym("ncclAllGather");
        api.AllReduce = (decltype(api.AllReduce))sym("ncclAllReduce");
        api.CommDestroy = (decltype(api.CommDestroy))sym("ncclCommDestroy");
        api.CommAbort = (decltype(api.CommAbort))sym("ncclCommAbort");
        api.CommGetAsyncError = (decltype(api.CommGetAsyncError))sym("ncclCommGetAsyncError");
        api.GetErrorString = (decltype(api.GetErrorString))sym("ncclGetErrorString");
        api.loaded = api.GetUniqueId && api.CommInitRank && api.AllGather && api.AllReduce && api.CommDestroy &&
                     api.CommAbort && api.GetErrorString;
        if (!api.loaded) api.why = "libnccl.so.2 lacks a required symbol";
    });
    return api;
}

heph_status nccl_fail(ncclResult_t r, const char *what) {
    const char *s = nccl().GetErrorString ? nccl().GetErrorString(r) : "unknown";
    return fail(HEPH_DISPATCH_FAILED, std::string(what) + ": " + s);
}

template <typename T, int OP>
__global__ void fold_ranks_kernel(const T *__restrict__ gathered, int count, T *__restrict__ out) {
    T acc = identity<T, OP>();
    for (int r = 0; r < count; ++r) acc = combine<T, OP>(acc, gathered[r]);
    *out = acc;
}

template <typename T>
heph_status launch_fold(cudaStream_t s, int op, const void *g, int count, void *out) {
    const T *tg = static_cast<const T *>(g);
    T *to = static_cast<T *>(out);
    switch (op) {
        case OP_SUM: fold_ranks_kernel<T, OP_SUM><<<1, 1, 0, s>>>(tg, count, to); break;
        case OP_PROD: fold_ranks_kernel<T, OP_PROD><<<1, 1, 0, s>>>(tg, count, to); break;
        case OP_MIN: fold_ranks_kernel<T, OP_MIN><<<1, 1, 0, s>>>(tg, count, to); break;
        case OP_MAX: fold_ranks_kernel<T, OP_MAX><<<1, 1, 0, s>>>(tg, count, to); break;
        default: return fail(HEPH_INVALID_CONFIGURATION, "unknown operator");
    }
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "rank fold launch");
    return HEPH_OK;
}

// carry = op1-fold of the totals of ranks < rank; global = op2-fold of every
// rank's partial; pairs are [T total | pad][Tacc partial | pad], 16 bytes each.
template <typename T, int OP1, typename Tacc, int OP2>
__global__ void fold_pairs_kernel(const unsigned char *__restrict__ pairs, int nranks, int rank, T *__restrict__ carry,
                                  Tacc *__restrict__ global) {
    T c = identity<T, OP1>();
    Tacc g = identity<Tacc, OP2>();
    for (int r = 0; r < nranks; ++r) {
        const T t = *reinterpret_cast<const T *>(pairs + 16 * r);
        const Tacc v = *reinterpret_cast<const Tacc *>(pairs + 16 * r + 8);
        if (r < rank) c = combine<T, OP1>(c, t);
        g = combine<Tacc, OP2>(g, v);
    }
    *carry = c;
    *global = g;
}

template <typename T, int OP1, typename Tacc>
heph_status launch_fold_pairs(cudaStream_t s, int op2, const void *pairs, int nranks, int rank, void *carry,
                              void *global) {
    const unsigned char *pp = static_cast<const unsigned char *>(pairs);
    T *c = static_cast<T *>(carry);
    Tacc *g = static_cast<Tacc *>(global);
    switch (op2) {
        case OP_SUM: fold_pairs_kernel<T, OP1, Tacc, OP_SUM><<<1, 1, 0, s>>>(pp, nranks, rank, c, g); break;
        case OP_PROD: fold_pairs_kernel<T, OP1, Tacc, OP_PROD><<<1, 1, 0, s>>>(pp, nranks, rank, c, g); break;
        case OP_MIN: fold_pairs_kernel<T, OP1, Tacc, OP_MIN><<<1, 1, 0, s>>>(pp, nranks, rank, c, g); break;
        case OP_MAX: fold_pairs_kernel<T, OP1, Tacc, OP_MAX><<<1, 1, 0, s>>>(pp, nranks, rank, c, g); break;
        default: return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
    }
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "rank fold launch");
    return HEPH_OK;
}

// Mailbox of a rank: 2 epoch parities x nranks entries of 32 bytes, entry r
// = [rank r's 16-byte pair][flag: the epoch of the call that wrote it][pad].
// Parity alternates per call, so a fast rank writing call e+1 never
// overwrites an entry a slow rank still has to read for call e (a rank can
// only reach call e+2 after every rank has published call e+1, i.e. after
// every rank finished reading call e).
constexpr int kMailboxEntry = 32;
constexpr int kMaxP2PRanks = 32;

__device__ __forceinline__ void st_relaxed_sys(unsigned char *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(unsigned char *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned char *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned char *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// One warp: lane r (< nranks) publishes this rank's pair into rank r's
// mailbox (the partitioned reduction uses only the partial, the scan only
// the total: the other output pointer is null)
// mailbox, then waits for rank r's pair in this rank's mailbox; lane 0 folds
// carry (lower ranks' totals, OP1) and the global reduction (all partials,
// OP2) in rank order.  A pair that never arrives within the wait deadline
// raises the device error bit and counts as the identity.
template <typename T, int OP1, typename Tacc, int OP2>
__global__ void __launch_bounds__(32) exchange_pairs_kernel(const unsigned char *__restrict__ pair,
                                                            unsigned char *const *__restrict__ boxes,
                                                            unsigned char *mybox, int nranks, int rank,
                                                            unsigned long long epoch, T *__restrict__ carry,
                                                            Tacc *__restrict__ global, unsigned int *err) {
    __shared__ unsigned long long s_pair[kMaxP2PRanks][2];
    const int r = threadIdx.x;
    const size_t par = (size_t)(epoch & 1ull) * nranks;
    if (r < nranks) {
        const unsigned long long a = reinterpret_cast<const unsigned long long *>(pair)[0];
        const unsigned long long b = reinterpret_cast<const unsigned long long *>(pair)[1];
        unsigned char *dst = boxes[r] + (par + rank) * kMailboxEntry;
        st_relaxed_sys(dst, a);
        st_relaxed_sys(dst + 8, b);
        st_release_sys(dst + 16, epoch);
    }
    if (r < nranks) {
        const unsigned char *src = mybox + (par + r) * kMailboxEntry;
        WaitDeadline deadline;
        bool ok = true;
        while (ld_acquire_sys(src + 16) != epoch) {
            if (deadline.expired()) {
                raise_device_error(err, DEVERR_EXCHANGE_TIMEOUT);
                ok = false;
                break;
            }
            __nanosleep(64);
        }
        if (ok) {
            s_pair[r][0] = ld_relaxed_sys(src);
            s_pair[r][1] = ld_relaxed_sys(src + 8);
        } else {
            const T ti = identity<T, OP1>();
            const Tacc ai = identity<Tacc, OP2>();
            s_pair[r][0] = 0;
            s_pair[r][1] = 0;
            memcpy(&s_pair[r][0], &ti, sizeof(T));
            memcpy(&s_pair[r][1], &ai, sizeof(Tacc));
        }
    }
    __syncwarp();
    if (r == 0) {
        T c = identity<T, OP1>();
        Tacc g = identity<Tacc, OP2>();
        for (int q = 0; q < nranks; ++q) {
            T t;
            Tacc v;
            memcpy(&t, &s_pair[q][0], sizeof(T));
            memcpy(&v, &s_pair[q][1], sizeof(Tacc));
            if (q < rank) c = combine<T, OP1>(c, t);
            g = combine<Tacc, OP2>(g, v);
        }
        if (carry) *carry = c;
        if (global) *global = g;
    }
}

template <typename T, int OP1, typename Tacc>
heph_status launch_exchange_pairs(cudaStream_t s, int op2, const void *pair, unsigned char *const *boxes,
                                  unsigned char *mybox, int nranks, int rank, unsigned long long epoch, void *carry,
                                  void *global, unsigned int *err) {
    const unsigned char *pp = static_cast<const unsigned char *>(pair);
    T *c = static_cast<T *>(carry);
    Tacc *g = static_cast<Tacc *>(global);
    switch (op2) {
#define HEPH_X(OP2_) exchange_pairs_kernel<T, OP1, Tacc, OP2_><<<1, 32, 0, s>>>(pp, boxes, mybox, nranks, rank, epoch, c, g, err)
        case OP_SUM: HEPH_X(OP_SUM); break;
        case OP_PROD: HEPH_X(OP_PROD); break;
        case OP_MIN: HEPH_X(OP_MIN); break;
        case OP_MAX: HEPH_X(OP_MAX); break;
#undef HEPH_X
        default: return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
    }
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "pair exchange launch");
    return HEPH_OK;
}

}  // namespace
}  // namespace heph

using namespace heph;

struct heph_comm {
    Device *device = nullptr;
    ncclComm_t nccl = nullptr;
    int nranks = 0, rank = 0;
    // [total: 8 B][carry: 8 B][gathered: 8 B x nranks] then, from pair_off:
    // [pair: 16 B][carry: 16 B][gathered pairs: 16 B x nranks]
    void *scratch = nullptr;
    size_t pair_off = 0;
    bool aborted = false;
    // Peer-memory exchange (all ranks or none): this rank's mailbox, every
    // rank's mailbox as mapped here (device array), the IPC mappings to
    // close, and the epoch of the next call.
    bool p2p = false;
    unsigned char *mailbox = nullptr;
    unsigned char **boxes_dev = nullptr;
    std::vector<void *> opened;
    unsigned long long epoch = 0;
};

namespace {

// Maps every peer's mailbox through CUDA IPC.  Collective: every rank calls it
// and every rank ends with the same p2p decision (all-reduces of the per-rank
// outcome, min), so no rank waits on a mailbox a peer never writes: first
// every rank must have created its mailbox and handle, then every rank must
// have opened every peer's handle.
void setup_p2p(heph_comm *c, cudaStream_t s) {
    NcclApi &api = nccl();
    const int n = c->nranks;
    c->epoch = 1;
    if (n < 2 || n > kMaxP2PRanks) return;  // the same on every rank
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    unsigned char *xfer = nullptr;  // [my handle][all handles][flag]
    if (cudaMalloc(&xfer, hb * (n + 1) + 16) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    int32_t *flag = reinterpret_cast<int32_t *>(xfer + hb * (n + 1));
    auto agree = [&](int mine) {  // min over the ranks; 0 on any failure
        int all = 0;
        if (cudaMemcpy(flag, &mine, sizeof(int32_t), cudaMemcpyHostToDevice) == cudaSuccess &&
            api.AllReduce(flag, flag, 1, ncclInt32, ncclMin, c->nccl, s) == ncclSuccess &&
            cudaStreamSynchronize(s) == cudaSuccess &&
            cudaMemcpy(&all, flag, sizeof(int32_t), cudaMemcpyDeviceToHost) == cudaSuccess)
            return all;
        cudaGetLastError();
        return 0;
    };
    const char *e = getenv("HEPH_DIST_EXCHANGE");
    int ok = !(e && std::string(e) == "nccl");
    const size_t box_bytes = 2 * (size_t)n * kMailboxEntry;
    if (ok) {
        cudaIpcMemHandle_t h;
        ok = cudaMalloc(&c->mailbox, box_bytes) == cudaSuccess && cudaMemset(c->mailbox, 0, box_bytes) == cudaSuccess &&
             cudaMalloc(&c->boxes_dev, sizeof(void *) * n) == cudaSuccess &&
             cudaIpcGetMemHandle(&h, c->mailbox) == cudaSuccess &&
             cudaMemcpy(xfer, &h, hb, cudaMemcpyHostToDevice) == cudaSuccess;
        cudaGetLastError();
    }
    if (agree(ok) == 1) {
        std::vector<unsigned char> handles(hb * n);
        ok = api.AllGather(xfer, xfer + hb, hb, ncclUint8, c->nccl, s) == ncclSuccess &&
             cudaStreamSynchronize(s) == cudaSuccess &&
             cudaMemcpy(handles.data(), xfer + hb, hb * n, cudaMemcpyDeviceToHost) == cudaSuccess;
        std::vector<unsigned char *> boxes(n, nullptr);
        for (int r = 0; r < n && ok; ++r) {
            if (r == c->rank) {
                boxes[r] = c->mailbox;
                continue;
            }
            cudaIpcMemHandle_t h;
            std::memcpy(&h, handles.data() + hb * r, hb);
            void *p = nullptr;
            if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                ok = 0;
                break;
            }
            c->opened.push_back(p);
            boxes[r] = static_cast<unsigned char *>(p);
        }
        if (ok) ok = cudaMemcpy(c->boxes_dev, boxes.data(), sizeof(void *) * n, cudaMemcpyHostToDevice) == cudaSuccess;
        cudaGetLastError();
        c->p2p = agree(ok) == 1;
    }
    cudaFree(xfer);
}

void teardown_p2p(heph_comm *c) {
    for (void *p : c->opened) cudaIpcCloseMemHandle(p);
    c->opened.clear();
    if (c->p2p && !c->aborted) {
        // Every rank has closed its mappings of the others' mailboxes before
        // any rank frees its own: a one-element all-reduce as the barrier,
        // waited for at most 5 s (a rank that is gone aborts the NCCL
        // communicator instead of hanging the teardown).
        int32_t *flag = reinterpret_cast<int32_t *>(c->mailbox);
        cudaStream_t s = c->device->stream;
        if (nccl().AllReduce(flag, flag, 1, ncclInt32, ncclMax, c->nccl, s) == ncclSuccess) {
            const auto t0 = std::chrono::steady_clock::now();
            while (cudaStreamQuery(s) == cudaErrorNotReady) {
                if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(5)) {
                    nccl().CommAbort(c->nccl);
                    c->aborted = true;
                    break;
                }
                std::this_thread::sleep_for(std::chrono::microseconds(100));
            }
        }
        cudaGetLastError();
    }
    if (c->boxes_dev) cudaFree(c->boxes_dev);
    if (c->mailbox) cudaFree(c->mailbox);
    c->boxes_dev = nullptr;
    c->mailbox = nullptr;
    c->p2p = false;
}

}  // namespace

extern "C" heph_status heph_comm_unique_id(uint8_t id[HEPH_COMM_ID_BYTES]) {
    static_assert(sizeof(ncclUniqueId) == HEPH_COMM_ID_BYTES, "NCCL id size");
    NcclApi &api = nccl();
    if (!api.loaded) return fail(HEPH_ADAPTER_UNAVAILABLE, api.why);
    ncclUniqueId uid;
    ncclResult_t r = api.GetUniqueId(&uid);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    std::memcpy(id, &uid, sizeof(uid));
    return HEPH_OK;
}

extern "C" heph_status heph_comm_init(heph_device *device, const uint8_t id[HEPH_COMM_ID_BYTES],
                                      int nranks, int rank, heph_comm **out) {
    if (!device || !id || !out) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks)
        return fail(HEPH_INVALID_CONFIGURATION, "rank " + std::to_string(rank) + " of " +
                                                    std::to_string(nranks) + " is invalid");
    NcclApi &api = nccl();
    if (!api.loaded) return fail(HEPH_ADAPTER_UNAVAILABLE, api.why);
    Device *dev = reinterpret_cast<Device *>(device);
    heph_status st = bind(dev);
    if (st != HEPH_OK) return st;
    heph_comm *c = new heph_comm();
    c->device = dev;
    c->nranks = nranks;
    c->rank = rank;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclResult_t r = api.CommInitRank(&c->nccl, nranks, uid, rank);
    if (r != ncclSuccess) {
        delete c;
        return nccl_fail(r, "ncclCommInitRank");
    }
    c->pair_off = (16 + 8 * (size_t)nranks + 15) & ~size_t(15);
    if (cudaMalloc(&c->scratch, c->pair_off + 32 + 16 * (size_t)nranks) != cudaSuccess) {
        cudaGetLastError();
        api.CommDestroy(c->nccl);
        delete c;
        return fail(HEPH_ALLOCATION_FAILED, "communicator scratch allocation failed");
    }
    setup_p2p(c, dev->stream);
    *out = c;
    return HEPH_OK;
}

extern "C" heph_status heph_comm_destroy(heph_comm *comm) {
    if (!comm) return HEPH_OK;
    cudaSetDevice(comm->device->ordinal);
    if (!comm->aborted) cudaDeviceSynchronize();  // no exchange in flight before the mappings go
    teardown_p2p(comm);
    if (comm->nccl && !comm->aborted) nccl().CommDestroy(comm->nccl);
    if (comm->scratch) cudaFree(comm->scratch);
    delete comm;
    return HEPH_OK;
}

extern "C" heph_status heph_comm_peer_exchange(const heph_comm *comm, int *out) {
    if (!comm || !out) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    *out = comm->p2p ? 1 : 0;
    return HEPH_OK;
}

extern "C" heph_status heph_comm_abort(heph_comm *comm) {
    if (!comm) return HEPH_OK;
    if (comm->nccl && !comm->aborted) {
        nccl().CommAbort(comm->nccl);
        comm->aborted = true;
    }
    return HEPH_OK;
}

extern "C" heph_status heph_comm_wait(heph_comm *comm, heph_stream stream, uint32_t timeout_ms) {
    if (!comm) return fail(HEPH_INVALID_CONFIGURATION, "null communicator");
    if (comm->aborted) return fail(HEPH_DISPATCH_FAILED, "communicator was aborted");
    heph_status st = bind(comm->device);
    if (st != HEPH_OK) return st;
    cudaStream_t s = resolve_stream(comm->device, stream);
    NcclApi &api = nccl();
    cudaError_t stream_err = cudaSuccess;
    const CommWaitResult r = comm_wait_policy(
        timeout_ms,
        [&] {
            const cudaError_t e = cudaStreamQuery(s);
            if (e == cudaSuccess) return StreamPoll::Done;
            if (e == cudaErrorNotReady) return StreamPoll::Pending;
            stream_err = e;
            return StreamPoll::Failed;
        },
        [&] {
            ncclResult_t async = ncclSuccess;
            if (api.CommGetAsyncError(comm->nccl, &async) != ncclSuccess) return CommPoll::Failed;
            return (async == ncclSuccess || async == ncclInProgress) ? CommPoll::Ok : CommPoll::Failed;
        },
        [&] {
            api.CommAbort(comm->nccl);
            comm->aborted = true;
        },
        steady_ms, [] { std::this_thread::sleep_for(std::chrono::microseconds(50)); });
    if (r.ok) return HEPH_OK;
    if (stream_err != cudaSuccess) return cuda_fail(HEPH_DISPATCH_FAILED, stream_err, r.message.c_str());
    return fail(HEPH_DISPATCH_FAILED, r.message);
}

// Runs comm_wait_policy against scripted fakes (no GPU, no NCCL): 0 = the
// stream completes on its third poll; 1 = NCCL reports an asynchronous error
// while the stream is pending; 2 = the stream never completes (deadline);
// 3 = the stream fails.  *out_aborted tells how often the policy aborted.
extern "C" heph_status heph_selftest_comm_wait_policy(int scenario, uint32_t timeout_ms, int *out_aborted) {
    if (scenario < 0 || scenario > 3 || !out_aborted) return fail(HEPH_INVALID_CONFIGURATION, "bad self-test argument");
    int polls = 0, aborts = 0;
    uint64_t clock = 0;
    const CommWaitResult r = comm_wait_policy(
        timeout_ms,
        [&] {
            ++polls;
            if (scenario == 0 && polls >= 3) return StreamPoll::Done;
            if (scenario == 3) return StreamPoll::Failed;
            return StreamPoll::Pending;
        },
        [&] { return scenario == 1 && polls >= 2 ? CommPoll::Failed : CommPoll::Ok; },
        [&] { ++aborts; }, [&] { return clock; }, [&] { clock += 1; });
    *out_aborted = aborts;
    if (r.ok) return HEPH_OK;
    return fail(HEPH_DISPATCH_FAILED, r.message);
}

static heph_status partitioned_args(heph_comm *comm, const heph_buffer *in, const heph_layout *il,
                                    const heph_buffer *out, const heph_layout *ol) {
    if (!comm || !in || !il || !out || !ol) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    if (comm->aborted) return fail(HEPH_DISPATCH_FAILED, "communicator was aborted");
    const Buffer *bi = reinterpret_cast<const Buffer *>(in);
    const Buffer *bo = reinterpret_cast<const Buffer *>(out);
    if (bi->device != comm->device || bo->device != comm->device)
        return fail(HEPH_DISPATCH_FAILED, "operand buffers belong to another device");
    if (il->rank != 1) return fail(HEPH_DISPATCH_FAILED, "partitioned operands are rank-1 slices");
    return HEPH_OK;
}

extern "C" heph_status heph_partitioned_reduce_full(heph_comm *comm, heph_op op,
                                                    const heph_buffer *in, const heph_layout *in_layout,
                                                    heph_buffer *out, const heph_layout *out_layout,
                                                    heph_stream stream) {
    heph_status st = partitioned_args(comm, in, in_layout, out, out_layout);
    if (st != HEPH_OK) return st;
    const Buffer *bi = reinterpret_cast<const Buffer *>(in);
    Buffer *bo = reinterpret_cast<Buffer *>(out);
    if (op != HEPH_SUM && op != HEPH_PROD && op != HEPH_MIN && op != HEPH_MAX)
        return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
    const bool widen = (bi->dtype == HEPH_I32 && bo->dtype == HEPH_I64) ||
                       (bi->dtype == HEPH_F32 && bo->dtype == HEPH_F64);
    if (bi->dtype != bo->dtype && !widen)
        return fail(HEPH_DISPATCH_FAILED, "full reduction output element type must match the input or widen it");
    uint64_t count = 0;
    st = plan_full_reduction(*in_layout, bi->len, *out_layout, bo->len, &count);
    if (st != HEPH_OK) return st;
    Device *dev = comm->device;
    st = bind(dev);
    if (st != HEPH_OK) return st;
    cudaStream_t s = resolve_stream(dev, stream);
    char *scratch = static_cast<char *>(comm->scratch);
    const size_t es = dtype_size(bo->dtype);
    void *dst = static_cast<char *>(bo->ptr) + out_layout->offset * es;
    if (comm->p2p) {
        // The partial goes in the pair's second slot; one kernel exchanges
        // and folds every rank's partial into `dst`.
        char *pair = scratch + comm->pair_off;
        st = launch_reduce_full(dev, s, op, bi->dtype, bo->dtype, bi->ptr, *in_layout, count, pair + 8);
        if (st != HEPH_OK) return st;
        const unsigned long long epoch = comm->epoch++;
        return dispatch_dtype(bo->dtype, [&]<typename T>() {
            return launch_exchange_pairs<T, OP_SUM, T>(s, op, pair, comm->boxes_dev, comm->mailbox, comm->nranks,
                                                       comm->rank, epoch, nullptr, dst, dev->error_dev);
        });
    }
    st = launch_reduce_full(dev, s, op, bi->dtype, bo->dtype, bi->ptr, *in_layout, count, scratch);
    if (st != HEPH_OK) return st;
    ncclResult_t r = nccl().AllGather(scratch, scratch + 16, es, ncclUint8, comm->nccl, s);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    return dispatch_dtype(bo->dtype, [&]<typename T>() {
        return launch_fold<T>(s, op, scratch + 16, comm->nranks, dst);
    });
}

extern "C" heph_status heph_partitioned_scan(heph_comm *comm, heph_op op, int exclusive,
                                             const heph_buffer *in, const heph_layout *in_layout,
                                             heph_buffer *out, const heph_layout *out_layout,
                                             heph_stream stream) {
    heph_status st = partitioned_args(comm, in, in_layout, out, out_layout);
    if (st != HEPH_OK) return st;
    const Buffer *bi = reinterpret_cast<const Buffer *>(in);
    Buffer *bo = reinterpret_cast<Buffer *>(out);
    if (op != HEPH_SUM && op != HEPH_PROD)
        return fail(HEPH_INVALID_CONFIGURATION, "scans support the sum (cumsum) and product (cumprod) operators");
    if (bi->dtype != bo->dtype) return fail(HEPH_DISPATCH_FAILED, "scan output element type must match the input");
    bool noop = false;
    AxisProblem p;
    const bool alias = bi->ptr == bo->ptr;
    st = plan_axis_scan(*in_layout, bi->len, *out_layout, bo->len, 0, alias, &noop, &p);
    if (st != HEPH_OK) return st;
    Device *dev = comm->device;
    st = bind(dev);
    if (st != HEPH_OK) return st;
    cudaStream_t s = resolve_stream(dev, stream);
    char *scratch = static_cast<char *>(comm->scratch);
    const size_t es = dtype_size(bi->dtype);
    // 1. total of the local slice (the identity for an empty slice).
    if (comm->p2p) {
        // Exchanged over peer memory (the pair's first slot) and folded into
        // the carry by one kernel.
        char *pair = scratch + comm->pair_off;
        st = launch_reduce_full(dev, s, op, bi->dtype, bi->dtype, bi->ptr, *in_layout, noop ? 0 : p.len, pair);
        if (st != HEPH_OK) return st;
        const unsigned long long epoch = comm->epoch++;
        st = dispatch_dtype(bi->dtype, [&]<typename T>() {
            if (op == HEPH_SUM)
                return launch_exchange_pairs<T, OP_SUM, T>(s, OP_SUM, pair, comm->boxes_dev, comm->mailbox,
                                                           comm->nranks, comm->rank, epoch, scratch + 8, nullptr,
                                                           dev->error_dev);
            return launch_exchange_pairs<T, OP_PROD, T>(s, OP_SUM, pair, comm->boxes_dev, comm->mailbox, comm->nranks,
                                                        comm->rank, epoch, scratch + 8, nullptr, dev->error_dev);
        });
        if (st != HEPH_OK || noop) return st;
        return launch_scan(dev, s, op, bi->dtype, bi->ptr, bo->ptr, p, false, exclusive != 0, scratch + 8);
    }
    st = launch_reduce_full(dev, s, op, bi->dtype, bi->dtype, bi->ptr, *in_layout, noop ? 0 : p.len, scratch);
    if (st != HEPH_OK) return st;
    // 2. every rank's total.
    ncclResult_t r = nccl().AllGather(scratch, scratch + 16, es, ncclUint8, comm->nccl, s);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    // 3. carry = fold of the totals of the lower ranks.
    st = dispatch_dtype(bi->dtype, [&]<typename T>() {
        return launch_fold<T>(s, op, scratch + 16, comm->rank, scratch + 8);
    });
    if (st != HEPH_OK) return st;
    if (noop) return HEPH_OK;
    // 4. single-pass scan of the slice seeded with the carry.
    return launch_scan(dev, s, op, bi->dtype, bi->ptr, bo->ptr, p, false, exclusive != 0, scratch + 8);
}

extern "C" heph_status heph_partitioned_scan_reduce(heph_comm *comm, heph_op scan_op, int exclusive,
                                                    const heph_buffer *in, const heph_layout *in_layout,
                                                    heph_buffer *scan_out, const heph_layout *scan_layout,
                                                    heph_op reduce_op, heph_buffer *reduce_out,
                                                    const heph_layout *reduce_layout, heph_stream stream) {
    heph_status st = partitioned_args(comm, in, in_layout, scan_out, scan_layout);
    if (st != HEPH_OK) return st;
    if (!reduce_out || !reduce_layout) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    const Buffer *bi = reinterpret_cast<const Buffer *>(in);
    Buffer *bo = reinterpret_cast<Buffer *>(scan_out);
    Buffer *br = reinterpret_cast<Buffer *>(reduce_out);
    if (br->device != comm->device) return fail(HEPH_DISPATCH_FAILED, "operand buffers belong to another device");
    if (scan_op != HEPH_SUM && scan_op != HEPH_PROD)
        return fail(HEPH_INVALID_CONFIGURATION, "scans support the sum (cumsum) and product (cumprod) operators");
    if (reduce_op != HEPH_SUM && reduce_op != HEPH_PROD && reduce_op != HEPH_MIN && reduce_op != HEPH_MAX)
        return fail(HEPH_INVALID_CONFIGURATION, "full reduction supports sum, prod, min and max");
    if (bi->dtype != bo->dtype) return fail(HEPH_DISPATCH_FAILED, "scan output element type must match the input");
    const bool widen = (bi->dtype == HEPH_I32 && br->dtype == HEPH_I64) ||
                       (bi->dtype == HEPH_F32 && br->dtype == HEPH_F64);
    if (bi->dtype != br->dtype && !widen)
        return fail(HEPH_DISPATCH_FAILED, "full reduction output element type must match the input or widen it");
    uint64_t count = 0;
    st = plan_full_reduction(*in_layout, bi->len, *reduce_layout, br->len, &count);
    if (st != HEPH_OK) return st;
    bool noop = false;
    AxisProblem p;
    st = plan_axis_scan(*in_layout, bi->len, *scan_layout, bo->len, 0, bi->ptr == bo->ptr, &noop, &p);
    if (st != HEPH_OK) return st;
    Device *dev = comm->device;
    st = bind(dev);
    if (st != HEPH_OK) return st;
    cudaStream_t s = resolve_stream(dev, stream);
    char *pair = static_cast<char *>(comm->scratch) + comm->pair_off;
    char *carry = pair + 16, *gathered = pair + 32;
    // 1. the slice's scan total and reduction partial in one read (two reads
    //    when the slice is not one dense run).
    const int64_t first = (int64_t)in_layout->offset;
    if (count > 0 && layout_is_dense(*in_layout)) {
        const void *base = static_cast<const char *>(bi->ptr) + first * (int64_t)dtype_size(bi->dtype);
        st = launch_reduce_dual(dev, s, scan_op, reduce_op, bi->dtype, br->dtype, base, count, pair, pair + 8);
    } else {
        st = launch_reduce_full(dev, s, scan_op, bi->dtype, bi->dtype, bi->ptr, *in_layout, count, pair);
        if (st == HEPH_OK)
            st = launch_reduce_full(dev, s, reduce_op, bi->dtype, br->dtype, bi->ptr, *in_layout, count, pair + 8);
    }
    if (st != HEPH_OK) return st;
    // 2 + 3. every rank's pair, then carry (lower ranks' totals) and the
    // global reduction (all partials): over peer memory in one kernel, or an
    // NCCL all-gather and a fold kernel.
    void *gdst = static_cast<char *>(br->ptr) + reduce_layout->offset * dtype_size(br->dtype);
    const unsigned long long epoch = comm->epoch++;
    ncclResult_t r = ncclSuccess;
    if (!comm->p2p) {
        r = nccl().AllGather(pair, gathered, 16, ncclUint8, comm->nccl, s);
        if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    }
    auto fold = [&]<typename T, typename Tacc>() -> heph_status {
        if (comm->p2p) {
            if (scan_op == HEPH_SUM)
                return launch_exchange_pairs<T, OP_SUM, Tacc>(s, reduce_op, pair, comm->boxes_dev, comm->mailbox,
                                                             comm->nranks, comm->rank, epoch, carry, gdst,
                                                             dev->error_dev);
            return launch_exchange_pairs<T, OP_PROD, Tacc>(s, reduce_op, pair, comm->boxes_dev, comm->mailbox,
                                                          comm->nranks, comm->rank, epoch, carry, gdst, dev->error_dev);
        }
        if (scan_op == HEPH_SUM)
            return launch_fold_pairs<T, OP_SUM, Tacc>(s, reduce_op, gathered, comm->nranks, comm->rank, carry, gdst);
        return launch_fold_pairs<T, OP_PROD, Tacc>(s, reduce_op, gathered, comm->nranks, comm->rank, carry, gdst);
    };
    if (bi->dtype == br->dtype)
        st = dispatch_dtype(bi->dtype, [&]<typename T>() { return fold.template operator()<T, T>(); });
    else if (bi->dtype == HEPH_I32)
        st = fold.template operator()<int32_t, int64_t>();
    else
        st = fold.template operator()<float, double>();
    if (st != HEPH_OK) return st;
    if (noop) return HEPH_OK;
    // 4. the slice's scan seeded with the carry.
    return launch_scan(dev, s, scan_op, bi->dtype, bi->ptr, bo->ptr, p, false, exclusive != 0, carry);
}
