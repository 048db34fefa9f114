// comm_wait.h — the host-side deadline on a partitioned call's NCCL exchange.
//
// A collective whose peer rank died or never arrives spins on the GPU until
// NCCL is told to give up.  The caller waits on the host instead: poll the
// stream, poll the communicator's asynchronous error, and abort the
// communicator when NCCL reports an error or the deadline passes (the NCCL
// kernels then exit and the stream drains).  The policy is written against
// callbacks so that it runs, and is tested, without a GPU.
#pragma once

#include <chrono>
#include <cstdint>
#include <string>

namespace heph {

enum class StreamPoll { Done, Pending, Failed };
enum class CommPoll { Ok, Failed };

struct CommWaitResult {
    bool ok = false;
    bool aborted = false;
    std::string message;  // why it failed (empty when ok)
};

// stream(): the stream's state; comm(): NCCL's asynchronous error state;
// abort(): abort the communicator; now_ms(): a monotonic clock; pause(): a
// short sleep between polls.
template <typename StreamFn, typename CommFn, typename AbortFn, typename NowFn, typename PauseFn>
CommWaitResult comm_wait_policy(uint32_t timeout_ms, StreamFn stream, CommFn comm, AbortFn abort, NowFn now_ms,
                                PauseFn pause) {
    CommWaitResult r;
    const uint64_t start = now_ms();
    while (true) {
        const StreamPoll s = stream();
        if (s == StreamPoll::Done) {
            r.ok = true;
            return r;
        }
        if (s == StreamPoll::Failed) {
            r.message = "the stream of the partitioned call failed";
            return r;
        }
        if (comm() == CommPoll::Failed) {
            abort();
            r.aborted = true;
            r.message = "NCCL reported an asynchronous error; the communicator was aborted";
            return r;
        }
        if (now_ms() - start >= timeout_ms) {
            abort();
            r.aborted = true;
            r.message = "collective deadline of " + std::to_string(timeout_ms) +
                        " ms expired (a peer rank is gone or late); the communicator was aborted";
            return r;
        }
        pause();
    }
}

inline uint64_t steady_ms() {
    return (uint64_t)std::chrono::duration_cast<std::chrono::milliseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

}  // namespace heph
