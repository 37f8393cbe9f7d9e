// watchdog.h -- bounded wait for stream-ordered work that may never finish
// (an NCCL kernel whose peer stopped).  Host logic only; the callbacks make
// it testable without a GPU (s2b_debug_watchdog_selftest).
#pragma once
#include <chrono>
#include <cstdint>
#include <thread>

namespace s2b {

enum WatchQuery { WATCH_Q_DONE = 0, WATCH_Q_PENDING = 1, WATCH_Q_ERROR = 2 };
enum WatchResult { WATCH_DONE = 0, WATCH_ASYNC_ERROR = 1, WATCH_EXPIRED = 2, WATCH_STREAM_ERROR = 3 };

// Polls query() (a WatchQuery) every poll_ns until the work is done or failed.
// While it is pending, async_error() (true when the communicator reports an
// asynchronous error) is polled too; on such an error, or once timeout_ns
// have passed, abort() is called once and the wait ends.
template <class Query, class AsyncError, class Abort>
int watch_completion(Query query, AsyncError async_error, Abort abort, uint64_t timeout_ns, uint64_t poll_ns) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const int q = query();
        if (q == WATCH_Q_DONE) return WATCH_DONE;
        if (q == WATCH_Q_ERROR) return WATCH_STREAM_ERROR;
        if (async_error()) {
            abort();
            return WATCH_ASYNC_ERROR;
        }
        const auto waited = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0);
        if ((uint64_t)waited.count() > timeout_ns) {
            abort();
            return WATCH_EXPIRED;
        }
        std::this_thread::sleep_for(std::chrono::nanoseconds(poll_ns));
    }
}

}  // namespace s2b
