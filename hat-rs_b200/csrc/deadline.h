// Waiting for device work that depends on other GPUs, with a deadline.
//
// A strip-sharded pass exchanges halo rows with its neighbours; if a neighbour's process
// died, or it stopped calling, the NCCL kernels of this rank wait for data that never
// comes and a plain cudaStreamSynchronize blocks forever. The reference turns every
// failure into an error return (src/main.rs:160-196), so the engine waits by polling
// instead: the stream's completion, the communicator's asynchronous error state and a
// host clock. On an asynchronous error or when the deadline passes it aborts the
// communicator (which makes the outstanding NCCL kernels return) and reports the cause.
//
// Header-only and free of CUDA and NCCL types, so the logic is tested on the CPU with
// fakes of the three probes.
#pragma once

#include <chrono>
#include <thread>

namespace hat {

enum class WaitEnd { Done, StreamError, PeerError, TimedOut };

// `done()`: 1 when the work completed, 0 while it runs, -1 on a stream error.
// `peer_failed()`: true when the communicator reports an asynchronous error.
// `abort()`: called once, before returning PeerError or TimedOut.
// `timeout_s` <= 0 waits without a deadline (the asynchronous error is still polled).
template <class Done, class PeerFailed, class Abort>
WaitEnd wait_with_deadline(Done&& done, PeerFailed&& peer_failed, Abort&& abort, double timeout_s,
                           int poll_us = 50) {
    using clock = std::chrono::steady_clock;
    const auto t0 = clock::now();
    for (;;) {
        const int d = done();
        if (d > 0) return WaitEnd::Done;
        if (d < 0) return WaitEnd::StreamError;
        if (peer_failed()) {
            abort();
            return WaitEnd::PeerError;
        }
        if (timeout_s > 0 && std::chrono::duration<double>(clock::now() - t0).count() > timeout_s) {
            abort();
            return WaitEnd::TimedOut;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(poll_us));
    }
}

}  // namespace hat
