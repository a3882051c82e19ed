// CPU check of the engine's deadline wait (hat-rs_b200/csrc/deadline.h) with fakes of
// the three probes: a stream that completes, one that fails, a communicator that reports
// an asynchronous error, and work that never completes. Prints one line per case and
// exits nonzero on the first mismatch.
#include <chrono>
#include <cstdio>

#include "deadline.h"

using hat::WaitEnd;

static int fails = 0;

static void expect(const char* name, bool ok) {
    std::printf("%s %s\n", ok ? "ok" : "FAIL", name);
    if (!ok) ++fails;
}

int main() {
    using clock = std::chrono::steady_clock;
    {  // completes after a few polls; no abort
        int polls = 0, aborts = 0;
        WaitEnd e = hat::wait_with_deadline([&] { return ++polls >= 5 ? 1 : 0; }, [] { return false; },
                                            [&] { ++aborts; }, 5.0, 10);
        expect("done", e == WaitEnd::Done && polls == 5 && aborts == 0);
    }
    {  // the stream reports an error; no abort (the communicator is not to blame)
        int aborts = 0;
        WaitEnd e = hat::wait_with_deadline([] { return -1; }, [] { return false; }, [&] { ++aborts; }, 5.0, 10);
        expect("stream error", e == WaitEnd::StreamError && aborts == 0);
    }
    {  // a peer fails after a while: abort exactly once, well before the deadline
        int polls = 0, aborts = 0;
        const auto t0 = clock::now();
        WaitEnd e = hat::wait_with_deadline([] { return 0; }, [&] { return ++polls >= 20; }, [&] { ++aborts; },
                                            30.0, 10);
        const double s = std::chrono::duration<double>(clock::now() - t0).count();
        expect("peer error", e == WaitEnd::PeerError && aborts == 1 && s < 5.0);
    }
    {  // never completes: the deadline ends the wait with one abort
        int aborts = 0;
        const auto t0 = clock::now();
        WaitEnd e = hat::wait_with_deadline([] { return 0; }, [] { return false; }, [&] { ++aborts; }, 0.3, 100);
        const double s = std::chrono::duration<double>(clock::now() - t0).count();
        expect("timed out", e == WaitEnd::TimedOut && aborts == 1 && s >= 0.3 && s < 5.0);
    }
    {  // no deadline: completion still ends the wait
        int polls = 0;
        WaitEnd e = hat::wait_with_deadline([&] { return ++polls >= 3 ? 1 : 0; }, [] { return false; }, [] {}, 0.0,
                                            10);
        expect("no deadline", e == WaitEnd::Done);
    }
    return fails ? 1 : 0;
}
