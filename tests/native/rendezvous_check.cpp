// CPU check of the host rendezvous that starts every strip-sharded pass
// (hat-rs_b200/csrc/rendezvous.h): ranks as processes (fork) and as threads over one
// shared-memory word. Prints one line per case and exits nonzero on the first mismatch.
#include <sys/wait.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <random>
#include <thread>
#include <vector>

#include "rendezvous.h"

using hat::Rendezvous;

static int fails = 0;

static void expect(const char* name, bool ok) {
    std::printf("%s %s\n", ok ? "ok" : "FAIL", name);
    std::fflush(stdout);
    if (!ok) ++fails;
}

static double secs_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

int main() {
    // A key of its own per run, as a fresh unique id would be.
    char key[32];
    std::snprintf(key, sizeof key, "rv-check-%d", (int)getpid());

    {  // two processes meet for three passes; then rank 1 stops calling: rank 0 times out
       // twice (withdrawing each time), and meets rank 1 again once it comes back
        int fd[2];
        if (pipe(fd) != 0) return 2;
        const pid_t child = fork();
        if (child == 0) {
            Rendezvous rv(key, sizeof key, 1, 2);
            int ok = 1;
            for (int i = 0; i < 3; ++i) ok &= rv.arrive(10.0) == Rendezvous::Met;
            char c;
            if (read(fd[0], &c, 1) != 1) ok = 0;  // stays away until rank 0 has timed out twice
            ok &= rv.arrive(10.0) == Rendezvous::Met;
            ok &= rv.pass() == 4;
            _exit(ok ? 0 : 1);
        }
        Rendezvous rv(key, sizeof key, 0, 2);
        bool met3 = true;
        for (int i = 0; i < 3; ++i) met3 &= rv.arrive(10.0) == Rendezvous::Met;
        auto t0 = std::chrono::steady_clock::now();
        const Rendezvous::Result r1 = rv.arrive(0.3);
        const double s1 = secs_since(t0);
        const Rendezvous::Result r2 = rv.arrive(0.3);
        const uint64_t still = rv.pass();
        if (write(fd[1], "x", 1) != 1) return 2;
        const Rendezvous::Result r3 = rv.arrive(10.0);
        int st = 0;
        waitpid(child, &st, 0);
        expect("processes meet for three passes", met3);
        expect("a peer that stops calling ends the wait at the deadline",
               r1 == Rendezvous::TimedOut && s1 >= 0.3 && s1 < 5.0);
        expect("the call can be repeated at the same pass", r2 == Rendezvous::TimedOut && still == 3);
        expect("the peer comes back and both run the pass",
               r3 == Rendezvous::Met && rv.pass() == 4 && WIFEXITED(st) && WEXITSTATUS(st) == 0);
        // A rank whose calls are out of step (a fresh handle at pass 0 against pass 4).
        Rendezvous late(key, sizeof key, 1, 2);
        expect("ranks at different passes are told so", late.arrive(0.2) == Rendezvous::Mismatch);
    }

    {  // four threads, 300 passes, random delays and deadlines short enough that many arrivals
       // are withdrawn: every pass is met by all, and never before every rank has reached it
        char key2[40];
        std::snprintf(key2, sizeof key2, "rv-stress-%d", (int)getpid());
        constexpr int T = 4, PASSES = 300;
        std::atomic<long> cur[T];
        for (auto& c : cur) c.store(-1);
        std::atomic<int> early{0}, mism{0}, withdrawn{0};
        std::vector<std::thread> th;
        for (int i = 0; i < T; ++i)
            th.emplace_back([&, i] {
                Rendezvous rv(key2, sizeof key2, i, T);
                std::mt19937 g(1234 + i);
                for (long k = 0; k < PASSES; ++k) {
                    cur[i].store(k);
                    for (;;) {
                        if (g() % 8 == 0) std::this_thread::sleep_for(std::chrono::microseconds(g() % 3000));
                        const Rendezvous::Result r = rv.arrive(0.0005 + (g() % 4) * 0.0005, 5);
                        if (r == Rendezvous::Met) break;
                        if (r == Rendezvous::Mismatch) {
                            ++mism;
                            return;
                        }
                        ++withdrawn;
                    }
                    for (int j = 0; j < T; ++j)
                        if (cur[j].load() < k) ++early;
                }
            });
        for (auto& t : th) t.join();
        bool all = true;
        for (auto& c : cur) all &= c.load() == PASSES - 1;
        std::printf("  (%d withdrawn arrivals)\n", withdrawn.load());
        expect("threads meet at every pass, none before all have arrived",
               all && early.load() == 0 && mism.load() == 0 && withdrawn.load() > 0);
    }
    return fails ? 1 : 0;
}
