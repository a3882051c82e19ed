// The host-side start of every strip-sharded pass: the ranks meet before any of them
// enqueues NCCL work for it.
//
// Once a rank has launched a pass, its NCCL kernels wait on the GPU for its neighbours'
// halo rows. If a neighbour's process stopped calling (it is alive but issues nothing),
// those kernels wait forever and only an abort of the communicator ends them, which leaves
// the handle unusable. So each pass starts with a rendezvous on the host: every rank
// announces that it has reached pass k and waits, under the deadline, until all have. A rank
// whose peers do not come withdraws its arrival, enqueues nothing and returns an error; the
// communicator stays intact and the call can be repeated (the ranks meet again at the same
// pass k). A rank that dies after arriving but before the pass is sealed looks, to the
// others, as if it had arrived; they launch and fall to the in-pass deadline instead.
//
// The ranks of a strip communicator run on one node (NVLink peers), so the meeting point is
// a POSIX shared-memory word named after the communicator's unique id, shared by the
// processes (one per GPU) or threads (one handle over several GPUs) of the job. The word
// holds the pass number, a sealed bit and the count of ranks that have arrived; every
// change is one compare-and-swap, so sealing (the last arrival) and a withdrawal (a rank
// giving up) exclude each other: either every rank proceeds or none does.
//
// Header-only and free of CUDA and NCCL types, so it is tested on the CPU with processes.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <string>
#include <thread>

namespace hat {

static_assert(std::atomic<uint64_t>::is_always_lock_free, "the shared word needs address-free atomics");

class Rendezvous {
public:
    // `key`/`len`: the bytes every rank of the job shares (the NCCL unique id).
    Rendezvous(const void* key, size_t len, int rank, int n) : rank_(rank), n_(n) {
        // FNV-1a over the key: the segment's name.
        uint64_t h = 1469598103934665603ull;
        const unsigned char* p = static_cast<const unsigned char*>(key);
        for (size_t i = 0; i < len; ++i) h = (h ^ p[i]) * 1099511628211ull;
        char name[64];
        std::snprintf(name, sizeof name, "/hat_b200_rv_%016llx", (unsigned long long)h);
        name_ = name;
        const int fd = shm_open(name, O_CREAT | O_RDWR, 0600);
        if (fd < 0) return;
        // A new segment reads as zeros: pass 0, not sealed, nobody arrived.
        if (ftruncate(fd, 64) == 0) {
            void* m = mmap(nullptr, 64, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
            if (m != MAP_FAILED) word_ = static_cast<std::atomic<uint64_t>*>(m);
        }
        close(fd);
    }
    ~Rendezvous() {
        if (word_) munmap(word_, 64);
        shm_unlink(name_.c_str());  // the ranks still mapping it keep their mapping
    }
    Rendezvous(const Rendezvous&) = delete;
    Rendezvous& operator=(const Rendezvous&) = delete;

    bool ok() const { return word_ != nullptr; }
    uint64_t pass() const { return pass_; }
    const std::string& name() const { return name_; }

    enum Result { Met = 1, TimedOut = 0, Mismatch = -1 };

    // Waits until every rank has arrived at this rank's next pass, for at most `timeout_s`
    // seconds (<= 0: no deadline). Met: the pass is sealed and the rank moves on to the next
    // one. TimedOut: the peers did not all come; this rank's arrival is withdrawn and the next
    // call waits for the same pass again. Mismatch: the shared word is at a pass this rank
    // cannot join (the ranks' calls were not matched one for one).
    Result arrive(double timeout_s, int poll_us = 20) {
        const uint64_t k = pass_;
        std::atomic<uint64_t>& w = *word_;
        // Join pass k: from pass k - 1 sealed (the first arrival opens pass k) or pass k open.
        uint64_t cur = w.load(std::memory_order_acquire);
        for (;;) {
            uint64_t next;
            if (k > 0 && seq(cur) + 1 == k && sealed(cur))
                next = make(k, false, 1);
            else if (seq(cur) == k && !sealed(cur))
                next = make(k, false, count(cur) + 1);
            else
                return Mismatch;
            if (count(next) >= (uint64_t)n_) next = make(k, true, count(next));
            if (w.compare_exchange_weak(cur, next, std::memory_order_acq_rel, std::memory_order_acquire)) break;
        }
        using clock = std::chrono::steady_clock;
        const auto t0 = clock::now();
        for (;;) {
            cur = w.load(std::memory_order_acquire);
            if (passed(cur, k)) {
                ++pass_;
                return Met;
            }
            if (timeout_s > 0 && std::chrono::duration<double>(clock::now() - t0).count() > timeout_s) {
                // Withdraw, unless the last rank sealed the pass in the meantime.
                for (;;) {
                    if (passed(cur, k)) {
                        ++pass_;
                        return Met;
                    }
                    const uint64_t next = make(k, false, count(cur) - 1);
                    if (w.compare_exchange_weak(cur, next, std::memory_order_acq_rel, std::memory_order_acquire))
                        return TimedOut;
                }
            }
            std::this_thread::sleep_for(std::chrono::microseconds(poll_us));
        }
    }

private:
    // word: pass number (bits 24..63) | sealed (bit 23) | ranks arrived (bits 0..22)
    static uint64_t seq(uint64_t v) { return v >> 24; }
    static bool sealed(uint64_t v) { return (v >> 23) & 1; }
    static uint64_t count(uint64_t v) { return v & ((1u << 23) - 1); }
    static uint64_t make(uint64_t s, bool sl, uint64_t c) { return (s << 24) | ((uint64_t)sl << 23) | c; }
    // Pass k is sealed, or a later pass has opened (which needs k sealed first).
    static bool passed(uint64_t v, uint64_t k) { return (seq(v) == k && sealed(v)) || seq(v) > k; }
    int rank_, n_;
    uint64_t pass_ = 0;
    std::string name_;
    std::atomic<uint64_t>* word_ = nullptr;
};

}  // namespace hat
