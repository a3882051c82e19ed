// NCCL for the strip-sharded pass: the library is opened at run time (the process
// already has it loaded when torch.distributed runs NCCL), so libhat_b200 itself has no
// link dependency on it. Only the calls the halo exchange and the channel-sum
// all-reduce use are bound.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <memory>
#include <string>

#include "rendezvous.h"

namespace hat {

// A communicator over `n` ranks, one GPU each, created collectively from one unique id.
class Comm {
public:
    // `timeout_s`: the deadline of every host-side wait on the peers (initialisation, group
    // launches) and of wait(); <= 0 waits without one.
    Comm(int rank, int n, const void* id, size_t idlen, int device, double timeout_s);
    ~Comm();
    int rank() const { return rank_; }
    int size() const { return n_; }
    // Inside group(): the calls are matched per peer in the order they are posted.
    void group_start();
    void group_end();
    void send(const float* buf, size_t count, int peer, cudaStream_t st);
    void recv(float* buf, size_t count, int peer, cudaStream_t st);
    void allreduce_sum(float* buf, size_t count, cudaStream_t st);
    // The start of a pass, before any of its NCCL calls is enqueued: waits, under the
    // deadline, until every rank has reached the same pass (rendezvous.h). A peer that does
    // not come ends the wait with Error(3); nothing was enqueued, the communicator stays
    // intact and the call can be repeated.
    void begin_pass();
    // Waits for the work on `st` (which holds this communicator's calls) for at most
    // `timeout_s` seconds (<= 0: no deadline), polling the communicator's asynchronous
    // error state. If a peer failed or the deadline passed, the communicator is aborted
    // (its pending kernels return) and Error(3) names the cause; an aborted communicator
    // refuses every later call.
    void wait(cudaStream_t st, double timeout_s);
    bool aborted() const { return aborted_; }
    void set_timeout(double s) { timeout_s_ = s; }

private:
    void live() const;  // throws once aborted
    // Waits until the communicator's state leaves ncclInProgress, under the deadline; on an
    // error or at the deadline aborts the communicator and throws.
    void settle(const char* what);
    // Marks the communicator aborted and runs ncclCommAbort (which makes its pending kernels
    // return), waiting for it at most ABORT_WAIT_S seconds: the caller gets its error even if
    // the abort itself does not return.
    void abort_comm();
    static constexpr double ABORT_WAIT_S = 10.0;
    int rank_, n_;
    double timeout_s_ = 120.0;
    ncclComm_t comm_ = nullptr;
    bool aborted_ = false;
    std::unique_ptr<Rendezvous> rv_;
};

// ncclGetUniqueId into `out` (at least sizeof(ncclUniqueId) = 128 bytes).
void nccl_unique_id(void* out, size_t len);

}  // namespace hat
