// NCCL bound at run time with dlopen (see nccl_rt.h).
#include "nccl_rt.h"

#include <dlfcn.h>

#include <atomic>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>

#include "common.cuh"
#include "deadline.h"

#ifndef HAT_NCCL_LIB
#define HAT_NCCL_LIB "libnccl.so.2"
#endif

namespace hat {

namespace {

struct Api {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
};

template <class F>
void bind(void* lib, const char* name, F& fn) {
    fn = reinterpret_cast<F>(dlsym(lib, name));
    if (!fn) throw Error(3, std::string("nccl: symbol ") + name + " not found");
}

const Api& api() {
    static Api a;
    static std::once_flag once;
    static std::string failure;
    std::call_once(once, [] {
        // The copy the process already loaded (torch's), else the search path, else the
        // path recorded at build time.
        void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW);
        if (!lib) lib = dlopen(HAT_NCCL_LIB, RTLD_NOW);
        if (!lib) {
            failure = std::string("nccl: cannot open libnccl.so.2 (") + (dlerror() ? dlerror() : "?") + ")";
            return;
        }
        try {
            bind(lib, "ncclGetUniqueId", a.get_unique_id);
            bind(lib, "ncclCommInitRank", a.comm_init_rank);
            bind(lib, "ncclCommDestroy", a.comm_destroy);
            bind(lib, "ncclGroupStart", a.group_start);
            bind(lib, "ncclGroupEnd", a.group_end);
            bind(lib, "ncclSend", a.send);
            bind(lib, "ncclRecv", a.recv);
            bind(lib, "ncclAllReduce", a.all_reduce);
            bind(lib, "ncclGetErrorString", a.error_string);
            bind(lib, "ncclCommGetAsyncError", a.get_async_error);
            bind(lib, "ncclCommAbort", a.comm_abort);
            bind(lib, "ncclCommInitRankConfig", a.comm_init_rank_config);
        } catch (const Error& e) {
            failure = e.what();
        }
    });
    if (!failure.empty()) throw Error(3, failure);
    return a;
}

void check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) throw Error(3, std::string("nccl: ") + what + " failed: " + api().error_string(r));
}

}  // namespace

void nccl_unique_id(void* out, size_t len) {
    if (len < sizeof(ncclUniqueId)) throw Error(1, "nccl: the unique id needs 128 bytes");
    ncclUniqueId id;
    check(api().get_unique_id(&id), "ncclGetUniqueId");
    memcpy(out, &id, sizeof id);
}

Comm::Comm(int rank, int n, const void* id, size_t idlen, int device, double timeout_s)
    : rank_(rank), n_(n), timeout_s_(timeout_s) {
    if (n < 1 || rank < 0 || rank >= n) throw Error(1, "nccl: bad rank / size");
    if (!id || idlen < sizeof(ncclUniqueId)) throw Error(1, "nccl: the unique id needs 128 bytes");
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    rv_.reset(new Rendezvous(&uid, sizeof uid, rank, n));
    if (!rv_->ok()) throw Error(3, "nccl: cannot map the shared-memory rendezvous " + rv_->name());
    HAT_CUDA(cudaSetDevice(device));
    // Non-blocking: no NCCL call waits on the peers inside NCCL (connection set-up, the buffer
    // registration of a graph capture, group launches); each returns at once and settle()
    // waits for the communicator's state under the deadline instead.
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t r = api().comm_init_rank_config(&comm_, n, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) check(r, "ncclCommInitRankConfig");
    settle("ncclCommInitRankConfig");
}

void Comm::settle(const char* what) {
    ncclResult_t state = ncclSuccess;
    const WaitEnd end = wait_with_deadline(
        [&] {
            const ncclResult_t r = api().get_async_error(comm_, &state);
            if (r != ncclSuccess) state = r;
            if (state == ncclSuccess) return 1;
            return state == ncclInProgress ? 0 : -1;
        },
        [] { return false; },
        [&] { abort_comm(); }, timeout_s_);
    if (end == WaitEnd::Done) return;
    if (end == WaitEnd::StreamError) {
        abort_comm();
        throw Error(3, std::string("nccl: ") + what + " failed on rank " + std::to_string(rank_) + ": " +
                           api().error_string(state) + "; the communicator was aborted");
    }
    char buf[64];
    snprintf(buf, sizeof buf, "%.1f", timeout_s_);
    throw Error(3, std::string("nccl: rank ") + std::to_string(rank_) + " of " + std::to_string(n_) + ": " + what +
                       " did not complete within " + buf +
                       " s (a peer rank stopped calling or died); the communicator was aborted");
}

void Comm::abort_comm() {
    if (aborted_) return;
    aborted_ = true;
    auto done = std::make_shared<std::atomic<int>>(0);
    ncclComm_t c = comm_;
    std::thread([c, done] {
        api().comm_abort(c);
        done->store(1, std::memory_order_release);
    }).detach();
    wait_with_deadline([&] { return done->load(std::memory_order_acquire); }, [] { return false; }, [] {},
                       ABORT_WAIT_S, 200);
}

void Comm::begin_pass() {
    live();
    const uint64_t k = rv_->pass();
    const Rendezvous::Result r = rv_->arrive(timeout_s_);
    if (r == Rendezvous::Met) return;
    char buf[64];
    snprintf(buf, sizeof buf, "%.1f", timeout_s_);
    if (r == Rendezvous::TimedOut)
        throw Error(3, std::string("nccl: rank ") + std::to_string(rank_) + " of " + std::to_string(n_) +
                           ": the other ranks did not start pass " + std::to_string(k) + " within " + buf +
                           " s (a peer rank stopped calling or died); nothing was enqueued and the "
                           "communicator is intact, so the call can be repeated");
    throw Error(3, std::string("nccl: rank ") + std::to_string(rank_) + " of " + std::to_string(n_) +
                       ": the ranks are not at the same pass (their calls were not matched one for one)");
}

Comm::~Comm() {
    // An aborted communicator has already released its resources.
    if (comm_ && !aborted_) api().comm_destroy(comm_);
}

void Comm::live() const {
    if (aborted_)
        throw Error(3, "nccl: the communicator was aborted after a failed or timed-out exchange; attach the "
                       "strips again to continue");
}

void Comm::group_start() {
    live();
    check(api().group_start(), "ncclGroupStart");
}
void Comm::group_end() {
    const ncclResult_t r = api().group_end();
    if (r != ncclSuccess && r != ncclInProgress) check(r, "ncclGroupEnd");
    settle("ncclGroupEnd");
}

void Comm::send(const float* buf, size_t count, int peer, cudaStream_t st) {
    live();
    check(api().send(buf, count, ncclFloat32, peer, comm_, st), "ncclSend");
}

void Comm::recv(float* buf, size_t count, int peer, cudaStream_t st) {
    live();
    check(api().recv(buf, count, ncclFloat32, peer, comm_, st), "ncclRecv");
}

void Comm::allreduce_sum(float* buf, size_t count, cudaStream_t st) {
    group_start();  // a group, so that group_end() settles the non-blocking call
    check(api().all_reduce(buf, buf, count, ncclFloat32, ncclSum, comm_, st), "ncclAllReduce");
    group_end();
}

void Comm::wait(cudaStream_t st, double timeout_s) {
    live();
    ncclResult_t async = ncclSuccess;
    cudaError_t serr = cudaSuccess;
    const WaitEnd end = wait_with_deadline(
        [&] {
            serr = cudaStreamQuery(st);
            if (serr == cudaSuccess) return 1;
            if (serr == cudaErrorNotReady) return 0;
            return -1;
        },
        [&] {
            const ncclResult_t r = api().get_async_error(comm_, &async);
            if (r != ncclSuccess) async = r;
            return async != ncclSuccess && async != ncclInProgress;
        },
        [&] { abort_comm(); }, timeout_s);
    switch (end) {
        case WaitEnd::Done:
            return;
        case WaitEnd::StreamError:
            throw Error(3, std::string("gpu: the strip pass failed on the device: ") + cudaGetErrorString(serr));
        case WaitEnd::PeerError:
            throw Error(3, std::string("nccl: rank ") + std::to_string(rank_) + " of " + std::to_string(n_) +
                               ": the communicator reported an asynchronous error (" + api().error_string(async) +
                               "); a peer rank failed or left, and the communicator was aborted");
        case WaitEnd::TimedOut:
            break;
    }
    char buf[64];
    snprintf(buf, sizeof buf, "%.1f", timeout_s);
    throw Error(3, std::string("nccl: rank ") + std::to_string(rank_) + " of " + std::to_string(n_) +
                       ": the strip pass did not finish within " + buf +
                       " s (a peer rank stopped calling or died); the communicator was aborted");
}

}  // namespace hat
