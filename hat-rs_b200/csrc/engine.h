// The layer scheduler: the HAT graph as a sequence of fused kernel launches on one
// stream of one device (the role of src/gpu.rs in the reference).
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "conv_last.h"
#include "umma.cuh"
#include "weights.h"

namespace hat {

class Comm;

// Every device buffer one pass needs, as one list used both to allocate and to
// predict (the reference's `Sizes`, src/gpu.rs:166-290): a pass allocates exactly
// `total()` floats, and the memory guard refuses on the same number.
struct Sizes {
    long x0 = 0, body = 0, xa = 0, xb = 0, n1 = 0, n1lo = 0, cmid = 0, cmidlo = 0, convx = 0, qkv = 0, attn = 0,
         attnlo = 0, hid = 0, hidlo = 0;
    long chsum = 0, casum = 0, gate = 0, headA = 0, headAlo = 0, headB = 0, headBlo = 0, din = 0, dout = 0;
    long cabstat = 0;  // per-row sums of the CAB's middle plane (launch_cab_pool)
    int cmid_stride = 0;  // channel stride of the CAB's middle plane
    static Sizes of(const Weights& wt, const Plan& p);
    long total() const {
        return x0 + body + xa + xb + n1 + n1lo + cmid + cmidlo + convx + qkv + attn + attnlo + hid + hidlo + chsum +
               casum + gate + headA + headAlo + headB + headBlo + din + dout + cabstat;
    }
};

class Engine {
public:
    Engine(const std::string& path, int device, int mode, bool use_graph, bool simt_only);
    ~Engine();
    const Weights& weights() const { return wt_; }
    int device() const { return device_; }
    // Host in / host out (Backend::forward).
    void forward_host(int n, int h, int w, const float* in, float* out);
    // Device in / device out, enqueued on `st` (nullptr: the engine's stream).
    void forward_device(int n, int h, int w, const float* din, float* dout, cudaStream_t st);
    size_t footprint_bytes(int h, int w) const;
    void check_memory(int h, int w) const;  // throws Error(4, refusal) when it does not fit
    uint64_t launches() const { return launches_; }
    cudaStream_t stream() const { return stream_; }
    // Per-kind device time of one eager pass, as JSON (see Engine::profile).
    std::string profile(int h, int w);
    // Reads (and clears) the tensor-core kernels' error flag; throws if it was set.
    void check_device_error();
    // Waits for the work enqueued on the engine's stream and reports a device error.
    void sync();
    // fp16 operand pairs (kind::f16) in use; false once a pass fell back to tf32 pairs.
    bool fp16_pairs() const { return h16_; }
    int fallbacks() const { return fallbacks_; }
    // Strip sharding: from now on every pass computes only this rank's window-aligned
    // row strip of the image (Plan::make_strip), exchanging halo rows with the
    // neighbouring ranks over NCCL; `id` is the communicator's unique id (the same on
    // every rank). The output rows of the other ranks are not written.
    void attach_strip(int rank, int n, const void* id, size_t idlen);
    bool sharded() const { return comm_ != nullptr; }
    // Deadline of a sharded call's device work (seconds; <= 0: none): past it the
    // communicator is aborted and the call fails instead of blocking (see Comm::wait).
    void set_timeout(double s);

private:
    struct Acts;
    Plan plan_for(int h, int w) const;
    void upload_weights();
    int take_device_error();  // the error word's value (cleared on the device)
    void fall_back(int code);  // after ERR_RANGE_*: tf32 pairs (and the attention on CUDA cores)
    // Waits for the engine's stream: plainly, or with the communicator's deadline when sharded.
    void wait_stream();
    void refuse_if_aborted() const;  // throws once the communicator was aborted
    void ensure_plan(int h, int w);
    // Strip mode: fill `n` halo rows on each side of `plane` (`ch` channels, at `res`
    // times the base resolution) from the neighbours' own rows; top and bottom ranks
    // wrap around to each other (what the shifted windows need; elsewhere the rows
    // beyond the image are never read as data). No-op when not sharded.
    void exchange(float* plane, int ch, int res, int n, cudaStream_t st = nullptr);
    void exchange(Dst d, int ch, int res, int n);
    // A 3x3 conv over a plane at `res` times the base resolution. Sharded, the input is
    // read over the local rows that hold image data (the halo rows beyond the image's
    // top or bottom edge are left out, so the conv's zero padding applies there) and
    // only this strip's own output rows are computed unless `all_rows`.
    long conv_res(const std::string& wname, Opnd x, int xch, Dst y, int ych, int res, bool all_rows, Epi e);
    // Copies this pass's output (all of it, or the strip's own rows) from the arena.
    void copy_out(float* dst, cudaMemcpyKind kind, cudaStream_t st);
    void run_graph(cudaStream_t run);  // the whole pass over the internal din/dout buffers
    void enqueue_pass();               // the launch sequence itself
    void hab(int stage, int blk, const float* in, float* out);
    void ocab(int stage, const float* in, float* out);
    void mlp(const std::string& p, float* x, Dst out);
    void mark(const char* kind, double flops, double bytes);
    const float* W(const std::string& name) const;
    const GemmW& G(const std::string& name) const;
    long linear(const std::string& wname, Opnd x, Dst y, const Epi& e);
    // The same over `m` tokens from the given operand and output positions.
    long linear_m(const std::string& wname, Opnd x, Dst y, const Epi& e, long m);
    // This plan's own tokens: strip-sharded, the rows between the halos (pointwise layers
    // whose halo rows the next exchange overwrites compute only these); else the plane.
    long own_t0() const { return (long)plan_.halo * plan_.wp; }
    long own_tokens() const { return (long)plan_.own() * plan_.wp; }
    long conv(const std::string& wname, Opnd x, Dst y, int hgt, int wid, const Epi& e);
    // Operand planes: split into hi/lo halves when the tensor cores run in fp32-parity
    // mode (fp16 pairs when `h16_`, tf32 pairs otherwise), plain fp32 otherwise.
    bool split() const { return mode_ == 0 && !simt_only_; }
    Dst D(float* hi, float* lo) const {
        return split() ? Dst{hi, lo, h16_, derr_} : Dst{hi, nullptr, false, nullptr};
    }
    Opnd O(const float* hi, const float* lo) const { return split() ? Opnd{hi, lo, h16_} : Opnd{hi, nullptr, false}; }
    // Halo rows of a plane of `rowf` floats per row at `res` times the base resolution.
    void exchange_rows(float* plane, long rowf, int res, int n, cudaStream_t st = nullptr);

    Weights wt_;
    // The CAB's first conv as a per-tap linear + tap sum when its output is narrow
    // (9 * compressed <= 64): the linear reads the normed plane once instead of nine
    // times. tap_ld_ is the row stride of the per-tap plane (it borrows the qkv buffer).
    bool tap_cab_ = false;
    int tap_ld_ = 0;
    // fp16 split planes (kind::f16 GEMMs): parity mode with a width of a multiple of 8,
    // so every split plane's rows are whole 16-byte units. cmid_ld_: the CAB's middle
    // plane's channel stride in elements (16 or a multiple of 8 as fp16; the buffer's
    // own stride as tf32 pairs or fp32).
    bool h16_ = false;
    bool attn_simt_ = false;  // the attention on the fp32 CUDA-core kernels (after ERR_RANGE_ATTN)
    int fallbacks_ = 0;
    // conv_last runs on the bandwidth kernel (k_conv_last.cu) when its shape fits.
    bool cl_ok_ = false;
    // The CAB's second conv folded into proj (k_proj_cab): the gate-scaled conv weight in
    // the tensor-core layout (hi, lo) and the folded bias, rewritten by every HAB's gate
    // kernel; zero padding written once at upload.
    float *fold_hi_ = nullptr, *fold_lo_ = nullptr, *fold_bias_ = nullptr;
    bool fold_ok(const std::string& blk) const;
    int cmid_ld_ = 0;
    int device_ = 0, mode_ = 0;
    std::unique_ptr<Comm> comm_;
    double timeout_s_ = 120.0;
    // Sharded: a second stream for the collectives that overlap compute (the HABs' halo
    // exchange and channel-sum all-reduce), joined back by events.
    cudaStream_t cstream_ = nullptr;
    cudaEvent_t ev_fork_ = nullptr, ev_halo_ = nullptr, ev_ca_ = nullptr;
    bool use_graph_ = true, simt_only_ = false;
    cudaStream_t stream_ = nullptr;
    cudaEvent_t join_ = nullptr;
    float* dweights_ = nullptr;
    int* derr_ = nullptr;
    std::map<std::string, const float*> w_;
    std::map<std::string, GemmW> gw_;
    Plan plan_;
    bool have_plan_ = false;
    Sizes sizes_;
    float* arena_ = nullptr;
    size_t arena_floats_ = 0;  // capacity of the arena (plans no larger reuse it)
    std::unique_ptr<Acts> a_;
    cudaGraphExec_t graph_ = nullptr;
    int eager_runs_ = 0;
    uint64_t launches_ = 0;
    uint64_t per_pass_ = 0;  // kernel launches in one pass (counted on the eager run)
    struct Mark {
        std::string kind;
        double flops, bytes;
        cudaEvent_t ev;
    };
    bool profiling_ = false;
    std::vector<Mark> marks_;
};

}  // namespace hat
