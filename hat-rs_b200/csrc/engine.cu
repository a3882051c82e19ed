// The layer scheduler. Activations are token-major planes [hp][wp][c] (channels
// innermost), so a token linear is a plain row-major GEMM over the whole plane, a 3x3
// conv is an implicit GEMM over K = 9*cin, and the windowed attentions read their
// windows out of the qkv plane by address arithmetic. Every layer is one launch; the
// whole pass is captured once per plan in a CUDA graph and replayed.
#include "engine.h"

#include <algorithm>
#include <cmath>

#include "nccl_rt.h"
#include <cstring>
#include <sstream>

namespace hat {

// ------------------------------------------------------------------ sizes
Sizes Sizes::of(const Weights& wt, const Plan& p) {
    Sizes s;
    const long P = p.tokens(), c = wt.embed;
    s.cmid_stride = wt.compressed <= 8 ? 8 : (wt.compressed + 3) / 4 * 4;
    s.x0 = P * 3;
    s.body = P * c;
    s.xa = P * c;
    s.xb = P * c;
    s.n1 = P * c;
    s.n1lo = P * c;
    s.cmid = P * s.cmid_stride;
    s.cmidlo = P * s.cmid_stride;
    s.convx = P * c;
    s.qkv = P * 3 * c;
    s.attn = P * c;
    s.attnlo = P * c;
    s.hid = P * wt.mlp_ratio * c;
    s.hidlo = P * wt.mlp_ratio * c;
    // The channel-attention pool's partial sums: at most four rows of c per 128-pixel tile.
    s.chsum = (P + 127) / 128 * 4 * c;
    s.casum = c;
    s.gate = c;
    s.cabstat = 3L * wt.compressed * (p.rows + 2);
    // The head's planes ping-pong between two buffers: plane 0 (conv_before_upsample's
    // output, at P) and every other shuffled plane go to A, the rest to B.
    long res = P, a = P * wt.head_feat, b = 0;
    int i = 1;
    for (auto& blk : wt.up_blocks()) {
        res *= (long)blk.first * blk.first;
        long need = res * wt.head_feat;
        if (i % 2)
            b = std::max(b, need);
        else
            a = std::max(a, need);
        ++i;
    }
    s.headA = a;
    s.headAlo = a;
    s.headB = b;
    s.headBlo = b;
    s.din = 3L * p.h * p.w;
    s.dout = 3L * p.h * wt.scale * p.w * wt.scale;
    return s;
}

struct Engine::Acts {
    float *x0, *body, *xa, *xb, *n1, *n1lo, *cmid, *cmidlo, *convx, *qkv, *attn, *attnlo, *hid, *hidlo, *chsum,
        *casum, *gate, *headA, *headAlo, *headB, *headBlo, *din, *dout, *cabstat;
};

// ------------------------------------------------------------------ attention dispatch
void launch_window_attention_simt(const float* qkv, const float* table, Dst out, const Plan& p, int c, int heads,
                                  int shift, cudaStream_t st);
void launch_overlap_attention_simt(const float* qkv, const float* table, Dst out, const Plan& p, int c, int heads,
                                   cudaStream_t st);

void launch_attention_tc(int mode, bool oca, const float* qkv, const float* table, Dst out, const Plan& p, int c,
                         int heads, int shift, int* err, cudaStream_t st, bool pre = false);

// The tensor-core kernel in parity and fast modes; the CUDA-core one for the debug path.
void launch_window_attention(int mode, bool simt, const float* qkv, const float* table, Dst out, const Plan& p, int c,
                             int heads, int shift, int* err, cudaStream_t st, bool pre) {
    if (simt && (p.strip() || pre)) throw Error(1, "attention: strips and the pre-split layout need the tensor-core kernel");
    if (simt)
        launch_window_attention_simt(qkv, table, out, p, c, heads, shift, st);
    else
        launch_attention_tc(mode, false, qkv, table, out, p, c, heads, shift, err, st, pre);
}

void launch_overlap_attention(int mode, bool simt, const float* qkv, const float* table, Dst out, const Plan& p, int c,
                              int heads, int* err, cudaStream_t st, bool pre) {
    if (simt && (p.strip() || pre)) throw Error(1, "attention: strips and the pre-split layout need the tensor-core kernel");
    if (simt)
        launch_overlap_attention_simt(qkv, table, out, p, c, heads, st);
    else
        launch_attention_tc(mode, true, qkv, table, out, p, c, heads, 0, err, st, pre);
}

// ------------------------------------------------------------------ engine
static std::string fmt_bytes(double n) {
    char buf[64];
    double mib = n / 1048576.0;
    if (mib >= 1024.0)
        snprintf(buf, sizeof buf, "%.1f GiB", mib / 1024.0);
    else
        snprintf(buf, sizeof buf, "%.0f MiB", mib);
    return buf;
}

static const double SLACK = 1.05;            // src/memguard.rs:42
static const double BASE = 128.0 * 1048576;  // src/memguard.rs:49

static bool is_gemm_weight(const std::string& name, const TensorInfo& ti) {
    if (ti.shape.size() == 4 && ti.shape[2] == 3 && ti.shape[3] == 3) return true;  // 3x3 conv
    if (ti.shape.size() != 2) return false;
    // Linear weights; the relative-position tables are 2-D too but are not GEMM operands.
    return name.find("relative_position") == std::string::npos;
}

Engine::Engine(const std::string& path, int device, int mode, bool use_graph, bool simt_only)
    : device_(device), mode_(mode), use_graph_(use_graph), simt_only_(simt_only) {
    wt_.load(path);
    int ndev = 0;
    HAT_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev)
        throw Error(1, "device " + std::to_string(device) + " does not exist (" + std::to_string(ndev) + " visible)");
    HAT_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    HAT_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        throw Error(3, std::string("device ") + prop.name + " is compute capability " + std::to_string(prop.major) +
                           "." + std::to_string(prop.minor) + "; this backend is built for sm_100a only");
    // check_gpu_weights (src/memguard.rs:211-225)
    size_t fr = 0, tot = 0;
    HAT_CUDA(cudaMemGetInfo(&fr, &tot));
    if ((double)wt_.f32_bytes + BASE > (double)fr)
        throw Error(4, "not enough video memory for the checkpoint alone\nhat: " + wt_.variant + " uploads as " +
                           fmt_bytes((double)wt_.f32_bytes) + " of tensors, and " + fmt_bytes((double)fr) +
                           " is free on the device\nhat: a smaller checkpoint is what fits");
    HAT_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    HAT_CUDA(cudaEventCreateWithFlags(&join_, cudaEventDisableTiming));
    HAT_CUDA(cudaMalloc(&derr_, sizeof(int)));
    HAT_CUDA(cudaMemsetAsync(derr_, 0, sizeof(int), stream_));

    h16_ = split() && wt_.embed % 8 == 0;
    upload_weights();
}

// One device allocation: every f32 tensor as stored, then every GEMM operand in the
// kernels' layouts (CUDA-core layout, tensor-core hi/lo split as fp16 pairs when `h16_`,
// tf32 pairs otherwise). Called at construction and again when a pass falls back from
// fp16 to tf32 operand pairs.
void Engine::upload_weights() {
    if (dweights_) {
        HAT_CUDA(cudaStreamSynchronize(stream_));
        cudaFree(dweights_);
        dweights_ = nullptr;
    }
    w_.clear();
    gw_.clear();
    {
        auto it = wt_.st.tensors.find("conv_last.weight");
        cl_ok_ = it != wt_.st.tensors.end() && it->second.shape == std::vector<int64_t>{3, CL_CIN, 3, 3} &&
                 wt_.st.tensors.count("conv_last.bias");
    }
    const int cmid_stride = Sizes::of(wt_, Plan::make(16, 16, wt_.window)).cmid_stride;
    tap_cab_ = 9 * wt_.compressed <= 64;
    tap_ld_ = (9 * wt_.compressed + 3) / 4 * 4;
    // fp16 stride of the middle plane: 16 (one 32-byte k-step) or a multiple of 8; it
    // fits in the buffer's cmid_stride floats (cmid_stride >= max(compressed, 8)).
    cmid_ld_ = !h16_ ? cmid_stride : wt_.compressed <= 16 ? 16 : (wt_.compressed + 7) / 8 * 8;
    if (2 * cmid_ld_ > 4 * cmid_stride && h16_) throw Error(3, "gpu: the CAB's middle plane is too narrow");
    // h16 weights: the factor that puts the largest |w| of each weight near 2^14.
    auto h16_scale = [&](const std::string& name, const TensorInfo& ti) {
        const float* w = wt_.st.f32(name);
        float mx = 0.f;
        for (size_t i = 0, n = (size_t)ti.numel(); i < n; ++i) mx = std::max(mx, std::fabs(w[i]));
        return 1.f / h16_weight_factor(mx);
    };
    auto is_cab1 = [](const std::string& n) { return n.find("conv_block.cab.0.weight") != std::string::npos; };
    size_t total = 0;
    std::vector<std::string> names;
    for (auto& kv : wt_.st.tensors) {
        if (kv.second.dtype != "F32") continue;
        names.push_back(kv.first);
        total += ((size_t)kv.second.numel() + 63) / 64 * 64;
        if (is_gemm_weight(kv.first, kv.second)) {
            GemmW g;
            const auto& s = kv.second.shape;
            if (s.size() == 4) {
                const bool cab2 = kv.first.find("conv_block.cab.2.weight") != std::string::npos;
                plan_gemm_w(g, (int)s[0], (int)s[1], true, cab2 ? cmid_ld_ : (int)s[1], h16_);
            } else {
                plan_gemm_w(g, (int)s[0], (int)s[1], false, 0, h16_);
            }
            if (g.h16) g.scale = h16_scale(kv.first, kv.second);
            gw_[kv.first] = g;
            total += (gemm_w_floats(g) + 64) / 64 * 64 + 192;
            if (tap_cab_ && is_cab1(kv.first)) {
                GemmW t;
                plan_gemm_w(t, 9 * (int)s[0], (int)s[1], false, 0, h16_);
                t.scale = g.scale;  // the same values, reordered
                gw_[kv.first + "#taps"] = t;
                total += ((size_t)t.n * t.k + 63) / 64 * 64 + (gemm_w_floats(t) + 64) / 64 * 64 + 192;
            }
        }
    }
    // The folded conv weight and bias (one set, rewritten by each HAB's gate kernel).
    size_t fold_off = total, fold_n = 0;
    for (auto& kv : gw_)
        if (kv.first.find("conv_block.cab.2.weight") != std::string::npos && kv.second.umma) {
            fold_n = ((size_t)kv.second.n_pad * kv.second.k_pad + 63) / 64 * 64;
            total += 2 * fold_n + ((size_t)kv.second.n_pad + 63) / 64 * 64;
            break;
        }
    HAT_CUDA(cudaMalloc(&dweights_, total * sizeof(float)));
    fold_hi_ = fold_lo_ = fold_bias_ = nullptr;
    if (fold_n) {
        fold_hi_ = dweights_ + fold_off;
        fold_lo_ = fold_hi_ + fold_n;
        fold_bias_ = fold_lo_ + fold_n;
        HAT_CUDA(cudaMemsetAsync(fold_hi_, 0, (total - fold_off) * sizeof(float), stream_));
    }
    size_t off = 0;
    uint64_t* prev = g_launch_counter;
    g_launch_counter = &launches_;
    try {
        for (auto& name : names) {
            const TensorInfo& ti = wt_.st.tensors[name];
            size_t n = (size_t)ti.numel();
            float* d = dweights_ + off;
            HAT_CUDA(cudaMemcpyAsync(d, wt_.st.f32(name), n * sizeof(float), cudaMemcpyHostToDevice, stream_));
            w_[name] = d;
            off += (n + 63) / 64 * 64;
            auto it = gw_.find(name);
            if (it != gw_.end()) {
                GemmW& g = it->second;
                float* simt = dweights_ + off;
                off += ((size_t)g.n * g.k + 63) / 64 * 64;
                float *hi = nullptr, *lo = nullptr;
                if (g.umma) {
                    hi = dweights_ + off;
                    off += ((size_t)g.n_pad * g.k_pad + 63) / 64 * 64;
                    lo = dweights_ + off;
                    off += ((size_t)g.n_pad * g.k_pad + 63) / 64 * 64;
                }
                launch_prep_gemm_w(d, simt, hi, lo, g, stream_);
                g.simt = simt;
                g.hi = hi;
                g.lo = lo;
                if (tap_cab_ && is_cab1(name)) {
                    GemmW& t = gw_[name + "#taps"];
                    float* taps = dweights_ + off;
                    off += ((size_t)t.n * t.k + 63) / 64 * 64;
                    launch_prep_taps(d, taps, wt_.compressed, wt_.embed, stream_);
                    float* tsimt = dweights_ + off;
                    off += ((size_t)t.n * t.k + 63) / 64 * 64;
                    float *thi = nullptr, *tlo = nullptr;
                    if (t.umma) {
                        thi = dweights_ + off;
                        off += ((size_t)t.n_pad * t.k_pad + 63) / 64 * 64;
                        tlo = dweights_ + off;
                        off += ((size_t)t.n_pad * t.k_pad + 63) / 64 * 64;
                    }
                    launch_prep_gemm_w(taps, tsimt, thi, tlo, t, stream_);
                    t.simt = tsimt;
                    t.hi = thi;
                    t.lo = tlo;
                }
            }
        }
    } catch (...) {
        g_launch_counter = prev;
        throw;
    }
    g_launch_counter = prev;
    if (off > fold_off) throw Error(3, "gpu: weight arena overflow");
    HAT_CUDA(cudaStreamSynchronize(stream_));
}


Engine::~Engine() {
    cudaSetDevice(device_);
    if (graph_) cudaGraphExecDestroy(graph_);
    for (auto& m : marks_) cudaEventDestroy(m.ev);
    if (arena_) cudaFree(arena_);
    if (dweights_) cudaFree(dweights_);
    if (derr_) cudaFree(derr_);
    if (join_) cudaEventDestroy(join_);
    for (cudaEvent_t ev : {ev_fork_, ev_halo_, ev_ca_})
        if (ev) cudaEventDestroy(ev);
    if (cstream_) cudaStreamDestroy(cstream_);
    if (stream_) cudaStreamDestroy(stream_);
}

const float* Engine::W(const std::string& name) const {
    auto it = w_.find(name);
    if (it == w_.end()) throw Error(2, "gpu: no weight `" + name + "`");
    return it->second;
}

const GemmW& Engine::G(const std::string& name) const {
    auto it = gw_.find(name);
    if (it == gw_.end()) throw Error(2, "gpu: no GEMM weight `" + name + "`");
    return it->second;
}

long Engine::linear(const std::string& wname, Opnd x, Dst y, const Epi& e) {
    GemmCtx c{mode_, simt_only_, derr_};
    return gemm_linear(c, x, G(wname), y, plan_.tokens(), e, stream_);
}

long Engine::linear_m(const std::string& wname, Opnd x, Dst y, const Epi& e, long m) {
    GemmCtx c{mode_, simt_only_, derr_};
    return gemm_linear(c, x, G(wname), y, m, e, stream_);
}

long Engine::conv(const std::string& wname, Opnd x, Dst y, int hgt, int wid, const Epi& e) {
    if (wname == "conv_last.weight" && e.planar_out && cl_ok_ && !simt_only_ && conv_last_ok(x, CL_CIN, 3))
        return launch_conv_last(x, W("conv_last.weight"), W("conv_last.bias"), y.hi, hgt, wid, e, stream_);
    GemmCtx c{mode_, simt_only_, derr_};
    return gemm_conv3x3(c, x, G(wname), y, hgt, wid, e, stream_);
}

// Halo rows a strip holds on each side: the shifted windows reach 8 rows (win / 2) past a
// window-aligned strip, the OCAB keys 4, a 3x3 conv 1.
static const int STRIP_HALO = 8;

Plan Engine::plan_for(int h, int w) const {
    if (comm_) return Plan::make_strip(h, w, wt_.window, comm_->rank(), comm_->size(), STRIP_HALO);
    return Plan::make(h, w, wt_.window);
}

size_t Engine::footprint_bytes(int h, int w) const {
    return (size_t)Sizes::of(wt_, plan_for(h, w)).total() * sizeof(float);
}

void Engine::attach_strip(int rank, int n, const void* id, size_t idlen) {
    HAT_CUDA(cudaSetDevice(device_));
    if (simt_only_) throw Error(1, "strip sharding needs the tensor-core kernels (simt_only is set)");
    if (wt_.window != 16) throw Error(1, "strip sharding is built for window 16");
    if (graph_) {
        cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
    }
    if (arena_) {
        HAT_CUDA(cudaStreamSynchronize(stream_));
        cudaFree(arena_);
        arena_ = nullptr;
        arena_floats_ = 0;
    }
    have_plan_ = false;
    comm_.reset(new Comm(rank, n, id, idlen, device_, timeout_s_));
    if (!cstream_) {
        HAT_CUDA(cudaStreamCreateWithFlags(&cstream_, cudaStreamNonBlocking));
        HAT_CUDA(cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming));
        HAT_CUDA(cudaEventCreateWithFlags(&ev_halo_, cudaEventDisableTiming));
        HAT_CUDA(cudaEventCreateWithFlags(&ev_ca_, cudaEventDisableTiming));
    }
}

void Engine::exchange(float* plane, int ch, int res, int n, cudaStream_t st) {
    exchange_rows(plane, (long)plan_.wp * res * ch, res, n, st);
}

void Engine::exchange_rows(float* plane, long rowf, int res, int n, cudaStream_t st) {
    if (!st) st = stream_;
    if (!comm_) return;
    const Plan& p = plan_;
    if (n > p.halo * res) throw Error(1, "exchange: more rows than the halo holds");
    const int top = p.halo * res, bot = (p.halo + p.own()) * res;  // first own row, first bottom-halo row
    const int N = comm_->size(), r = comm_->rank();
    const int up = (r - 1 + N) % N, down = (r + 1) % N;
    // Matched per peer in posting order: a rank's first send (its top rows, to `up`) is
    // the up rank's first receive (from its `down`), and likewise for the second pair.
    comm_->group_start();
    comm_->send(plane + top * rowf, n * rowf, up, st);
    comm_->send(plane + (bot - n) * rowf, n * rowf, down, st);
    comm_->recv(plane + bot * rowf, n * rowf, down, st);
    comm_->recv(plane + (top - n) * rowf, n * rowf, up, st);
    comm_->group_end();
}

void Engine::exchange(Dst d, int ch, int res, int n) {
    if (d.lo && d.h16) {
        // fp16 rows: half the floats (wp is a multiple of 16, so rows stay whole floats)
        const long rowf = (long)plan_.wp * res * ch / 2;
        exchange_rows(d.hi, rowf, res, n);
        exchange_rows(d.lo, rowf, res, n);
        return;
    }
    exchange(d.hi, ch, res, n);
    if (d.lo) exchange(d.lo, ch, res, n);
}

long Engine::conv_res(const std::string& wname, Opnd x, int xch, Dst y, int ych, int res, bool all_rows, Epi e) {
    const Plan& p = plan_;
    const int wid = p.wp * res, R = p.rows * res;
    int lo = 0, hi = R;
    if (p.strip()) {
        if (p.r0 == 0) lo = p.halo * res;                // above the image: zero padding
        if (p.r1 == p.hp) hi = (p.halo + p.own()) * res;  // below the image
    }
    const long xoff = (long)lo * wid * xch;
    Opnd xv = opnd_at(x, xoff);
    long yoff = 0;
    if (e.planar_out)
        e.oy0 += p.gy0() * res + lo;  // padded output row of view row 0
    else if (e.shuffle)
        yoff = (long)lo * e.shuffle * wid * e.shuffle * ych;
    else
        yoff = (long)lo * wid * ych;
    Dst yv = dst_at(y, yoff);
    if (e.res) e.res += yoff;
    if (e.cx) e.cx += yoff;
    if (p.strip() && !all_rows) {
        e.y_lo = p.halo * res - lo;
        e.y_hi = (p.halo + p.own()) * res - lo;
    }
    return conv(wname, xv, yv, hi - lo, wid, e);
}

void Engine::copy_out(float* dst, cudaMemcpyKind kind, cudaStream_t st) {
    const Plan& p = plan_;
    const long OH = (long)p.h * wt_.scale, OW = (long)p.w * wt_.scale;
    if (!p.strip()) {
        HAT_CUDA(cudaMemcpyAsync(dst, a_->dout, 3 * OH * OW * sizeof(float), kind, st));
        return;
    }
    const long a = (long)p.r0 * wt_.scale, b = std::min<long>((long)p.r1 * wt_.scale, OH);
    for (int ch = 0; ch < 3 && a < b; ++ch) {
        const long off = (ch * OH + a) * OW;
        HAT_CUDA(cudaMemcpyAsync(dst + off, a_->dout + off, (b - a) * OW * sizeof(float), kind, st));
    }
}

void Engine::check_memory(int h, int w) const {
    // check_gpu (src/memguard.rs:183-201)
    double acts = (double)footprint_bytes(h, w);
    double need = acts * SLACK + (double)wt_.f32_bytes + BASE;
    size_t fr = 0, tot = 0;
    HAT_CUDA(cudaSetDevice(device_));
    HAT_CUDA(cudaMemGetInfo(&fr, &tot));
    // The engine's current arena is released before a new plan allocates, so it counts.
    double avail = (double)fr + (arena_ ? (double)arena_floats_ * sizeof(float) : 0.0);
    if (need > avail) {
        std::ostringstream o;
        o << "not enough video memory for a " << w << "x" << h << " pass on the GPU\n"
          << "hat: it needs about " << fmt_bytes(need) << " (" << fmt_bytes(acts) << " of device buffers + "
          << fmt_bytes((double)wt_.f32_bytes) << " of weights + " << fmt_bytes(BASE) << " of runtime, plus " << 5
          << "% of slack); " << fmt_bytes(avail) << " is free on the device\n"
          << "hat: `--mem` runs it in tiles on the device (each tile allocates its own buffers, so the "
             "tile's size is the number that must fit); a smaller image does too";
        throw Error(4, o.str());
    }
}

int Engine::take_device_error() {
    int v = 0;
    HAT_CUDA(cudaMemcpyAsync(&v, derr_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    HAT_CUDA(cudaStreamSynchronize(stream_));
    if (v) HAT_CUDA(cudaMemsetAsync(derr_, 0, sizeof(int), stream_));
    return v;
}

static void raise_device_error(int v) {
    if (!v) return;
    if (v == ERR_RANGE_ATTN)
        throw Error(3, "gpu: an attention operand (q, k or v) reached fp16's range (|x| >= 65504), which the "
                       "tensor-core split cannot carry (code " + std::to_string(v) + "); the pass's output is invalid");
    if (v == ERR_RANGE_GEMM)
        throw Error(3, "gpu: an activation reached fp16's range (|x| >= 65504), which the fp16 operand split "
                       "cannot carry (code " + std::to_string(v) + "); the pass's output is invalid");
    throw Error(3, "gpu: a tensor-core kernel gave up waiting on its pipeline (code " + std::to_string(v) +
                       "); the pass's output is invalid");
}

void Engine::check_device_error() { raise_device_error(take_device_error()); }

void Engine::set_timeout(double s) {
    timeout_s_ = s;
    if (comm_) comm_->set_timeout(s);
}

void Engine::refuse_if_aborted() const {
    // After an abort the communicator's buffers are gone, while the captured pass still names
    // them: nothing may be enqueued any more, and the stream is not waited on either.
    if (comm_ && comm_->aborted())
        throw Error(3, "nccl: the communicator was aborted after a failed or timed-out exchange; attach the "
                       "strips again to continue");
}

void Engine::sync() {
    refuse_if_aborted();
    HAT_CUDA(cudaSetDevice(device_));
    wait_stream();
    check_device_error();
}

void Engine::wait_stream() {
    if (comm_)
        comm_->wait(stream_, timeout_s_);
    else
        HAT_CUDA(cudaStreamSynchronize(stream_));
}

// fp16 operand pairs carry 22 significant bits but only fp16's exponent range; a value of
// 65504 or more sets ERR_RANGE_GEMM (a GEMM operand plane) or ERR_RANGE_ATTN (q, k or v).
// The weights are prepared again as tf32 pairs (the same 22 bits with fp32's exponent
// range), the arena is cleared (the planes change layout) and the handle stays on tf32
// pairs from then on. The tensor-core attention splits its operands into fp16 pairs in
// every mode, so an attention operand out of that range moves the attention to the fp32
// CUDA-core kernels as well.
void Engine::fall_back(int code) {
    HAT_CUDA(cudaStreamSynchronize(stream_));
    if (graph_) {
        cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
    }
    if (code == ERR_RANGE_ATTN) attn_simt_ = true;
    if (h16_) {
        h16_ = false;
        upload_weights();
    }
    have_plan_ = false;  // the next ensure_plan clears the arena
    eager_runs_ = 0;
    ++fallbacks_;
}

void Engine::ensure_plan(int h, int w) {
    Plan p = plan_for(h, w);
    if (have_plan_ && p == plan_) return;
    Sizes s = Sizes::of(wt_, p);
    if (graph_) {
        cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
    }
    if (arena_ && (size_t)s.total() <= arena_floats_) {
        // A plan no larger than the arena (a smaller tile, say) is carved out of it.
        wait_stream();
    } else {
        check_memory(h, w);
        if (arena_) {
            wait_stream();
            cudaFree(arena_);
            arena_ = nullptr;
            arena_floats_ = 0;
            have_plan_ = false;
        }
        HAT_CUDA(cudaMalloc(&arena_, (size_t)s.total() * sizeof(float)));
        arena_floats_ = (size_t)s.total();
    }
    HAT_CUDA(cudaMemsetAsync(arena_, 0, (size_t)s.total() * sizeof(float), stream_));
    a_.reset(new Acts);
    float* q = arena_;
    auto take = [&](long n) {
        float* r = q;
        q += n;
        return r;
    };
    a_->x0 = take(s.x0);
    a_->body = take(s.body);
    a_->xa = take(s.xa);
    a_->xb = take(s.xb);
    a_->n1 = take(s.n1);
    a_->n1lo = take(s.n1lo);
    a_->cmid = take(s.cmid);
    a_->cmidlo = take(s.cmidlo);
    a_->convx = take(s.convx);
    a_->qkv = take(s.qkv);
    a_->attn = take(s.attn);
    a_->attnlo = take(s.attnlo);
    a_->hid = take(s.hid);
    a_->hidlo = take(s.hidlo);
    a_->chsum = take(s.chsum);
    a_->casum = take(s.casum);
    a_->gate = take(s.gate);
    a_->headA = take(s.headA);
    a_->headAlo = take(s.headAlo);
    a_->headB = take(s.headB);
    a_->headBlo = take(s.headBlo);
    a_->din = take(s.din);
    a_->dout = take(s.dout);
    a_->cabstat = take(s.cabstat);
    // THE PREDICTION IS HELD TO THE ALLOCATION (src/gpu.rs:779-786).
    if (q - arena_ != s.total()) throw Error(3, "gpu: the buffer set does not match the guard's prediction");
    plan_ = p;
    sizes_ = s;
    have_plan_ = true;
    eager_runs_ = 0;
}

// `out = x + fc2(gelu(fc1(norm2(x))))` (src/gpu.rs:449-466). `out` may be `x` itself,
// or the split n1 planes when the result feeds only the stage's conv. Strip-sharded, it
// runs over the strip's own rows: the next layer's halo exchange overwrites the others.
void Engine::mlp(const std::string& p, float* x, Dst out) {
    const long t0 = own_t0(), P = own_tokens();
    const int c = wt_.embed, hid = wt_.mlp_ratio * c;
    float* xo = x + t0 * c;
    const Dst n1 = dst_at(D(a_->n1, a_->n1lo), t0 * c);
    const Opnd n1o = opnd_at(O(a_->n1, a_->n1lo), t0 * c);
    const Dst yo = dst_at(out, t0 * c);
    mark("layernorm", 0, 8.0 * P * c);
    launch_layernorm(xo, W(p + ".norm2.weight"), W(p + ".norm2.bias"), n1, P, c, stream_);
    const GemmW& w1 = G(p + ".mlp.fc1.weight");
    const GemmW& w2 = G(p + ".mlp.fc2.weight");
    if (!simt_only_ && umma_mlp_ok(w1, w2)) {
        // fc1 + GELU + fc2 + residual in one launch, the hidden plane never written out.
        mark("mlp.fused", 4.0 * P * hid * c, 4.0 * P * (2 * c + c));
        umma_mlp(mode_, n1o, w1, W(p + ".mlp.fc1.bias"), w2, W(p + ".mlp.fc2.bias"), xo, yo, P, derr_, stream_);
        return;
    }
    Epi e1;
    e1.bias = W(p + ".mlp.fc1.bias");
    e1.act = ACT_GELU;
    mark("linear.fc1", 2.0 * P * hid * c, 4.0 * P * (c + hid));
    linear_m(p + ".mlp.fc1.weight", n1o, dst_at(D(a_->hid, a_->hidlo), t0 * hid), e1, P);
    Epi e2;
    e2.bias = W(p + ".mlp.fc2.bias");
    e2.res = xo;
    mark("linear.fc2", 2.0 * P * hid * c, 4.0 * P * (hid + 2 * c));
    linear_m(p + ".mlp.fc2.weight", opnd_at(O(a_->hid, a_->hidlo), t0 * hid), yo, e2, P);
}

// Whether block `blk`'s CAB conv folds into its proj (k_proj_cab): tensor cores in use,
// both weights in layouts the fused kernel takes, and patch-aligned planes.
bool Engine::fold_ok(const std::string& blk) const {
    if (simt_only_ || !fold_hi_ || plan_.wp % 16 || plan_.rows % 8 || wt_.compressed > 64) return false;
    if (plan_.strip() && (plan_.halo % 8 || plan_.own() % 8)) return false;
    const GemmW& w2 = G(blk + ".conv_block.cab.2.weight");
    const GemmW& wpj = G(blk + ".attn.proj.weight");
    if (!umma_proj_cab_ok(wpj, w2)) return false;
    // parity mode: the operand planes are split the way the weights are
    return mode_ != 0 || wpj.h16 == h16_;
}

// One HAB (hat_arch.py:266-309; src/gpu.rs:469-520): `in` is the block input, `out`
// its output (may be the same buffer).
void Engine::hab(int stage, int blk, const float* in, float* out) {
    const long P = plan_.tokens();
    const int c = wt_.embed, cc = wt_.compressed;
    const std::string p = "layers." + std::to_string(stage) + ".residual_group.blocks." + std::to_string(blk);
    const std::string cb = p + ".conv_block.cab";
    mark("layernorm", 0, 8.0 * P * c);
    const float *g1 = W(p + ".norm1.weight"), *b1 = W(p + ".norm1.bias");
    if (comm_) {
        // Sharded: the block input's halo rows (the shifted windows reach 8 rows out) travel on
        // the communication stream while LayerNorm runs over the strip's own rows; the halo rows'
        // LayerNorm follows once they have arrived.
        const long t0 = own_t0(), Po = own_tokens(), rowt = plan_.wp;
        HAT_CUDA(cudaEventRecord(ev_fork_, stream_));
        HAT_CUDA(cudaStreamWaitEvent(cstream_, ev_fork_, 0));
        exchange(const_cast<float*>(in), c, 1, plan_.halo, cstream_);
        HAT_CUDA(cudaEventRecord(ev_halo_, cstream_));
        launch_layernorm(in + t0 * c, g1, b1, dst_at(D(a_->n1, a_->n1lo), t0 * c), Po, c, stream_);
        HAT_CUDA(cudaStreamWaitEvent(stream_, ev_halo_, 0));
        const long tb = t0 + Po, nb = P - tb;  // the bottom halo rows
        launch_layernorm(in, g1, b1, D(a_->n1, a_->n1lo), (long)plan_.halo * rowt, c, stream_);
        launch_layernorm(in + tb * c, g1, b1, dst_at(D(a_->n1, a_->n1lo), tb * c), nb, c, stream_);
    } else {
        launch_layernorm(in, g1, b1, D(a_->n1, a_->n1lo), P, c, stream_);
    }
    // CAB: conv c→cc + GELU; conv cc→c with per-tile channel sums of its output; the gate.
    Epi ec1;
    ec1.bias = W(cb + ".0.bias");
    ec1.act = ACT_GELU;
    ec1.ldo = cmid_ld_;
    mark("conv.cab1", 18.0 * P * c * cc, 4.0 * P * (c + cc));
    if (tap_cab_) {
        // Per-tap partial outputs into the (not yet used) qkv buffer, then the tap sum.
        Epi et;
        et.ldo = tap_ld_;
        linear(cb + ".0.weight#taps", O(a_->n1, a_->n1lo), Dst{a_->qkv, nullptr}, et);
        // Rows beyond the image (a strip's halo at the top or bottom edge) are padding.
        const int ylo = plan_.strip() && plan_.r0 == 0 ? plan_.halo : 0;
        const int yhi = plan_.strip() && plan_.r1 == plan_.hp ? plan_.halo + plan_.own() : plan_.rows;
        launch_tapsum_gelu(a_->qkv, tap_ld_, W(cb + ".0.bias"), D(a_->cmid, a_->cmidlo), cmid_ld_, cc,
                           plan_.rows, plan_.wp, ylo, yhi, stream_);
    } else {
        // Every row: the second conv reads one row past the strip's own rows.
        conv_res(cb + ".0.weight", O(a_->n1, a_->n1lo), c, D(a_->cmid, a_->cmidlo), cmid_ld_, 1, true, ec1);
    }
    // The second conv: folded into proj (its output never written; the pool's sums taken
    // from its input), or on its own with per-tile channel sums of its output.
    const bool fold = fold_ok(p);
    // its input view: the plane's rows inside the image; output rows: the strip's own
    int vlo = 0, vhi = plan_.rows;
    if (plan_.strip()) {
        if (plan_.r0 == 0) vlo = plan_.halo;
        if (plan_.r1 == plan_.hp) vhi = plan_.halo + plan_.own();
    }
    const int ylo = plan_.strip() ? plan_.halo : 0, yhi = plan_.strip() ? plan_.halo + plan_.own() : plan_.rows;
    long rows = 1;
    if (fold) {
        mark("cab.pool", 0, 4.0 * P * cc);
        launch_cab_pool(opnd_at(O(a_->cmid, a_->cmidlo), (long)vlo * plan_.wp * cmid_ld_), cmid_ld_, cc, plan_.wp,
                        vhi - vlo, ylo - vlo, yhi - vlo, a_->cabstat, W(cb + ".2.weight"), W(cb + ".2.bias"), c,
                        a_->chsum, stream_);
    } else {
        Epi ec2;
        ec2.bias = W(cb + ".2.bias");
        ec2.colsum = a_->chsum;
        mark("conv.cab2", 18.0 * P * c * cc, 4.0 * P * (c + cc));
        rows = conv_res(cb + ".2.weight", O(a_->cmid, a_->cmidlo), cmid_ld_, Dst{a_->convx, nullptr}, c, 1, false,
                        ec2);
    }
    // The pool averages over the whole padded plane (src/gpu.rs:435); sharded, the
    // strips' channel sums are added across ranks first, on the communication stream while
    // the qkv linear and the attention run (the gate is first needed by proj).
    const float inv_count = 1.f / (float)((long)plan_.hp * plan_.wp);
    const float* pooled = a_->chsum;
    if (comm_) {
        launch_rowsum(a_->chsum, rows, c, a_->casum, stream_);
        HAT_CUDA(cudaEventRecord(ev_fork_, stream_));
        HAT_CUDA(cudaStreamWaitEvent(cstream_, ev_fork_, 0));
        comm_->allreduce_sum(a_->casum, c, cstream_);
        HAT_CUDA(cudaEventRecord(ev_ca_, cstream_));
        pooled = a_->casum;
        rows = 1;
    }
    // Attention on the normed plane; odd blocks are shifted by win/2 with the mask. With fp16
    // operand pairs and head dim 24, the qkv linear writes q (pre-scaled by scale * log2(e)),
    // k and v^T as the pairs the attention kernel copies (Epi::qkv_split).
    Epi eq;
    eq.bias = W(p + ".attn.qkv.bias");
    const bool pre = h16_ && c / wt_.heads == 24 && c % wt_.heads == 0 && G(p + ".attn.qkv.weight").umma;
    if (pre) {
        eq.qkv_split = a_->qkv;
        eq.qscale = 1.f / sqrtf(24.f) * 1.4426950408889634f;
        eq.qcols = c;
    }
    mark("linear.qkv", 6.0 * P * c * c, 16.0 * P * c);
    linear(p + ".attn.qkv.weight", O(a_->n1, a_->n1lo), Dst{a_->qkv, nullptr}, eq);
    const int shift = blk % 2 ? plan_.shift : 0;
    mark("attn.window", 4.0 * P * 256 * c, 16.0 * P * c);
    launch_window_attention(mode_, simt_only_ || attn_simt_, a_->qkv, W(p + ".attn.relative_position_bias_table"),
                            D(a_->attn, a_->attnlo), plan_, c, wt_.heads, shift, derr_, stream_, pre);
    // The channel-attention gate.
    mark("ca_gate", 0, 4.0 * rows * c);
    if (comm_) HAT_CUDA(cudaStreamWaitEvent(stream_, ev_ca_, 0));
    CabFold cf;
    if (fold) {
        const GemmW& w2 = G(cb + ".2.weight");
        const GemmW& wpj = G(p + ".attn.proj.weight");
        cf.w = W(cb + ".2.weight");
        cf.b2 = W(cb + ".2.bias");
        cf.bp = W(p + ".attn.proj.bias");
        cf.cs = wt_.conv_scale;
        cf.factor = wpj.h16 ? 1.f / wpj.scale : 1.f;
        cf.cc = cc;
        cf.cinp = w2.cinp;
        cf.k_pad = w2.k_pad;
        cf.h16 = w2.h16;
        cf.hi = fold_hi_;
        cf.lo = fold_lo_;
        cf.bias = fold_bias_;
        cf.err = derr_;
    }
    launch_ca_gate(pooled, rows, inv_count, W(cb + ".3.attention.1.weight"), W(cb + ".3.attention.1.bias"),
                   W(cb + ".3.attention.3.weight"), W(cb + ".3.attention.3.bias"), a_->gate, c, wt_.squeezed,
                   stream_, cf);
    // (over the strip's own rows when sharded: the next block exchanges the halo rows)
    const long t0 = own_t0(), Po = own_tokens();
    if (fold) {
        // proj + the gated conv in one accumulator, the residual in its epilogue.
        mark("linear.proj_cab", 2.0 * Po * c * c + 18.0 * Po * c * cc, 12.0 * Po * c);
        const Opnd cm = opnd_at(O(a_->cmid, a_->cmidlo), (long)vlo * plan_.wp * cmid_ld_);
        umma_proj_cab(mode_, O(a_->attn, a_->attnlo), G(p + ".attn.proj.weight"), cm, cmid_ld_, vhi - vlo, vlo,
                      G(cb + ".2.weight"), fold_hi_, fold_lo_, fold_bias_, in, out, plan_.rows, plan_.wp, ylo, yhi,
                      derr_, stream_);
        mlp(p, out, Dst{out, nullptr});
        return;
    }
    // proj, then `(shortcut + attn) + conv_x * conv_scale` in the epilogue.
    Epi ep;
    ep.bias = W(p + ".attn.proj.bias");
    ep.res = in + t0 * c;
    ep.cx = a_->convx + t0 * c;
    ep.gate = a_->gate;
    ep.cscale = wt_.conv_scale;
    mark("linear.proj", 2.0 * Po * c * c, 16.0 * Po * c);
    linear_m(p + ".attn.proj.weight", opnd_at(O(a_->attn, a_->attnlo), t0 * c), Dst{out + t0 * c, nullptr}, ep, Po);
    mlp(p, out, Dst{out, nullptr});
}

// The OCAB (hat_arch.py:392-438; src/gpu.rs:533-588). Its result feeds only the
// stage's 3x3 conv, so the last MLP writes it (split) into the n1 planes.
void Engine::ocab(int stage, const float* in, float* out) {
    const long P = plan_.tokens();
    const int c = wt_.embed;
    const std::string p = "layers." + std::to_string(stage) + ".residual_group.overlap_attn";
    exchange(const_cast<float*>(in), c, 1, plan_.halo);  // the keys reach 4 rows out
    mark("layernorm", 0, 8.0 * P * c);
    launch_layernorm(in, W(p + ".norm1.weight"), W(p + ".norm1.bias"), D(a_->n1, a_->n1lo), P, c, stream_);
    Epi eq;
    eq.bias = W(p + ".qkv.bias");
    const bool pre = h16_ && c / wt_.heads == 24 && c % wt_.heads == 0 && G(p + ".qkv.weight").umma;
    if (pre) {  // as in the HAB: q, k and v^T written as the attention kernel's fp16 pairs
        eq.qkv_split = a_->qkv;
        eq.qscale = 1.f / sqrtf(24.f) * 1.4426950408889634f;
        eq.qcols = c;
    }
    mark("linear.qkv", 6.0 * P * c * c, 16.0 * P * c);
    linear(p + ".qkv.weight", O(a_->n1, a_->n1lo), Dst{a_->qkv, nullptr}, eq);
    mark("attn.overlap", 4.0 * P * 576 * c, 16.0 * P * c);
    launch_overlap_attention(mode_, simt_only_ || attn_simt_, a_->qkv, W(p + ".relative_position_bias_table"),
                             D(a_->attn, a_->attnlo), plan_, c, wt_.heads, derr_, stream_, pre);
    const long t0 = own_t0(), Po = own_tokens();
    Epi ep;
    ep.bias = W(p + ".proj.bias");
    ep.res = in + t0 * c;
    mark("linear.proj", 2.0 * Po * c * c, 12.0 * Po * c);
    linear_m(p + ".proj.weight", opnd_at(O(a_->attn, a_->attnlo), t0 * c), Dst{out + t0 * c, nullptr}, ep, Po);
    mlp(p, out, D(a_->n1, a_->n1lo));
}

// The whole forward over din → dout (hat_arch.py:971-984; src/gpu.rs:714-748).
void Engine::enqueue_pass() {
    const Plan& pl = plan_;
    const long P = pl.tokens();
    const int c = wt_.embed, feat = wt_.head_feat;
    mark("pre", 0, 24.0 * P);
    launch_pre(a_->din, a_->x0, pl, wt_.mean, wt_.img_range, stream_);
    Epi ef;
    ef.bias = W("conv_first.bias");
    mark("conv.first", 54.0 * P * c, 4.0 * P * (3 + c));
    conv_res("conv_first.weight", Opnd{a_->x0, nullptr}, 3, Dst{a_->body, nullptr}, c, 1, false, ef);
    // The LayerNorms of the body run over the strip's own rows (the halo rows of their
    // outputs are exchanged before they are read).
    const long t0 = own_t0(), Po = own_tokens();
    mark("layernorm", 0, 8.0 * Po * c);
    launch_layernorm(a_->body + t0 * c, W("patch_embed.norm.weight"), W("patch_embed.norm.bias"),
                     Dst{a_->xa + t0 * c, nullptr}, Po, c, stream_);
    // The stage input stays in `xa` (the RHAG residual); the blocks run in `xb`, the OCAB
    // leaves the stage's result split in n1, and the stage conv adds xa back into xa.
    for (size_t s = 0; s < wt_.depths.size(); ++s) {
        const float* in = a_->xa;
        for (int b = 0; b < wt_.depths[s]; ++b) {
            hab((int)s, b, in, a_->xb);
            in = a_->xb;
        }
        ocab((int)s, in, a_->xb);
        Epi er;
        er.bias = W("layers." + std::to_string(s) + ".conv.bias");
        er.res = a_->xa;
        exchange(D(a_->n1, a_->n1lo), c, 1, 1);
        mark("conv.rhag", 18.0 * P * c * c, 12.0 * P * c);
        conv_res("layers." + std::to_string(s) + ".conv.weight", O(a_->n1, a_->n1lo), c, Dst{a_->xa, nullptr}, c, 1,
                 false, er);
    }
    mark("layernorm", 0, 8.0 * Po * c);
    launch_layernorm(a_->xa + t0 * c, W("norm.weight"), W("norm.bias"), dst_at(D(a_->n1, a_->n1lo), t0 * c), Po, c,
                     stream_);
    Epi eb;
    eb.bias = W("conv_after_body.bias");
    eb.res = a_->body;
    exchange(D(a_->n1, a_->n1lo), c, 1, 1);
    mark("conv.body", 18.0 * P * c * c, 12.0 * P * c);
    conv_res("conv_after_body.weight", O(a_->n1, a_->n1lo), c, D(a_->attn, a_->attnlo), c, 1, false, eb);
    // Head: conv + LeakyReLU, then per block a conv whose store does the PixelShuffle.
    Epi eh;
    eh.bias = W("conv_before_upsample.0.bias");
    eh.act = ACT_LEAKY;
    exchange(D(a_->attn, a_->attnlo), c, 1, 1);
    mark("conv.head", 18.0 * P * c * feat, 4.0 * P * (c + feat));
    conv_res("conv_before_upsample.0.weight", O(a_->attn, a_->attnlo), c, D(a_->headA, a_->headAlo), feat, 1, false,
             eh);
    float *cur = a_->headA, *curlo = a_->headAlo;
    float *nxt = a_->headB, *nxtlo = a_->headBlo;
    int hh = pl.rows, ww = pl.wp, res = 1;
    auto blocks = wt_.up_blocks();
    for (size_t i = 0; i < blocks.size(); ++i) {
        Epi eu;
        eu.bias = W("upsample." + std::to_string(2 * i) + ".bias");
        eu.shuffle = blocks[i].first;
        exchange(D(cur, curlo), feat, res, 1);
        mark("conv.up", 18.0 * hh * ww * feat * blocks[i].second, 4.0 * hh * ww * (feat + blocks[i].second));
        conv_res("upsample." + std::to_string(2 * i) + ".weight", O(cur, curlo), feat, D(nxt, nxtlo), feat, res,
                 false, eu);
        hh *= blocks[i].first;
        ww *= blocks[i].first;
        res *= blocks[i].first;
        std::swap(cur, nxt);
        std::swap(curlo, nxtlo);
    }
    // conv_last with the crop and `x / img_range + mean` in its store (src/backend.rs:94-109).
    Epi el;
    el.bias = W("conv_last.bias");
    el.planar_out = 1;
    el.oh = pl.h * wt_.scale;
    el.ow = pl.w * wt_.scale;
    el.img_range = wt_.img_range;
    for (int i = 0; i < 3; ++i) el.mean[i] = wt_.mean[i];
    exchange(D(cur, curlo), feat, res, 1);
    mark("conv.last", 18.0 * hh * ww * feat * 3, 4.0 * hh * ww * (feat + 3));
    conv_res("conv_last.weight", O(cur, curlo), feat, Dst{a_->dout, nullptr}, 3, res, false, el);
    mark(nullptr, 0, 0);
}

void Engine::mark(const char* kind, double flops, double bytes) {
    if (!profiling_) return;
    cudaEvent_t ev;
    HAT_CUDA(cudaEventCreate(&ev));
    HAT_CUDA(cudaEventRecord(ev, stream_));
    marks_.push_back({kind ? kind : "", flops, bytes, ev});
}

// One eager pass with an event between every launch: per kind of kernel, the number of
// launches, their summed device time and their algorithmic FLOPs and bytes.
std::string Engine::profile(int h, int w) {
    refuse_if_aborted();
    HAT_CUDA(cudaSetDevice(device_));
    ensure_plan(h, w);
    for (auto& m : marks_) cudaEventDestroy(m.ev);
    marks_.clear();
    if (comm_) comm_->begin_pass();
    profiling_ = true;
    uint64_t* prev = g_launch_counter;
    g_launch_counter = &launches_;
    try {
        enqueue_pass();
    } catch (...) {
        profiling_ = false;
        g_launch_counter = prev;
        throw;
    }
    profiling_ = false;
    g_launch_counter = prev;
    wait_stream();
    struct Agg {
        int n = 0;
        double ms = 0, flops = 0, bytes = 0;
    };
    std::map<std::string, Agg> agg;
    for (size_t i = 0; i + 1 < marks_.size(); ++i) {
        float ms = 0;
        HAT_CUDA(cudaEventElapsedTime(&ms, marks_[i].ev, marks_[i + 1].ev));
        Agg& a = agg[marks_[i].kind];
        a.n += 1;
        a.ms += ms;
        a.flops += marks_[i].flops;
        a.bytes += marks_[i].bytes;
    }
    for (auto& m : marks_) cudaEventDestroy(m.ev);
    marks_.clear();
    check_device_error();
    std::ostringstream o;
    o << "{";
    bool first = true;
    for (auto& kv : agg) {
        char buf[256];
        snprintf(buf, sizeof buf, "%s\"%s\": {\"launches\": %d, \"ms\": %.6f, \"flops\": %.6e, \"bytes\": %.6e}",
                 first ? "" : ", ", kv.first.c_str(), kv.second.n, kv.second.ms, kv.second.flops, kv.second.bytes);
        o << buf;
        first = false;
    }
    o << "}";
    return o.str();
}

void Engine::run_graph(cudaStream_t run) {
    // Sharded: the ranks meet on the host before any of them enqueues the pass's exchanges.
    if (comm_) comm_->begin_pass();
    uint64_t* prev = g_launch_counter;
    g_launch_counter = &launches_;
    try {
        if (!use_graph_ || eager_runs_ < 1) {
            // Eager: the launches go to the engine's stream, joined to `run` both ways.
            if (run != stream_) {
                HAT_CUDA(cudaEventRecord(join_, run));
                HAT_CUDA(cudaStreamWaitEvent(stream_, join_, 0));
            }
            uint64_t before = launches_;
            enqueue_pass();
            per_pass_ = launches_ - before;
            ++eager_runs_;
            if (run != stream_) {
                HAT_CUDA(cudaEventRecord(join_, stream_));
                HAT_CUDA(cudaStreamWaitEvent(run, join_, 0));
            }
        } else {
            if (!graph_) {
                // Captured on the engine's own stream; replayed on whichever stream the
                // caller runs on.
                cudaGraph_t g = nullptr;
                uint64_t before = launches_;
                HAT_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
                try {
                    enqueue_pass();
                } catch (...) {
                    // A sharded pass may have left the communication stream forked into the
                    // capture: join it back so that the capture can end (errors ignored).
                    if (cstream_) {
                        cudaEventRecord(ev_fork_, cstream_);
                        cudaStreamWaitEvent(stream_, ev_fork_, 0);
                    }
                    cudaStreamEndCapture(stream_, &g);
                    if (g) cudaGraphDestroy(g);
                    cudaGetLastError();
                    throw;
                }
                HAT_CUDA(cudaStreamEndCapture(stream_, &g));
                launches_ = before;  // capture does not launch; replays are counted below
                HAT_CUDA(cudaGraphInstantiate(&graph_, g, 0));
                cudaGraphDestroy(g);
            }
            HAT_CUDA(cudaGraphLaunch(graph_, run));
            launches_ += per_pass_;
        }
    } catch (...) {
        g_launch_counter = prev;
        throw;
    }
    g_launch_counter = prev;
}

void Engine::forward_device(int n, int h, int w, const float* din, float* dout, cudaStream_t st) {
    if (n <= 0 || h <= 0 || w <= 0) throw Error(1, std::to_string(h) + "x" + std::to_string(w) + " is empty");
    refuse_if_aborted();
    HAT_CUDA(cudaSetDevice(device_));
    ensure_plan(h, w);
    cudaStream_t run = st ? st : stream_;
    const long inN = 3L * h * w, outN = 3L * h * wt_.scale * w * wt_.scale;
    for (int i = 0; i < n; ++i) {
        HAT_CUDA(cudaMemcpyAsync(a_->din, din + i * inN, inN * sizeof(float), cudaMemcpyDeviceToDevice, run));
        run_graph(run);
        copy_out(dout + i * outN, cudaMemcpyDeviceToDevice, run);
    }
}

void Engine::forward_host(int n, int h, int w, const float* in, float* out) {
    if (n <= 0 || h <= 0 || w <= 0) throw Error(1, std::to_string(h) + "x" + std::to_string(w) + " is empty");
    refuse_if_aborted();
    HAT_CUDA(cudaSetDevice(device_));
    const long inN = 3L * h * w, outN = 3L * h * wt_.scale * w * wt_.scale;
    for (int attempt = 0;; ++attempt) {
        ensure_plan(h, w);
        for (int i = 0; i < n; ++i) {
            HAT_CUDA(cudaMemcpyAsync(a_->din, in + i * inN, inN * sizeof(float), cudaMemcpyHostToDevice, stream_));
            run_graph(stream_);
            // A copy into pageable host memory blocks until the pass is done; sharded, the
            // pass waits on the other ranks, so it is awaited under the deadline first.
            if (comm_) wait_stream();
            copy_out(out + i * outN, cudaMemcpyDeviceToHost, stream_);
        }
        wait_stream();
        const int v = take_device_error();
        // An operand beyond fp16's range: the whole call again on tf32 pairs, then with the
        // attention on the CUDA cores if q, k or v is the one (not on a strip-sharded handle,
        // whose ranks must keep one operand layout in step).
        const bool can = (v == ERR_RANGE_GEMM && h16_) || (v == ERR_RANGE_ATTN && !attn_simt_);
        if (can && !simt_only_ && !comm_ && attempt < 2) {
            fall_back(v);
            continue;
        }
        raise_device_error(v);
        return;
    }
}

}  // namespace hat
