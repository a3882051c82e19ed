// The layer scheduler. Activations are token-major planes [hp][wp][c] (channels
// innermost), so a token linear is a plain row-major GEMM over the whole plane, a 3x3
// conv is an implicit GEMM over K = 9*cin, and the windowed attentions read their
// windows out of the qkv plane by address arithmetic. Every layer is one launch.
#include "engine.h"

#include <cstring>
#include <sstream>

namespace hat {

// ------------------------------------------------------------------ sizes
Sizes Sizes::of(const Weights& wt, const Plan& p) {
    Sizes s;
    const long P = p.tokens(), c = wt.embed;
    s.x0 = P * 3;
    s.body = P * c;
    s.xa = P * c;
    s.xb = P * c;
    s.n1 = P * c;
    s.cmid = P * wt.compressed;
    s.convx = P * c;
    s.qkv = P * 3 * c;
    s.attn = P * c;
    s.hid = P * wt.mlp_ratio * c;
    s.chsum = c;
    s.gate = c;
    // The head's planes ping-pong between two buffers: plane 0 (conv_before_upsample's
    // output, at P) and every other shuffled plane go to A, the rest to B.
    long res = P, a = P * wt.head_feat, b = 0;
    int i = 1;
    for (auto& blk : wt.up_blocks()) {
        res *= (long)blk.first * blk.first;
        long need = res * wt.head_feat;
        if (i % 2) b = std::max(b, need); else a = std::max(a, need);
        ++i;
    }
    s.headA = a;
    s.headB = b;
    s.din = 3L * p.h * p.w;
    s.dout = 3L * p.h * wt.scale * p.w * wt.scale;
    return s;
}

struct Engine::Acts {
    float *x0, *body, *xa, *xb, *n1, *cmid, *convx, *qkv, *attn, *hid, *chsum, *gate, *headA, *headB,
        *din, *dout;
};

// ------------------------------------------------------------------ dispatch
void launch_linear_simt(const float* x, const float* w, float* y, long m, int n, int k, const Epi& e,
                        cudaStream_t st);
void launch_conv3x3_simt(const float* x, const float* wr, float* y, int hgt, int wid, int cin, int cout,
                         const Epi& e, cudaStream_t st);
void launch_window_attention_simt(const float* qkv, const float* table, float* out, const Plan& p, int c,
                                  int heads, int shift, cudaStream_t st);
void launch_overlap_attention_simt(const float* qkv, const float* table, float* out, const Plan& p, int c,
                                   int heads, cudaStream_t st);

void launch_linear(int mode, const float* x, const float* w, float* y, long m, int n, int k, const Epi& e,
                   cudaStream_t st) {
    (void)mode;
    launch_linear_simt(x, w, y, m, n, k, e, st);
}

void launch_conv3x3(int mode, const float* x, const float* wr, float* y, int hgt, int wid, int cin, int cout,
                    const Epi& e, cudaStream_t st) {
    (void)mode;
    launch_conv3x3_simt(x, wr, y, hgt, wid, cin, cout, e, st);
}

void launch_window_attention(int mode, const float* qkv, const float* table, float* out, const Plan& p, int c,
                             int heads, int shift, cudaStream_t st) {
    (void)mode;
    launch_window_attention_simt(qkv, table, out, p, c, heads, shift, st);
}

void launch_overlap_attention(int mode, const float* qkv, const float* table, float* out, const Plan& p,
                              int c, int heads, cudaStream_t st) {
    (void)mode;
    launch_overlap_attention_simt(qkv, table, out, p, c, heads, st);
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

static const double SLACK = 1.05;           // src/memguard.rs:42
static const double BASE = 128.0 * 1048576;  // src/memguard.rs:49

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

    // Upload every f32 tensor once, plus a tap-major copy of every 3x3 conv weight.
    size_t total = 0;
    std::vector<std::string> names;
    for (auto& kv : wt_.st.tensors) {
        if (kv.second.dtype != "F32") continue;
        names.push_back(kv.first);
        size_t n = (size_t)kv.second.numel();
        total += (n + 63) / 64 * 64;
        if (kv.second.shape.size() == 4 && kv.second.shape[2] == 3) total += (n + 63) / 64 * 64;
    }
    HAT_CUDA(cudaMalloc(&dweights_, total * sizeof(float)));
    size_t off = 0;
    uint64_t* prev = g_launch_counter;
    g_launch_counter = &launches_;
    for (auto& name : names) {
        const TensorInfo& ti = wt_.st.tensors[name];
        size_t n = (size_t)ti.numel();
        float* d = dweights_ + off;
        HAT_CUDA(cudaMemcpyAsync(d, wt_.st.f32(name), n * sizeof(float), cudaMemcpyHostToDevice, stream_));
        w_[name] = d;
        off += (n + 63) / 64 * 64;
        if (ti.shape.size() == 4 && ti.shape[2] == 3) {
            float* r = dweights_ + off;
            launch_reorder_conv(d, r, (int)ti.shape[0], (int)ti.shape[1], stream_);
            wconv_[name] = r;
            off += (n + 63) / 64 * 64;
        }
    }
    g_launch_counter = prev;
    HAT_CUDA(cudaStreamSynchronize(stream_));
}

Engine::~Engine() {
    cudaSetDevice(device_);
    if (graph_) cudaGraphExecDestroy(graph_);
    if (arena_) cudaFree(arena_);
    if (dweights_) cudaFree(dweights_);
    if (join_) cudaEventDestroy(join_);
    if (stream_) cudaStreamDestroy(stream_);
}

const float* Engine::W(const std::string& name) const {
    auto it = w_.find(name);
    if (it == w_.end()) throw Error(2, "gpu: no weight `" + name + "`");
    return it->second;
}

const float* Engine::Wconv(const std::string& name) const {
    auto it = wconv_.find(name);
    if (it == wconv_.end()) throw Error(2, "gpu: no conv weight `" + name + "`");
    return it->second;
}

size_t Engine::footprint_bytes(int h, int w) const {
    return (size_t)Sizes::of(wt_, Plan::make(h, w, wt_.window)).total() * sizeof(float);
}

void Engine::check_memory(int h, int w) const {
    // check_gpu (src/memguard.rs:183-201)
    double acts = (double)footprint_bytes(h, w);
    double need = acts * SLACK + (double)wt_.f32_bytes + BASE;
    size_t fr = 0, tot = 0;
    HAT_CUDA(cudaSetDevice(device_));
    HAT_CUDA(cudaMemGetInfo(&fr, &tot));
    // The engine's own current arena is reusable, so it counts as available.
    double avail = (double)fr + (have_plan_ ? (double)Sizes::of(wt_, plan_).total() * sizeof(float) : 0.0);
    if (need > avail) {
        std::ostringstream o;
        o << "not enough video memory for a " << w << "x" << h << " pass on the GPU\n"
          << "hat: it needs about " << fmt_bytes(need) << " (" << fmt_bytes(acts) << " of device buffers + "
          << fmt_bytes((double)wt_.f32_bytes) << " of weights + " << fmt_bytes(BASE) << " of runtime, plus "
          << 5 << "% of slack); " << fmt_bytes(avail) << " is free on the device\n"
          << "hat: `--mem` runs it in tiles on the device (each tile allocates its own buffers, so the "
             "tile's size is the number that must fit); a smaller image does too";
        throw Error(4, o.str());
    }
}

void Engine::ensure_plan(int h, int w) {
    Plan p = Plan::make(h, w, wt_.window);
    if (have_plan_ && p == plan_) return;
    check_memory(h, w);
    if (graph_) {
        cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
    }
    if (arena_) {
        HAT_CUDA(cudaStreamSynchronize(stream_));
        cudaFree(arena_);
        arena_ = nullptr;
        have_plan_ = false;
    }
    Sizes s = Sizes::of(wt_, p);
    HAT_CUDA(cudaMalloc(&arena_, (size_t)s.total() * sizeof(float)));
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
    a_->cmid = take(s.cmid);
    a_->convx = take(s.convx);
    a_->qkv = take(s.qkv);
    a_->attn = take(s.attn);
    a_->hid = take(s.hid);
    a_->chsum = take(s.chsum);
    a_->gate = take(s.gate);
    a_->headA = take(s.headA);
    a_->headB = take(s.headB);
    a_->din = take(s.din);
    a_->dout = take(s.dout);
    // THE PREDICTION IS HELD TO THE ALLOCATION (src/gpu.rs:779-786).
    if (q - arena_ != s.total())
        throw Error(3, "gpu: the buffer set does not match the guard's prediction");
    plan_ = p;
    have_plan_ = true;
    eager_runs_ = 0;
}

// `x + fc2(gelu(fc1(norm2(x))))`, in place on x (src/gpu.rs:449-466).
void Engine::mlp(const std::string& p, float* x) {
    const long P = plan_.tokens();
    const int c = wt_.embed, hid = wt_.mlp_ratio * c;
    mark("layernorm", 0, 8.0 * P * c);
    launch_layernorm(x, W(p + ".norm2.weight"), W(p + ".norm2.bias"), a_->n1, P, c, stream_);
    Epi e1;
    e1.bias = W(p + ".mlp.fc1.bias");
    e1.act = ACT_GELU;
    mark("linear.fc1", 2.0 * P * hid * c, 4.0 * P * (c + hid));
    launch_linear(mode_, a_->n1, W(p + ".mlp.fc1.weight"), a_->hid, P, hid, c, e1, stream_);
    Epi e2;
    e2.bias = W(p + ".mlp.fc2.bias");
    e2.res = x;
    mark("linear.fc2", 2.0 * P * hid * c, 4.0 * P * (hid + 2 * c));
    launch_linear(mode_, a_->hid, W(p + ".mlp.fc2.weight"), x, P, c, hid, e2, stream_);
}

// One HAB (hat_arch.py:266-309; src/gpu.rs:469-520): `in` is the block input, `out`
// its output (may be the same buffer).
void Engine::hab(int stage, int blk, const float* in, float* out) {
    const long P = plan_.tokens();
    const int c = wt_.embed, cc = wt_.compressed;
    const std::string p = "layers." + std::to_string(stage) + ".residual_group.blocks." + std::to_string(blk);
    const std::string cb = p + ".conv_block.cab";
    mark("layernorm", 0, 8.0 * P * c);
    launch_layernorm(in, W(p + ".norm1.weight"), W(p + ".norm1.bias"), a_->n1, P, c, stream_);
    // CAB: conv c→cc + GELU, conv cc→c with the channel sums of its output, the gate.
    Epi ec1;
    ec1.bias = W(cb + ".0.bias");
    ec1.act = ACT_GELU;
    mark("conv.cab1", 18.0 * P * c * cc, 4.0 * P * (c + cc));
    launch_conv3x3(mode_, a_->n1, Wconv(cb + ".0.weight"), a_->cmid, plan_.hp, plan_.wp, c, cc, ec1, stream_);
    mark("conv.cab2", 18.0 * P * c * cc, 4.0 * P * (c + cc));
    HAT_CUDA(cudaMemsetAsync(a_->chsum, 0, c * sizeof(float), stream_));
    Epi ec2;
    ec2.bias = W(cb + ".2.bias");
    ec2.colsum = a_->chsum;
    launch_conv3x3(mode_, a_->cmid, Wconv(cb + ".2.weight"), a_->convx, plan_.hp, plan_.wp, cc, c, ec2, stream_);
    mark("ca_gate", 0, 0);
    launch_ca_gate(a_->chsum, 1.f / (float)P, W(cb + ".3.attention.1.weight"), W(cb + ".3.attention.1.bias"),
                   W(cb + ".3.attention.3.weight"), W(cb + ".3.attention.3.bias"), a_->gate, c, wt_.squeezed,
                   stream_);
    // Attention on the normed plane; odd blocks are shifted by win/2 with the mask.
    Epi eq;
    eq.bias = W(p + ".attn.qkv.bias");
    mark("linear.qkv", 6.0 * P * c * c, 16.0 * P * c);
    launch_linear(mode_, a_->n1, W(p + ".attn.qkv.weight"), a_->qkv, P, 3 * c, c, eq, stream_);
    const int shift = blk % 2 ? plan_.shift : 0;
    mark("attn.window", 4.0 * P * 256 * c, 16.0 * P * c);
    launch_window_attention(mode_, a_->qkv, W(p + ".attn.relative_position_bias_table"), a_->attn, plan_, c,
                            wt_.heads, shift, stream_);
    // proj, then `(shortcut + attn) + conv_x * conv_scale` in the epilogue.
    Epi ep;
    ep.bias = W(p + ".attn.proj.bias");
    ep.res = in;
    ep.cx = a_->convx;
    ep.gate = a_->gate;
    ep.cscale = wt_.conv_scale;
    mark("linear.proj", 2.0 * P * c * c, 16.0 * P * c);
    launch_linear(mode_, a_->attn, W(p + ".attn.proj.weight"), out, P, c, c, ep, stream_);
    mlp(p, out);
}

// The OCAB (hat_arch.py:392-438; src/gpu.rs:533-588).
void Engine::ocab(int stage, const float* in, float* out) {
    const long P = plan_.tokens();
    const int c = wt_.embed;
    const std::string p = "layers." + std::to_string(stage) + ".residual_group.overlap_attn";
    mark("layernorm", 0, 8.0 * P * c);
    launch_layernorm(in, W(p + ".norm1.weight"), W(p + ".norm1.bias"), a_->n1, P, c, stream_);
    Epi eq;
    eq.bias = W(p + ".qkv.bias");
    mark("linear.qkv", 6.0 * P * c * c, 16.0 * P * c);
    launch_linear(mode_, a_->n1, W(p + ".qkv.weight"), a_->qkv, P, 3 * c, c, eq, stream_);
    mark("attn.overlap", 4.0 * P * 576 * c, 16.0 * P * c);
    launch_overlap_attention(mode_, a_->qkv, W(p + ".relative_position_bias_table"), a_->attn, plan_, c, wt_.heads,
                             stream_);
    Epi ep;
    ep.bias = W(p + ".proj.bias");
    ep.res = in;
    mark("linear.proj", 2.0 * P * c * c, 12.0 * P * c);
    launch_linear(mode_, a_->attn, W(p + ".proj.weight"), out, P, c, c, ep, stream_);
    mlp(p, out);
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
    launch_conv3x3(mode_, a_->x0, Wconv("conv_first.weight"), a_->body, pl.hp, pl.wp, 3, c, ef, stream_);
    mark("layernorm", 0, 8.0 * P * c);
    launch_layernorm(a_->body, W("patch_embed.norm.weight"), W("patch_embed.norm.bias"), a_->xa, P, c, stream_);
    // The stage input stays in `xa` (the RHAG residual); the blocks run in `xb`, and the
    // stage conv adds the two back into `xa`.
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
        mark("conv.rhag", 18.0 * P * c * c, 12.0 * P * c);
        launch_conv3x3(mode_, a_->xb, Wconv("layers." + std::to_string(s) + ".conv.weight"), a_->xa, pl.hp, pl.wp,
                       c, c, er, stream_);
    }
    mark("layernorm", 0, 8.0 * P * c);
    launch_layernorm(a_->xa, W("norm.weight"), W("norm.bias"), a_->n1, P, c, stream_);
    Epi eb;
    eb.bias = W("conv_after_body.bias");
    eb.res = a_->body;
    mark("conv.body", 18.0 * P * c * c, 12.0 * P * c);
    launch_conv3x3(mode_, a_->n1, Wconv("conv_after_body.weight"), a_->xb, pl.hp, pl.wp, c, c, eb, stream_);
    // Head: conv + LeakyReLU, then per block a conv whose store does the PixelShuffle.
    Epi eh;
    eh.bias = W("conv_before_upsample.0.bias");
    eh.act = ACT_LEAKY;
    mark("conv.head", 18.0 * P * c * feat, 4.0 * P * (c + feat));
    launch_conv3x3(mode_, a_->xb, Wconv("conv_before_upsample.0.weight"), a_->headA, pl.hp, pl.wp, c, feat, eh,
                   stream_);
    float* cur = a_->headA;
    float* nxt = a_->headB;
    int hh = pl.hp, ww = pl.wp;
    auto blocks = wt_.up_blocks();
    for (size_t i = 0; i < blocks.size(); ++i) {
        Epi eu;
        eu.bias = W("upsample." + std::to_string(2 * i) + ".bias");
        eu.shuffle = blocks[i].first;
        mark("conv.up", 18.0 * hh * ww * feat * blocks[i].second, 4.0 * hh * ww * (feat + blocks[i].second));
        launch_conv3x3(mode_, cur, Wconv("upsample." + std::to_string(2 * i) + ".weight"), nxt, hh, ww, feat,
                       blocks[i].second, eu, stream_);
        hh *= blocks[i].first;
        ww *= blocks[i].first;
        std::swap(cur, nxt);
    }
    // conv_last with the crop and `x / img_range + mean` in its store (src/backend.rs:94-109).
    Epi el;
    el.bias = W("conv_last.bias");
    el.planar_out = 1;
    el.oh = pl.h * wt_.scale;
    el.ow = pl.w * wt_.scale;
    el.img_range = wt_.img_range;
    for (int i = 0; i < 3; ++i) el.mean[i] = wt_.mean[i];
    mark("conv.last", 18.0 * hh * ww * feat * 3, 4.0 * hh * ww * (feat + 3));
    launch_conv3x3(mode_, cur, Wconv("conv_last.weight"), a_->dout, hh, ww, feat, 3, el, stream_);
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
    HAT_CUDA(cudaSetDevice(device_));
    ensure_plan(h, w);
    for (auto& m : marks_) cudaEventDestroy(m.ev);
    marks_.clear();
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
    HAT_CUDA(cudaStreamSynchronize(stream_));
    struct Agg { int n = 0; double ms = 0, flops = 0, bytes = 0; };
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
                    cudaStreamEndCapture(stream_, &g);
                    if (g) cudaGraphDestroy(g);
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
    HAT_CUDA(cudaSetDevice(device_));
    ensure_plan(h, w);
    cudaStream_t run = st ? st : stream_;
    const long inN = 3L * h * w, outN = 3L * h * wt_.scale * w * wt_.scale;
    for (int i = 0; i < n; ++i) {
        HAT_CUDA(cudaMemcpyAsync(a_->din, din + i * inN, inN * sizeof(float), cudaMemcpyDeviceToDevice, run));
        run_graph(run);
        HAT_CUDA(cudaMemcpyAsync(dout + i * outN, a_->dout, outN * sizeof(float), cudaMemcpyDeviceToDevice, run));
    }
}

void Engine::forward_host(int n, int h, int w, const float* in, float* out) {
    if (n <= 0 || h <= 0 || w <= 0) throw Error(1, std::to_string(h) + "x" + std::to_string(w) + " is empty");
    HAT_CUDA(cudaSetDevice(device_));
    ensure_plan(h, w);
    const long inN = 3L * h * w, outN = 3L * h * wt_.scale * w * wt_.scale;
    for (int i = 0; i < n; ++i) {
        HAT_CUDA(cudaMemcpyAsync(a_->din, in + i * inN, inN * sizeof(float), cudaMemcpyHostToDevice, stream_));
        run_graph(stream_);
        HAT_CUDA(cudaMemcpyAsync(out + i * outN, a_->dout, outN * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    }
    HAT_CUDA(cudaStreamSynchronize(stream_));
}

}  // namespace hat
