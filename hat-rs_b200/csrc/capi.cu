// The C ABI (include/hat_b200.h): exception-to-error-code translation around the
// engine and the kernel launchers.
#include <cstdarg>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/hat_b200.h"
#include "engine.h"
#include "nccl_rt.h"
#include "png.h"
#include "tile.h"

using namespace hat;

// One engine per GPU. A one-GPU handle is engs[0] alone; a handle over several GPUs runs
// each call's share on every engine from a host thread of its own.
struct hat_b200 {
    std::vector<std::unique_ptr<Engine>> engs;
    int shard = HAT_B200_SHARD_BATCH;
    Engine& e0() const { return *engs[0]; }
    bool multi() const { return engs.size() > 1; }
};

// Runs f(g) for every GPU g on its own thread and rethrows the first failure, naming the GPU.
template <class F>
static void on_every_gpu(const hat_b200* h, F&& f) {
    const size_t G = h->engs.size();
    if (G == 1) {
        f(0);
        return;
    }
    std::vector<std::exception_ptr> errs(G);
    std::vector<std::thread> ts;
    ts.reserve(G);
    for (size_t g = 0; g < G; ++g)
        ts.emplace_back([&, g] {
            try {
                f((int)g);
            } catch (...) {
                errs[g] = std::current_exception();
            }
        });
    for (auto& t : ts) t.join();
    for (size_t g = 0; g < G; ++g) {
        if (!errs[g]) continue;
        try {
            std::rethrow_exception(errs[g]);
        } catch (const Error& e) {
            throw Error(e.code, "gpu " + std::to_string(h->engs[g]->device()) + ": " + e.what());
        } catch (const std::exception& e) {
            throw Error(HAT_B200_EINVAL, "gpu " + std::to_string(h->engs[g]->device()) + ": " + e.what());
        }
    }
}

static void set_err(char* err, size_t errlen, const std::string& msg) {
    if (!err || errlen == 0) return;
    size_t n = msg.size() < errlen - 1 ? msg.size() : errlen - 1;
    memcpy(err, msg.data(), n);
    err[n] = 0;
}

template <class F>
static int guarded(char* err, size_t errlen, F&& f) {
    try {
        f();
        set_err(err, errlen, "");
        return HAT_B200_OK;
    } catch (const Error& e) {
        set_err(err, errlen, e.what());
        return e.code ? e.code : HAT_B200_EINVAL;
    } catch (const std::exception& e) {
        set_err(err, errlen, e.what());
        return HAT_B200_EINVAL;
    }
}

static void fill_info(const Weights& wt, hat_b200_info* o) {
    memset(o, 0, sizeof *o);
    o->scale = wt.scale;
    o->window = wt.window;
    o->owin = wt.owin;
    o->embed = wt.embed;
    o->heads = wt.heads;
    o->head_dim = wt.head_dim;
    o->mlp_ratio = wt.mlp_ratio;
    o->compressed = wt.compressed;
    o->squeezed = wt.squeezed;
    o->head_feat = wt.head_feat;
    o->n_stages = (int)wt.depths.size();
    for (int d : wt.depths) o->n_blocks += d;
    o->conv_scale = wt.conv_scale;
    o->img_range = wt.img_range;
    for (int i = 0; i < 3; ++i) o->mean[i] = wt.mean[i];
    snprintf(o->variant, sizeof o->variant, "%s", wt.variant.c_str());
}

extern "C" {

int hat_b200_create(const char* path, const hat_b200_opts* opts, hat_b200** out, char* err, size_t errlen) {
    if (!path || !out) {
        set_err(err, errlen, "hat_b200_create: null path or out");
        return HAT_B200_EINVAL;
    }
    *out = nullptr;
    hat_b200_opts o;
    memset(&o, 0, sizeof o);
    o.mode = HAT_B200_MODE_PARITY;
    o.use_graph = 1;
    if (opts) o = *opts;
    return guarded(err, errlen, [&] {
        const int G = o.ngpus > 1 ? o.ngpus : 1;
        if (G > 1 && o.shard != HAT_B200_SHARD_BATCH && o.shard != HAT_B200_SHARD_STRIP)
            throw Error(1, "hat_b200_create: unknown shard mode " + std::to_string(o.shard));
        std::vector<int> devs(G);
        for (int g = 0; g < G; ++g) devs[g] = o.devices ? o.devices[g] : o.device + g;
        for (int g = 0; g < G; ++g)
            for (int k = 0; k < g; ++k)
                if (devs[g] == devs[k])
                    throw Error(1, "hat_b200_create: device " + std::to_string(devs[g]) + " is listed twice");
        std::unique_ptr<hat_b200> h(new hat_b200);
        h->shard = G > 1 ? o.shard : HAT_B200_SHARD_BATCH;
        h->engs.resize(G);
        // Weights are read and uploaded on every GPU at once.
        on_every_gpu(h.get(), [&](int g) {
            h->engs[g].reset(new Engine(path, devs[g], o.mode, o.use_graph != 0, o.simt_only != 0));
            h->engs[g]->set_timeout(o.timeout_ms > 0 ? o.timeout_ms / 1000.0 : 120.0);
        });
        if (G > 1 && h->shard == HAT_B200_SHARD_STRIP) {
            // One communicator over the handle's GPUs; each rank joins from its own thread.
            unsigned char id[128];
            nccl_unique_id(id, sizeof id);
            on_every_gpu(h.get(), [&](int g) { h->engs[g]->attach_strip(g, G, id, sizeof id); });
        }
        *out = h.release();
    });
}

void hat_b200_destroy(hat_b200* h) { delete h; }

int hat_b200_get_info(const hat_b200* h, hat_b200_info* out) {
    if (!h || !out) return HAT_B200_EINVAL;
    fill_info(h->e0().weights(), out);
    return HAT_B200_OK;
}

static void png_out(const PngImage& img, float* out, size_t out_floats, int* width, int* height) {
    if (width) *width = img.w;
    if (height) *height = img.h;
    if (!out) return;
    if (out_floats < img.data.size())
        throw Error(1, "png: the output buffer holds " + std::to_string(out_floats) + " floats; the image needs " +
                           std::to_string(img.data.size()));
    memcpy(out, img.data.data(), img.data.size() * sizeof(float));
}

int hat_b200_png_load(const char* path, float* out, size_t out_floats, int* width, int* height, char* err,
                      size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!path) throw Error(1, "png: null path");
        png_out(png_load(path), out, out_floats, width, height);
    });
}

int hat_b200_png_decode(const uint8_t* bytes, size_t len, float* out, size_t out_floats, int* width, int* height,
                        char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!bytes) throw Error(1, "png: null buffer");
        png_out(png_decode(bytes, len), out, out_floats, width, height);
    });
}

int hat_b200_to_rgb8(const float* planar, int width, int height, uint8_t* rgb) {
    if (!planar || !rgb || width <= 0 || height <= 0) return HAT_B200_EINVAL;
    to_rgb8(planar, width, height, rgb);
    return HAT_B200_OK;
}

int hat_b200_png_save(const char* path, int width, int height, const uint8_t* rgb, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!path || !rgb) throw Error(1, "png: null path or pixels");
        png_save_rgb8(path, width, height, rgb);
    });
}

int hat_b200_png_encode(int width, int height, const uint8_t* rgb, uint8_t* out, size_t cap, size_t* len, char* err,
                        size_t errlen) {
    return guarded(err, errlen, [&] {
        if (!rgb) throw Error(1, "png: null pixels");
        const std::vector<uint8_t> b = png_encode_rgb8(width, height, rgb);
        if (len) *len = b.size();
        if (!out || cap < b.size())
            throw Error(1, "png: the output buffer holds " + std::to_string(cap) + " bytes; the file needs " +
                               std::to_string(b.size()));
        memcpy(out, b.data(), b.size());
    });
}

int hat_b200_set_timeout(hat_b200* h, int ms) {
    if (!h) return HAT_B200_EINVAL;
    for (auto& e : h->engs) e->set_timeout(ms > 0 ? ms / 1000.0 : 120.0);
    return HAT_B200_OK;
}

int hat_b200_gpu_count(const hat_b200* h) { return h ? (int)h->engs.size() : 0; }

// Checkpoint inspection without a device: what --list-weights and the loader tests use.
int hat_b200_inspect(const char* path, hat_b200_info* out, char* err, size_t errlen) {
    return guarded(err, errlen, [&] {
        Weights wt;
        wt.load(path ? path : "");
        if (out) fill_info(wt, out);
    });
}

int hat_b200_forward(hat_b200* h, int n, int height, int width, const float* in, float* out, char* err,
                     size_t errlen) {
    if (!h || !in || !out) {
        set_err(err, errlen, "hat_b200_forward: null handle or buffer");
        return HAT_B200_EINVAL;
    }
    return guarded(err, errlen, [&] {
        if (!h->multi()) {
            h->e0().forward_host(n, height, width, in, out);
            return;
        }
        if (n <= 0 || height <= 0 || width <= 0) throw Error(1, "hat_b200_forward: empty batch or image");
        if (h->shard == HAT_B200_SHARD_STRIP) {
            // Every GPU reads the whole images and writes its own rows of every output.
            on_every_gpu(h, [&](int g) { h->engs[g]->forward_host(n, height, width, in, out); });
            return;
        }
        // Batch: GPU g takes images [n*g/G, n*(g+1)/G).
        const int G = (int)h->engs.size();
        const int s = h->e0().weights().scale;
        const long inN = 3L * height * width, outN = 3L * height * s * width * s;
        on_every_gpu(h, [&](int g) {
            const int a = (int)((long)n * g / G), b = (int)((long)n * (g + 1) / G);
            if (b > a) h->engs[g]->forward_host(b - a, height, width, in + a * inN, out + a * outN);
        });
    });
}

int hat_b200_forward_device(hat_b200* h, int n, int height, int width, const float* d_in, float* d_out,
                            void* stream, char* err, size_t errlen) {
    if (!h || !d_in || !d_out) {
        set_err(err, errlen, "hat_b200_forward_device: null handle or buffer");
        return HAT_B200_EINVAL;
    }
    return guarded(err, errlen, [&] {
        if (h->multi()) throw Error(1, "hat_b200_forward_device: the handle drives several GPUs; use hat_b200_forward");
        h->e0().forward_device(n, height, width, d_in, d_out, (cudaStream_t)stream);
    });
}

int hat_b200_sync(hat_b200* h, char* err, size_t errlen) {
    if (!h) {
        set_err(err, errlen, "hat_b200_sync: null handle");
        return HAT_B200_EINVAL;
    }
    return guarded(err, errlen, [&] { on_every_gpu(h, [&](int g) { h->engs[g]->sync(); }); });
}

int hat_b200_fp16_pairs(const hat_b200* h) { return h && h->e0().fp16_pairs() ? 1 : 0; }

size_t hat_b200_footprint_bytes(const hat_b200* h, int height, int width) {
    if (!h || height <= 0 || width <= 0) return 0;
    return h->e0().footprint_bytes(height, width);
}

int hat_b200_check_memory(const hat_b200* h, int height, int width, char* err, size_t errlen) {
    if (!h) return HAT_B200_EINVAL;
    return guarded(err, errlen, [&] {
        for (auto& e : h->engs) e->check_memory(height, width);
    });
}

int hat_b200_free_vram(int device, size_t* free_bytes, size_t* total_bytes) {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return HAT_B200_ECUDA;
    if (cudaSetDevice(device) != cudaSuccess) return HAT_B200_ECUDA;
    size_t f = 0, t = 0;
    cudaError_t e = cudaMemGetInfo(&f, &t);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return HAT_B200_ECUDA;
    if (free_bytes) *free_bytes = f;
    if (total_bytes) *total_bytes = t;
    return HAT_B200_OK;
}

int hat_b200_probe(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return 0;
    }
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, 0) != cudaSuccess) return 0;
    return p.major == 10 ? 1 : 0;
}

uint64_t hat_b200_launch_count(const hat_b200* h) {
    uint64_t n = 0;
    if (h)
        for (auto& e : h->engs) n += e->launches();
    return n;
}

int hat_b200_profile(hat_b200* h, int height, int width, char* json, size_t jsonlen, char* err, size_t errlen) {
    if (!h) return HAT_B200_EINVAL;
    return guarded(err, errlen, [&] {
        // Every GPU runs the profiled pass (a strip-sharded pass has collectives); the
        // first GPU's timings are reported.
        std::vector<std::string> js(h->engs.size());
        on_every_gpu(h, [&](int g) { js[g] = h->engs[g]->profile(height, width); });
        set_err(json, jsonlen, js[0]);
    });
}

int hat_b200_forward_tiled(hat_b200* h, int height, int width, const float* in, float* out, int tile, int margin,
                           hat_b200_tiling* info, char* err, size_t errlen) {
    if (!h || !in || !out) {
        set_err(err, errlen, "hat_b200_forward_tiled: null handle or buffer");
        return HAT_B200_EINVAL;
    }
    return guarded(err, errlen, [&] {
        if (h->multi() || h->e0().sharded()) throw Error(1, "tiling: the handle is strip-sharded or drives several GPUs");
        Tiling t = tile_forward(h->e0(), height, width, in, out, tile, margin);
        if (info) {
            info->tile = t.tile;
            info->margin = t.margin;
            info->scale = t.scale;
            info->tiles = t.tiles;
            info->largest_h = t.largest_h;
            info->largest_w = t.largest_w;
        }
    });
}

int hat_b200_auto_tile(int height, int width, int window, uint64_t budget_bytes, uint64_t per_pixel_floats,
                       uint64_t constant_floats, int margin, int* tile) {
    if (height <= 0 || width <= 0 || window <= 0 || margin < 0 || !tile) return HAT_B200_EINVAL;
    auto t = auto_tile(height, width, window, budget_bytes, per_pixel_floats, constant_floats, margin);
    if (!t) return HAT_B200_ENOMEM;
    *tile = *t;
    return HAT_B200_OK;
}

int hat_b200_gpu_auto_tile(const hat_b200* h, int height, int width, int* tile, char* err, size_t errlen) {
    if (!h || !tile) return HAT_B200_EINVAL;
    return guarded(err, errlen, [&] {
        auto t = gpu_auto_tile(h->e0(), height, width);
        if (!t) throw Error(4, "one window does not fit the device's free memory");
        *tile = *t;
    });
}

int hat_b200_strip_rows(int height, int nranks, int rank, int* r0, int* r1) {
    if (height <= 0 || nranks <= 0 || rank < 0 || rank >= nranks || !r0 || !r1) return HAT_B200_EINVAL;
    const Plan p = Plan::make_strip(height, 16, 16, rank, nranks, 0);
    if (p.hp / 16 < nranks) return HAT_B200_EINVAL;  // every rank needs a window row
    *r0 = p.r0;
    *r1 = p.r1;
    return HAT_B200_OK;
}

int hat_b200_nccl_unique_id(void* id, size_t idlen, char* err, size_t errlen) {
    return guarded(err, errlen, [&] { nccl_unique_id(id, idlen); });
}

int hat_b200_attach_strip(hat_b200* h, int rank, int nranks, const void* id, size_t idlen, char* err,
                          size_t errlen) {
    if (!h) return HAT_B200_EINVAL;
    return guarded(err, errlen, [&] {
        if (h->multi()) throw Error(1, "hat_b200_attach_strip: the handle already drives several GPUs");
        h->e0().attach_strip(rank, nranks, id, idlen);
    });
}

// The GEMM operand of one kernel-level call, prepared on the caller's stream.
struct TempW {
    float* buf = nullptr;
    float* xs = nullptr;  // the activation split into tf32 hi/lo halves (parity mode)
    int* err = nullptr;
    GemmW g;
    cudaStream_t st = nullptr;
    ~TempW() {
        if (buf) cudaFreeAsync(buf, st);
        if (xs) cudaFreeAsync(xs, st);
        if (err) cudaFreeAsync(err, st);
    }
};

// The activation as the GEMMs read it: split for the parity-mode tensor-core path.
static Opnd temp_operand(TempW& t, int mode, const float* x, long n) {
    if (mode != HAT_B200_MODE_PARITY) return Opnd{x, nullptr};
    HAT_CUDA(cudaMallocAsync(&t.xs, 2 * n * sizeof(float) + 64, t.st));
    launch_split(x, t.xs, t.xs + n, n, t.st);
    return Opnd{t.xs, t.xs + n};
}

static void temp_gemm_w(TempW& t, const float* w, int n, int k_or_cin, bool conv, int cin_plane, cudaStream_t st) {
    t.st = st;
    plan_gemm_w(t.g, n, k_or_cin, conv, cin_plane);
    HAT_CUDA(cudaMallocAsync(&t.buf, (gemm_w_floats(t.g) + 64) * sizeof(float), st));
    HAT_CUDA(cudaMallocAsync(&t.err, sizeof(int), st));
    HAT_CUDA(cudaMemsetAsync(t.err, 0, sizeof(int), st));
    float* simt = t.buf;
    float* hi = simt + (size_t)t.g.n * t.g.k;
    float* lo = hi + (size_t)t.g.n_pad * t.g.k_pad;
    launch_prep_gemm_w(w, simt, t.g.umma ? hi : nullptr, t.g.umma ? lo : nullptr, t.g, st);
    t.g.simt = simt;
    t.g.hi = hi;
    t.g.lo = lo;
}

static void finish_kernel_call(TempW& t) {
    int v = 0;
    HAT_CUDA(cudaMemcpyAsync(&v, t.err, sizeof(int), cudaMemcpyDeviceToHost, t.st));
    HAT_CUDA(cudaStreamSynchronize(t.st));
    if (v) throw Error(3, "tensor-core kernel gave up waiting on its pipeline (code " + std::to_string(v) + ")");
}

int hat_b200_linear(int mode, const float* x, const float* w, const float* b, float* y, int m, int n, int k,
                    void* stream) {
    return guarded(nullptr, 0, [&] {
        cudaStream_t st = (cudaStream_t)stream;
        TempW t;
        temp_gemm_w(t, w, n, k, false, 0, st);
        Opnd xo = temp_operand(t, mode, x, (long)m * k);
        Epi e;
        e.bias = b;
        GemmCtx c{mode == HAT_B200_MODE_SIMT ? 0 : mode, mode == HAT_B200_MODE_SIMT, t.err};
        gemm_linear(c, xo, t.g, Dst{y, nullptr}, m, e, st);
        finish_kernel_call(t);
    });
}

int hat_b200_conv3x3(int mode, const float* x, const float* w, const float* b, float* y, int hgt, int wid,
                     int cin, int cout, void* stream) {
    return guarded(nullptr, 0, [&] {
        cudaStream_t st = (cudaStream_t)stream;
        TempW t;
        temp_gemm_w(t, w, cout, cin, true, cin, st);
        Opnd xo = temp_operand(t, mode, x, (long)hgt * wid * cin);
        Epi e;
        e.bias = b;
        GemmCtx c{mode == HAT_B200_MODE_SIMT ? 0 : mode, mode == HAT_B200_MODE_SIMT, t.err};
        gemm_conv3x3(c, xo, t.g, Dst{y, nullptr}, hgt, wid, e, st);
        finish_kernel_call(t);
    });
}

int hat_b200_window_attention(int mode, const float* qkv, const float* table, float* out, int hp, int wp, int c,
                              int heads, int shift, void* stream) {
    return guarded(nullptr, 0, [&] {
        Plan p = Plan::make(hp, wp, 16);
        if (p.hp != hp || p.wp != wp) throw Error(1, "window attention: plane is not a window multiple");
        TempW t;
        t.st = (cudaStream_t)stream;
        HAT_CUDA(cudaMallocAsync(&t.err, sizeof(int), t.st));
        HAT_CUDA(cudaMemsetAsync(t.err, 0, sizeof(int), t.st));
        launch_window_attention(mode == HAT_B200_MODE_SIMT ? 0 : mode, mode == HAT_B200_MODE_SIMT, qkv, table,
                                Dst{out, nullptr}, p, c, heads, shift, t.err, t.st);
        finish_kernel_call(t);
    });
}

int hat_b200_overlap_attention(int mode, const float* qkv, const float* table, float* out, int hp, int wp,
                               int c, int heads, void* stream) {
    return guarded(nullptr, 0, [&] {
        Plan p = Plan::make(hp, wp, 16);
        if (p.hp != hp || p.wp != wp) throw Error(1, "overlap attention: plane is not a window multiple");
        TempW t;
        t.st = (cudaStream_t)stream;
        HAT_CUDA(cudaMallocAsync(&t.err, sizeof(int), t.st));
        HAT_CUDA(cudaMemsetAsync(t.err, 0, sizeof(int), t.st));
        launch_overlap_attention(mode == HAT_B200_MODE_SIMT ? 0 : mode, mode == HAT_B200_MODE_SIMT, qkv, table,
                                 Dst{out, nullptr}, p, c, heads, t.err, t.st);
        finish_kernel_call(t);
    });
}

}  // extern "C"
