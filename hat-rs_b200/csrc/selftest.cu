// --cuda-selftest (src/selftest.rs:437-523): every kernel against a host twin on seeded
// inputs, at geometries that include non-square planes and the shift mask's wrap.
// No checkpoint is needed.
#include <array>
#include <cmath>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "../../include/hat_b200.h"
#include "common.cuh"

using namespace hat;

namespace {

struct Dev {
    float* p = nullptr;
    explicit Dev(const std::vector<float>& h) {
        HAT_CUDA(cudaMalloc(&p, h.size() * sizeof(float) + 16));
        HAT_CUDA(cudaMemcpy(p, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    explicit Dev(size_t n) {
        HAT_CUDA(cudaMalloc(&p, n * sizeof(float) + 16));
        HAT_CUDA(cudaMemset(p, 0, n * sizeof(float)));
    }
    ~Dev() { cudaFree(p); }
    std::vector<float> get(size_t n) const {
        std::vector<float> h(n);
        HAT_CUDA(cudaMemcpy(h.data(), p, n * sizeof(float), cudaMemcpyDeviceToHost));
        return h;
    }
};

std::vector<float> rnd(size_t n, unsigned seed, float lo = -1.f, float hi = 1.f) {
    std::mt19937 g(seed);
    std::uniform_real_distribution<float> u(lo, hi);
    std::vector<float> v(n);
    for (auto& x : v) x = u(g);
    return v;
}

double maxdiff(const std::vector<float>& a, const std::vector<double>& b) {
    double m = 0;
    for (size_t i = 0; i < a.size(); ++i) m = std::max(m, std::fabs((double)a[i] - b[i]));
    return m;
}

struct Log {
    std::string s;
    int fails = 0;
    void check(const std::string& what, double diff, double tol) {
        char buf[256];
        bool ok = diff <= tol && std::isfinite(diff);
        snprintf(buf, sizeof buf, "%-48s max |diff| %.3e (tol %.0e) %s\n", what.c_str(), diff, tol, ok ? "ok" : "FAIL");
        s += buf;
        if (!ok) ++fails;
    }
};

// Host twin of the window attention of one head of one window (hat_arch.py:165-196).
void attn_twin(const std::vector<float>& qkv, const std::vector<float>& tab, std::vector<double>& out, int hp,
               int wp, int c, int heads, int shift, bool oca) {
    const int win = 16, owin = 24, opad = 4, nx = wp / win, ny = hp / win, d = c / heads;
    const int nk = oca ? owin * owin : win * win;
    const int trows = oca ? 39 * 39 : 31 * 31;
    auto band = [&](int v, int n) { return v < n - win ? 0 : (v < n - shift ? 1 : 2); };
    std::vector<double> s(nk);
    for (int wy = 0; wy < ny; ++wy)
        for (int wx = 0; wx < nx; ++wx)
            for (int h = 0; h < heads; ++h)
                for (int t = 0; t < win * win; ++t) {
                    int qy = t / win, qx = t % win;
                    long qpos = oca ? (long)(wy * win + qy) * wp + wx * win + qx
                                    : (long)((wy * win + qy + shift) % hp) * wp + (wx * win + qx + shift) % wp;
                    double mx = -1e300;
                    for (int j = 0; j < nk; ++j) {
                        long kpos;
                        bool ok = true;
                        int ky = oca ? j / owin : j / win, kx = oca ? j % owin : j % win;
                        if (oca) {
                            int Y = wy * win - opad + ky, X = wx * win - opad + kx;
                            ok = Y >= 0 && Y < hp && X >= 0 && X < wp;
                            kpos = (long)Y * wp + X;
                        } else {
                            kpos = (long)((wy * win + ky + shift) % hp) * wp + (wx * win + kx + shift) % wp;
                        }
                        double dot = 0;
                        for (int i = 0; i < d; ++i) {
                            double q = (double)(qkv[qpos * 3 * c + h * d + i] * (1.f / sqrtf((float)d)));
                            double k = ok ? qkv[kpos * 3 * c + c + h * d + i] : 0.0;
                            dot += q * k;
                        }
                        int bi = oca ? ((ky - qy - 7) * 39 + (kx - qx - 7) + trows) % trows
                                     : (qy - ky + 15) * 31 + (qx - kx + 15);
                        double v = dot + tab[bi * heads + h];
                        if (!oca && shift) {
                            int lq = band(wy * win + qy, hp) * 3 + band(wx * win + qx, wp);
                            int lk = band(wy * win + ky, hp) * 3 + band(wx * win + kx, wp);
                            if (lq != lk) v += -100.0;
                        }
                        s[j] = v;
                        mx = std::max(mx, v);
                    }
                    double sum = 0;
                    for (int j = 0; j < nk; ++j) sum += (s[j] = std::exp(s[j] - mx));
                    for (int i = 0; i < d; ++i) {
                        double a = 0;
                        for (int j = 0; j < nk; ++j) {
                            long kpos;
                            bool ok = true;
                            int ky = oca ? j / owin : j / win, kx = oca ? j % owin : j % win;
                            if (oca) {
                                int Y = wy * win - opad + ky, X = wx * win - opad + kx;
                                ok = Y >= 0 && Y < hp && X >= 0 && X < wp;
                                kpos = (long)Y * wp + X;
                            } else {
                                kpos = (long)((wy * win + ky + shift) % hp) * wp + (wx * win + kx + shift) % wp;
                            }
                            a += s[j] * (ok ? qkv[kpos * 3 * c + 2 * c + h * d + i] : 0.0);
                        }
                        out[qpos * c + h * d + i] = a / sum;
                    }
                }
}

void run_all(Log& log) {
    // Linears: the HAB's shapes at a small token count, including a ragged M.
    for (auto sh : std::vector<std::array<int, 3>>{{1000, 432, 144}, {517, 144, 288}, {300, 540, 180}}) {
        int m = sh[0], n = sh[1], k = sh[2];
        auto x = rnd((size_t)m * k, 1), w = rnd((size_t)n * k, 2, -0.1f, 0.1f), b = rnd(n, 3);
        std::vector<double> ref((size_t)m * n);
        for (int i = 0; i < m; ++i)
            for (int j = 0; j < n; ++j) {
                double a = b[j];
                for (int q = 0; q < k; ++q) a += (double)x[(size_t)i * k + q] * w[(size_t)j * k + q];
                ref[(size_t)i * n + j] = a;
            }
        Dev dx(x), dw(w), db(b), dy((size_t)m * n);
        for (int mode : {HAT_B200_MODE_SIMT, HAT_B200_MODE_PARITY}) {
            int rc = hat_b200_linear(mode, dx.p, dw.p, db.p, dy.p, m, n, k, nullptr);
            HAT_CUDA(cudaDeviceSynchronize());
            log.check(std::string(mode == HAT_B200_MODE_SIMT ? "simt " : "tcgen05 3xtf32 ") + "linear " +
                          std::to_string(m) + "x" + std::to_string(n) + "x" + std::to_string(k),
                      rc ? 1e9 : maxdiff(dy.get((size_t)m * n), ref), 2e-5);
        }
    }
    // 3x3 convs: the CAB pair, the body conv, the head's thin ends, non-square planes.
    for (auto sh : std::vector<std::array<int, 4>>{{32, 48, 144, 6}, {48, 32, 6, 144}, {16, 16, 144, 144},
                                                  {32, 16, 3, 144}, {16, 32, 64, 3}, {16, 16, 60, 180}}) {
        int hg = sh[0], wd = sh[1], ci = sh[2], co = sh[3];
        auto x = rnd((size_t)hg * wd * ci, 4), w = rnd((size_t)co * ci * 9, 5, -0.1f, 0.1f), b = rnd(co, 6);
        std::vector<double> ref((size_t)hg * wd * co);
        for (int y = 0; y < hg; ++y)
            for (int xx = 0; xx < wd; ++xx)
                for (int o = 0; o < co; ++o) {
                    double a = b[o];
                    for (int dy = 0; dy < 3; ++dy)
                        for (int dx = 0; dx < 3; ++dx) {
                            int sy = y + dy - 1, sx = xx + dx - 1;
                            if (sy < 0 || sy >= hg || sx < 0 || sx >= wd) continue;
                            for (int i = 0; i < ci; ++i)
                                a += (double)x[((size_t)sy * wd + sx) * ci + i] * w[(((size_t)o * ci + i) * 3 + dy) * 3 + dx];
                        }
                    ref[((size_t)y * wd + xx) * co + o] = a;
                }
        Dev dx(x), dw(w), db(b), dy((size_t)hg * wd * co);
        for (int mode : {HAT_B200_MODE_SIMT, HAT_B200_MODE_PARITY}) {
            int rc = hat_b200_conv3x3(mode, dx.p, dw.p, db.p, dy.p, hg, wd, ci, co, nullptr);
            HAT_CUDA(cudaDeviceSynchronize());
            log.check(std::string(mode == HAT_B200_MODE_SIMT ? "simt " : "tcgen05 3xtf32 ") + "conv3x3 " +
                          std::to_string(hg) + "x" + std::to_string(wd) + " " + std::to_string(ci) + "->" +
                          std::to_string(co),
                      rc ? 1e9 : maxdiff(dy.get((size_t)hg * wd * co), ref),
                      // The tensor core adds each MMA's partial sum into the fp32
                      // accumulator with truncation, so a K = 9*144 conv at these
                      // magnitudes (|y| ~ 1) carries ~1e-5..1e-4 of one-sided error.
                      mode == HAT_B200_MODE_SIMT ? 5e-5 : 1.5e-4);
        }
    }
    // Attentions: both head dims, shifted and not, square and not.
    for (auto sh : std::vector<std::array<int, 4>>{{32, 48, 144, 8}, {48, 32, 144, 0}, {16, 16, 180, 8}, {32, 32, 180, 0}}) {
        int hp = sh[0], wp = sh[1], c = sh[2], shift = sh[3], heads = 6;
        auto qkv = rnd((size_t)hp * wp * 3 * c, 7);
        auto tsa = rnd(961 * heads, 8, -0.5f, 0.5f), toca = rnd(1521 * heads, 9, -0.5f, 0.5f);
        Dev dq(qkv), dts(tsa), dto(toca), dout((size_t)hp * wp * c);
        std::vector<double> ref((size_t)hp * wp * c), refo((size_t)hp * wp * c);
        attn_twin(qkv, tsa, ref, hp, wp, c, heads, shift, false);
        attn_twin(qkv, toca, refo, hp, wp, c, heads, 0, true);
        for (int mode : {HAT_B200_MODE_SIMT, HAT_B200_MODE_PARITY}) {
            const std::string tag = mode == HAT_B200_MODE_SIMT ? "simt " : "tcgen05 3xtf32 ";
            int rc = hat_b200_window_attention(mode, dq.p, dts.p, dout.p, hp, wp, c, heads, shift, nullptr);
            HAT_CUDA(cudaDeviceSynchronize());
            log.check(tag + "window attention " + std::to_string(hp) + "x" + std::to_string(wp) + " c" +
                          std::to_string(c) + " shift " + std::to_string(shift),
                      rc ? 1e9 : maxdiff(dout.get((size_t)hp * wp * c), ref), 2e-5);
            rc = hat_b200_overlap_attention(mode, dq.p, dto.p, dout.p, hp, wp, c, heads, nullptr);
            HAT_CUDA(cudaDeviceSynchronize());
            log.check(tag + "overlap attention " + std::to_string(hp) + "x" + std::to_string(wp) + " c" +
                          std::to_string(c),
                      rc ? 1e9 : maxdiff(dout.get((size_t)hp * wp * c), refo), 2e-5);
        }
    }
}

__global__ void k_gelu_probe(float* out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = gelu_fast(-10.f + 20.f * (float)i / (float)(n - 1));
}

// The GELU the tensor-core epilogues use (gelu_fast, erf after Abramowitz & Stegun 7.1.26)
// against the exact GELU in double precision over [-10, 10].
void gelu_check(Log& log) {
    const int n = 1 << 20;
    Dev d((size_t)n);
    k_gelu_probe<<<(n + 255) / 256, 256>>>(d.p, n);
    HAT_CUDA(cudaGetLastError());
    HAT_CUDA(cudaDeviceSynchronize());
    const std::vector<float> got = d.get((size_t)n);
    std::vector<double> ref((size_t)n);
    for (int i = 0; i < n; ++i) {
        const double x = (double)(-10.f + 20.f * (float)i / (float)(n - 1));
        ref[i] = 0.5 * x * (1.0 + std::erf(x / std::sqrt(2.0)));
    }
    log.check("gelu (erf after A&S 7.1.26) on [-10, 10]", maxdiff(got, ref), 1e-6);
}

}  // namespace

extern "C" int hat_b200_selftest(int device, char* log_out, size_t loglen) {
    Log log;
    int rc = HAT_B200_OK;
    try {
        HAT_CUDA(cudaSetDevice(device));
        run_all(log);
        gelu_check(log);
        if (log.fails) rc = HAT_B200_ESELFTEST;
    } catch (const std::exception& e) {
        log.s += std::string("selftest aborted: ") + e.what() + "\n";
        rc = HAT_B200_ECUDA;
    }
    if (log_out && loglen) {
        size_t n = std::min(log.s.size(), loglen - 1);
        memcpy(log_out, log.s.data(), n);
        log_out[n] = 0;
    }
    return rc;
}
