// Weight preparation for the GEMM kernels (once, at upload) and the dispatch between
// the tensor-core and CUDA-core GEMMs.
#include <cmath>

#include "umma.cuh"

namespace hat {

void plan_gemm_w(GemmW& g, int n, int k_or_cin, bool conv, int cin_plane, bool h16) {
    g.n = n;
    g.conv = conv;
    g.h16 = h16;
    g.scale = 1.f;
    if (conv) {
        g.cin = k_or_cin;
        g.k = 9 * k_or_cin;
        g.cin_plane = cin_plane;
        if (h16) {
            // One k-block of a tap covers 64 channels (128 bytes), or 16 (32 bytes) for a
            // plane narrower than 64; TMA needs 16-byte channel strides.
            const int chunk = cin_plane >= 64 ? 64 : 16;
            g.cinp = (k_or_cin + chunk - 1) / chunk * chunk;
            g.ckb = 2 * chunk;
            g.umma = cin_plane % 8 == 0 && cin_plane >= 16 && cin_plane >= k_or_cin && k_or_cin >= 4;
        } else {
            g.cinp = k_or_cin <= 8 ? 8 : (k_or_cin + 31) / 32 * 32;
            g.ckb = g.cinp == 8 ? 32 : 128;
            // Tensor cores need a 16-byte channel stride for TMA, and the channel chunk of a
            // tap must fit the plane's padded stride.
            g.umma = cin_plane % 4 == 0 && cin_plane >= (k_or_cin <= 8 ? 8 : 4) && k_or_cin >= 4;
        }
        g.k_pad = 9 * g.cinp;
    } else {
        g.k = k_or_cin;
        g.cin_plane = 0;
        g.ckb = 128;
        g.umma = k_or_cin % (h16 ? 8 : 4) == 0;
        g.k_pad = h16 ? (k_or_cin + 63) / 64 * 64 : (k_or_cin + 31) / 32 * 32;
    }
    g.bn = umma_bn(n);
    g.n_pad = (n + g.bn - 1) / g.bn * g.bn;
}

float h16_weight_factor(float max_abs) {
    if (!(max_abs > 0.f) || !std::isfinite(max_abs)) return 1.f;
    int ex = 0;
    std::frexp(max_abs, &ex);  // max_abs in [2^(ex-1), 2^ex)
    const int e = std::max(-100, std::min(100, 15 - ex));
    return std::ldexp(1.f, e);
}

size_t gemm_w_floats(const GemmW& g) {
    size_t s = (size_t)g.n * g.k;
    if (g.umma) s += 2 * (size_t)g.n_pad * g.k_pad;
    return s;
}

// simt: linear copy or conv reorder [n][cin][3][3] → [n][9][cin].
__global__ void k_prep_simt(const float* __restrict__ w, float* __restrict__ out, int n, int cin, bool conv) {
    long total = conv ? (long)n * cin * 9 : (long)n * cin;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        if (!conv) {
            out[i] = w[i];
        } else {
            int tap = (int)(i % 9);
            long r = i / 9;
            int ci = (int)(r % cin);
            int co = (int)(r / cin);
            out[((long)co * 9 + tap) * cin + ci] = w[i];
        }
    }
}

// hi/lo: the tensor-core layout [n_pad][k_pad] (conv: k = tap * cinp + ci), zero padded;
// tf32 pairs, or (H16) fp16 pairs of the weight times `factor`.
template <bool H16>
__global__ void k_prep_umma(const float* __restrict__ w, float* __restrict__ hi, float* __restrict__ lo, int n,
                            int k, int n_pad, int k_pad, bool conv, int cin, int cinp, float factor) {
    long total = (long)n_pad * k_pad;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int row = (int)(i / k_pad), kk = (int)(i % k_pad);
        float v = 0.f;
        if (row < n) {
            if (!conv) {
                if (kk < k) v = w[(long)row * k + kk];
            } else {
                int tap = kk / cinp, ci = kk - tap * cinp;
                if (tap < 9 && ci < cin) v = w[((long)row * cin + ci) * 9 + tap];
            }
        }
        if (H16) {
            __half h, l;
            split_h16(v * factor, h, l);
            reinterpret_cast<__half*>(hi)[i] = h;
            reinterpret_cast<__half*>(lo)[i] = l;
        } else {
            float h, l;
            split_tf32(v, h, l);
            hi[i] = h;
            lo[i] = l;
        }
    }
}

void launch_prep_gemm_w(const float* w, float* simt, float* hi, float* lo, const GemmW& g, cudaStream_t st) {
    k_prep_simt<<<256, 256, 0, st>>>(w, simt, g.n, g.conv ? g.cin : g.k, g.conv);
    HAT_CUDA(cudaGetLastError());
    count_launch();
    if (g.umma) {
        if (g.h16)
            k_prep_umma<true><<<512, 256, 0, st>>>(w, hi, lo, g.n, g.k, g.n_pad, g.k_pad, g.conv, g.cin, g.cinp,
                                                   1.f / g.scale);
        else
            k_prep_umma<false><<<512, 256, 0, st>>>(w, hi, lo, g.n, g.k, g.n_pad, g.k_pad, g.conv, g.cin, g.cinp, 1.f);
        HAT_CUDA(cudaGetLastError());
        count_launch();
    }
}

__global__ void k_prep_taps(const float* __restrict__ w, float* __restrict__ out, int cout, int cin) {
    const long total = 9L * cout * cin;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int ci = (int)(i % cin);
        const long r = i / cin;  // tap * cout + co
        const int co = (int)(r % cout), tap = (int)(r / cout);
        out[i] = w[((long)co * cin + ci) * 9 + tap];
    }
}

void launch_prep_taps(const float* w, float* out, int cout, int cin, cudaStream_t st) {
    k_prep_taps<<<64, 256, 0, st>>>(w, out, cout, cin);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

long gemm_linear(const GemmCtx& c, Opnd x, const GemmW& w, Dst y, long m, const Epi& e, cudaStream_t st) {
    // Parity mode needs the operand split by its producer; a plain plane (never the case
    // inside the forward) takes the exact CUDA-core path instead of losing precision.
    const bool ok = c.mode != 0 || x.lo;
    if (x.lo && x.h16 != w.h16) throw Error(1, "gemm: operand and weight split kinds differ");
    if (!c.simt_only && w.umma && ok && !e.planar_out && !e.shuffle)
        return umma_linear(c.mode, x, w, y, m, e, c.err, st);
    if (e.qkv_split) throw Error(1, "gemm: the qkv attention layout needs the tensor-core linear");
    return simt_linear(x, w, y, m, e, st);
}

long gemm_conv3x3(const GemmCtx& c, Opnd x, const GemmW& w, Dst y, int hgt, int wid, const Epi& e,
                  cudaStream_t st) {
    const bool ok = c.mode != 0 || x.lo;
    if (x.lo && x.h16 != w.h16) throw Error(1, "gemm: operand and weight split kinds differ");
    if (!c.simt_only && w.umma && ok && hgt % 8 == 0 && wid % 16 == 0)
        return umma_conv3x3(c.mode, x, w, y, hgt, wid, e, c.err, st);
    return simt_conv3x3(x, w, y, hgt, wid, e, st);
}

}  // namespace hat
