// CUDA-core fp32 window attention: the HAB's (shifted) 16x16 window attention and the
// OCAB's 16x16-query / 24x24-key overlapping attention, read straight from the
// token-major qkv plane. The window partition, the cyclic roll, the nn.Unfold of the
// keys (zero outside the plane), the relative-position bias gather and the shift mask
// are all folded into the addressing: nothing is materialised.
#include "common.cuh"

namespace hat {

// Region of a shifted-frame coordinate for calculate_mask's three bands
// (hat_arch.py:921-941): [0, n-win) → 0, [n-win, n-shift) → 1, [n-shift, n) → 2.
__device__ __forceinline__ int band(int v, int n, int win, int shift) {
    return v < n - win ? 0 : (v < n - shift ? 1 : 2);
}

// One CTA per (window, head); one thread per query (256 = win*win). Keys and values
// of the window are staged in shared memory; each thread runs an online softmax over
// chunks of 32 keys. OCA selects the overlapping attention.
template <int D, bool OCA>
__global__ void __launch_bounds__(256) k_attn_simt(const float* __restrict__ qkv,
                                                   const float* __restrict__ table,
                                                   Dst out, int hp, int wp, int c,
                                                   int heads, int shift, float scale) {
    constexpr int WIN = 16, OWIN = 24, OPAD = 4;
    constexpr int DP = (D + 3) / 4 * 4;
    constexpr int NK = OCA ? OWIN * OWIN : WIN * WIN;
    constexpr int TROWS = OCA ? (WIN + OWIN - 1) * (WIN + OWIN - 1) : (2 * WIN - 1) * (2 * WIN - 1);
    extern __shared__ __align__(16) float sm[];
    float* Ks = sm;
    float* Vs = Ks + NK * DP;
    float* tab = Vs + NK * DP;

    const int tid = threadIdx.x;
    const int wi = blockIdx.x, h = blockIdx.y;
    const int nx = wp / WIN;
    const int wy = wi / nx, wx = wi - wy * nx;
    const long c3 = 3L * c;

    for (int i = tid; i < TROWS; i += 256) tab[i] = table[(long)i * heads + h];
    for (int idx = tid; idx < NK * D; idx += 256) {
        int j = idx / D, dd = idx - j * D;
        bool ok = true;
        long pos;
        if (OCA) {
            int ky = j / OWIN, kx = j - ky * OWIN;
            int Y = wy * WIN - OPAD + ky, X = wx * WIN - OPAD + kx;
            ok = Y >= 0 && Y < hp && X >= 0 && X < wp;
            pos = (long)Y * wp + X;
        } else {
            int ky = j / WIN, kx = j - ky * WIN;
            int Y = (wy * WIN + ky + shift) % hp, X = (wx * WIN + kx + shift) % wp;
            pos = (long)Y * wp + X;
        }
        const float* src = qkv + pos * c3 + c + (long)h * D + dd;
        Ks[j * DP + dd] = ok ? src[0] : 0.f;
        Vs[j * DP + dd] = ok ? src[c] : 0.f;
    }

    const int qy = tid / WIN, qx = tid - qy * WIN;
    long qpos;
    if (OCA)
        qpos = (long)(wy * WIN + qy) * wp + wx * WIN + qx;
    else
        qpos = (long)((wy * WIN + qy + shift) % hp) * wp + (wx * WIN + qx + shift) % wp;
    float q[D];
#pragma unroll
    for (int dd = 0; dd < D; ++dd) q[dd] = qkv[qpos * c3 + (long)h * D + dd] * scale;
    const bool masked = !OCA && shift > 0;
    const int lq = masked ? band(wy * WIN + qy, hp, WIN, shift) * 3 + band(wx * WIN + qx, wp, WIN, shift) : 0;
    __syncthreads();

    float m = -INFINITY, l = 0.f, acc[D];
#pragma unroll
    for (int dd = 0; dd < D; ++dd) acc[dd] = 0.f;

    for (int j0 = 0; j0 < NK; j0 += 32) {
        float s[32];
        float cmax = -INFINITY;
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            int j = j0 + u;
            const float* kr = Ks + j * DP;
            float dot = 0.f;
#pragma unroll
            for (int dd = 0; dd < D; ++dd) dot = fmaf(q[dd], kr[dd], dot);
            int bi;
            if (OCA) {
                int ky = j / OWIN, kx = j - ky * OWIN;
                bi = (ky - qy + WIN - OWIN + 1) * (WIN + OWIN - 1) + (kx - qx + WIN - OWIN + 1);
                if (bi < 0) bi += TROWS;
            } else {
                int ky = j / WIN, kx = j - ky * WIN;
                bi = (qy - ky + WIN - 1) * (2 * WIN - 1) + (qx - kx + WIN - 1);
            }
            float sv = dot + tab[bi];
            if (masked) {
                int ky = j / WIN, kx = j - ky * WIN;
                int lk = band(wy * WIN + ky, hp, WIN, shift) * 3 + band(wx * WIN + kx, wp, WIN, shift);
                if (lk != lq) sv += -100.f;
            }
            s[u] = sv;
            cmax = fmaxf(cmax, sv);
        }
        float mn = fmaxf(m, cmax);
        float corr = expf(m - mn);
        l *= corr;
#pragma unroll
        for (int dd = 0; dd < D; ++dd) acc[dd] *= corr;
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            float p = expf(s[u] - mn);
            l += p;
            const float* vr = Vs + (j0 + u) * DP;
#pragma unroll
            for (int dd = 0; dd < D; ++dd) acc[dd] = fmaf(p, vr[dd], acc[dd]);
        }
        m = mn;
    }
    float inv = 1.f / l;
    const long o = qpos * c + (long)h * D;
#pragma unroll
    for (int dd = 0; dd < D; ++dd) put(out, o + dd, acc[dd] * inv);
}

template <int D, bool OCA>
static void run_attn(const float* qkv, const float* table, Dst out, const Plan& p, int c,
                     int heads, int shift, cudaStream_t st) {
    constexpr int DP = (D + 3) / 4 * 4;
    constexpr int NK = OCA ? 576 : 256;
    constexpr int TROWS = OCA ? 39 * 39 : 31 * 31;
    size_t smem = (2 * NK * DP + TROWS) * sizeof(float);
    allow_dyn_smem(k_attn_simt<D, OCA>, smem);
    dim3 grid(p.nw(), heads);
    k_attn_simt<D, OCA><<<grid, 256, smem, st>>>(qkv, table, out, p.hp, p.wp, c, heads, shift,
                                                 1.f / sqrtf((float)D));
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

static void check_geometry(const Plan& p, int c, int heads) {
    if (p.win != 16 || p.owin != 24)
        throw Error(1, "attention: the kernels are built for window 16 / overlap window 24");
    if (heads <= 0 || c % heads) throw Error(1, "attention: c is not divisible by heads");
}

void launch_window_attention_simt(const float* qkv, const float* table, Dst out, const Plan& p,
                                  int c, int heads, int shift, cudaStream_t st) {
    check_geometry(p, c, heads);
    int d = c / heads;
    if (d == 24)
        run_attn<24, false>(qkv, table, out, p, c, heads, shift, st);
    else if (d == 30)
        run_attn<30, false>(qkv, table, out, p, c, heads, shift, st);
    else
        throw Error(1, "window attention: head dim " + std::to_string(d) + " is not 24 or 30");
}

void launch_overlap_attention_simt(const float* qkv, const float* table, Dst out, const Plan& p,
                                   int c, int heads, cudaStream_t st) {
    check_geometry(p, c, heads);
    int d = c / heads;
    if (d == 24)
        run_attn<24, true>(qkv, table, out, p, c, heads, 0, st);
    else if (d == 30)
        run_attn<30, true>(qkv, table, out, p, c, heads, 0, st);
    else
        throw Error(1, "overlap attention: head dim " + std::to_string(d) + " is not 24 or 30");
}

}  // namespace hat
