// CUDA-core fp32 GEMM for the token linears and the 3x3 convolutions (as implicit
// GEMM over K = 9 * cin), with the fused epilogues the HAT graph needs. This is the
// exact-fp32 path: it serves shapes the tensor-core kernel does not take and is the
// on-device cross-check for it.
#include "umma.cuh"

namespace hat {

__device__ __forceinline__ float4 ld4o(const Opnd& o, long i) {
    if (o.lo && o.h16) {
        const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(o.hi) + i);
        const uint2 l = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(o.lo) + i);
        const float2 h0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
        const float2 h1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
        const float2 l0 = __half22float2(*reinterpret_cast<const __half2*>(&l.x));
        const float2 l1 = __half22float2(*reinterpret_cast<const __half2*>(&l.y));
        return make_float4(h0.x + l0.x, h0.y + l0.y, h1.x + l1.x, h1.y + l1.y);
    }
    float4 v = *reinterpret_cast<const float4*>(o.hi + i);
    if (o.lo) {
        const float4 l = *reinterpret_cast<const float4*>(o.lo + i);
        v.x += l.x;
        v.y += l.y;
        v.z += l.z;
        v.w += l.w;
    }
    return v;
}

// A operand of a token linear: row-major [m][k] (hi + lo when split).
struct ALinear {
    Opnd x;
    int k;
    __device__ __forceinline__ float ld(long m, int kk) const { return get(x, m * k + kk); }
    __device__ __forceinline__ float4 ld4(long m, int kk) const { return ld4o(x, m * k + kk); }
};

// A operand of a 3x3 conv over a token plane [hgt][wid][cin]: row m is pixel m, column
// kk = tap * cin + ci reads channel ci of the neighbour (dy, dx) = (tap/3 - 1, tap%3 - 1),
// zero outside the plane (Conv2d padding 1).
struct AConv {
    Opnd x;
    int hgt, wid, cin, ldc;  // ldc: channel stride of the plane (>= cin)
    __device__ __forceinline__ long at(long m, int kk, bool& ok) const {
        int tap = kk / cin, ci = kk - tap * cin;
        int y = (int)(m / wid) + tap / 3 - 1, xx = (int)(m % wid) + tap % 3 - 1;
        ok = y >= 0 && y < hgt && xx >= 0 && xx < wid;
        return ((long)y * wid + xx) * ldc + ci;
    }
    __device__ __forceinline__ float ld(long m, int kk) const {
        bool ok;
        const long i = at(m, kk, ok);
        return ok ? get(x, i) : 0.f;
    }
    __device__ __forceinline__ float4 ld4(long m, int kk) const {
        bool ok;
        const long i = at(m, kk, ok);
        return ok ? ld4o(x, i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
};

__device__ __forceinline__ float apply_act(float v, int act) {
    if (act == ACT_GELU) return 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
    if (act == ACT_LEAKY) return v > 0.f ? v : 0.01f * v;
    return v;
}

// Store one finished value; `wid` is the plane width for the spatial epilogues.
__device__ __forceinline__ void epi_store(const Epi& e, const Dst& y, long gm, int gn, int n, float v,
                                          int wid) {
    if (e.planar_out) {
        int py = (int)(gm / wid), px = (int)(gm % wid);
        if (py + e.oy0 >= 0 && py + e.oy0 < e.oh && px < e.ow)
            y.hi[((long)gn * e.oh + py + e.oy0) * e.ow + px] =
                v / e.img_range + (gn == 0 ? e.mean[0] : gn == 1 ? e.mean[1] : e.mean[2]);
        return;
    }
    if (e.shuffle) {
        int r = e.shuffle, cout = n / (r * r);
        int c = gn / (r * r), rem = gn - c * r * r, i = rem / r, j = rem - i * r;
        int py = (int)(gm / wid), px = (int)(gm % wid);
        long oy = (long)py * r + i, ox = (long)px * r + j;
        put(y, (oy * ((long)wid * r) + ox) * cout + c, v);
        return;
    }
    long idx = gm * (e.ldo ? e.ldo : n) + gn;
    if (e.cx)
        v = (e.res[idx] + v) + (e.cx[idx] * e.gate[gn]) * e.cscale;
    else if (e.res)
        v = e.res[idx] + v;
    put(y, idx, v);
}

template <int BN, bool VEC, class AL>
__global__ void __launch_bounds__(256) k_gemm_simt(AL al, const float* __restrict__ w,
                                                   Dst y, long M, int N, int K,
                                                   Epi e, int wid) {
    constexpr int BM = 128, BK = 16, TN = BN / 16;
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Bs[BK][BN + 4];
    __shared__ float red[16][BN];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const long m0 = (long)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;
    float acc[8][TN];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

    for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            int idx = tid + r * 256, kq = idx & 3, mm = idx >> 2;
            long gm = m0 + mm;
            int gk = k0 + kq * 4;
            float v[4];
            if (VEC) {
                float4 t = (gm < M && gk < K) ? al.ld4(gm, gk) : make_float4(0.f, 0.f, 0.f, 0.f);
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = (gm < M && gk + u < K) ? al.ld(gm, gk + u) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) As[kq * 4 + u][mm] = v[u];
        }
        for (int idx = tid; idx < BN * 4; idx += 256) {
            int kq = idx & 3, nn = idx >> 2, gn = n0 + nn, gk = k0 + kq * 4;
            float v[4];
            if (VEC) {
                float4 t = (gn < N && gk < K) ? *reinterpret_cast<const float4*>(w + (long)gn * K + gk)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = (gn < N && gk + u < K) ? w[(long)gn * K + gk + u] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) Bs[kq * 4 + u][nn] = v[u];
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[8], b[TN];
            float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 8]);
            float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * 8 + 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
            a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
#pragma unroll
            for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }

    float cs[TN];
#pragma unroll
    for (int j = 0; j < TN; ++j) cs[j] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        long gm = m0 + ty * 8 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            int gn = n0 + tx + 16 * j;
            if (gn >= N) continue;
            float v = acc[i][j] + (e.bias ? e.bias[gn] : 0.f);
            v = apply_act(v, e.act);
            epi_store(e, y, gm, gn, N, v, wid);
            cs[j] += v;
        }
    }
    if (e.colsum) {
        // Deterministic: one partial row per M tile, summed in tile order by the gate.
#pragma unroll
        for (int j = 0; j < TN; ++j) red[ty][tx + 16 * j] = cs[j];
        __syncthreads();
        if (tid < BN && n0 + tid < N) {
            float s = 0.f;
#pragma unroll
            for (int r = 0; r < 16; ++r) s += red[r][tid];
            e.colsum[(long)blockIdx.x * N + n0 + tid] = s;
        }
    }
}

static int pick_bn(int n) {
    int best = 64, waste = 1 << 30;
    for (int bn : {64, 48, 32, 16}) {
        int wst = (n + bn - 1) / bn * bn - n;
        if (wst < waste) {
            waste = wst;
            best = bn;
        }
    }
    return best;
}

template <class AL>
static void run_simt(const AL& al, bool vec, const float* w, Dst y, long m, int n, int k,
                     const Epi& e, int wid, cudaStream_t st) {
    int bn = pick_bn(n);
    dim3 grid((unsigned)((m + 127) / 128), (unsigned)((n + bn - 1) / bn));
#define HAT_GEMM_CASE(BN)                                                                      \
    if (bn == BN) {                                                                            \
        if (vec)                                                                               \
            k_gemm_simt<BN, true, AL><<<grid, 256, 0, st>>>(al, w, y, m, n, k, e, wid);        \
        else                                                                                   \
            k_gemm_simt<BN, false, AL><<<grid, 256, 0, st>>>(al, w, y, m, n, k, e, wid);       \
    }
    HAT_GEMM_CASE(16)
    HAT_GEMM_CASE(32)
    HAT_GEMM_CASE(48)
    HAT_GEMM_CASE(64)
#undef HAT_GEMM_CASE
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

long simt_linear(Opnd x, const GemmW& w, Dst y, long m, const Epi& e, cudaStream_t st) {
    run_simt(ALinear{x, w.k}, w.k % 4 == 0, w.simt, y, m, w.n, w.k, e, 1, st);
    return (m + 127) / 128;
}

long simt_conv3x3(Opnd x, const GemmW& w, Dst y, int hgt, int wid, const Epi& e, cudaStream_t st) {
    const int ldc = w.cin_plane ? w.cin_plane : w.cin;
    const long m = (long)hgt * wid;
    run_simt(AConv{x, hgt, wid, w.cin, ldc}, w.cin % 4 == 0 && ldc % 4 == 0, w.simt, y, m, w.n, 9 * w.cin, e, wid,
             st);
    return (m + 127) / 128;
}

}  // namespace hat
