// conv_last of the head (hat_arch.py:966; src/gpu.rs:650-653): a 3x3 conv from the head's
// 64 channels to 3 at the output resolution, with the crop and `v / img_range + mean`
// of Pre::finish (src/backend.rs:94-109) in its store, written as the planar output.
//
// N = 3 leaves a tensor-core tile almost empty, and the implicit GEMM reads each input
// pixel once per tap (nine times, from L2). This kernel is a bandwidth kernel instead:
// a CTA stages an 8 x 32 output tile's (8+2) x (32+2) input pixels as fp32 in shared
// memory (the hi + lo pair summed, so the arithmetic is fp32), 32 channels at a time so
// that three CTAs fit an SM and one CTA's staging overlaps another's arithmetic, and each
// thread computes one output pixel's 3 channels with fp32 FMAs. The 1728 weights sit in
// shared memory too, ordered (tap, 4 input channels, output channel, 4) so that the 12
// weights one input float4 meets are three broadcast 16-byte loads. (Weights as kernel
// parameters, read as constant operands, measured 1.8 ms a launch at 2048x2048: the
// constant cache could not hold the 6.9 KB.) Per output pixel it reads 256 bytes of input
// (x1.33 for the halo) and writes 12.
#include "common.cuh"
#include "conv_last.h"

namespace hat {

namespace {

constexpr int TW = 32, TH = 8;            // output tile: columns x rows (one thread per pixel)
constexpr int SW = TW + 2, SH = TH + 2;   // staged input tile with the 3x3 halo
constexpr int CH = 32;                    // channels staged at a time
constexpr int PS = CH + 4;                // floats per staged pixel: 36 keeps LDS.128 conflict-free
constexpr int NW = 3 * CL_CIN * 9;          // weights
constexpr size_t SMEM = ((size_t)SH * SW * PS + NW) * sizeof(float);

struct Geo {
    int hgt, wid;       // the input view (rows outside it are the conv's zero padding)
    int y_lo, y_hi;     // output rows of the view to compute
    int oh, ow, oy0;    // planar output: crop and the output row of view row 0
    float img_range, mean[3];
};

// Four consecutive channels of pixel element `e` (an index into the [hgt][wid][64] plane)
// as fp32: the fp16 pair or tf32 pair summed, or the plain fp32 plane.
__device__ __forceinline__ float4 load4(const Opnd& x, long e) {
    if (x.lo && x.h16) {
        const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(x.hi) + e);
        const uint2 l = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(x.lo) + e);
        const float2 h0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
        const float2 h1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
        const float2 l0 = __half22float2(*reinterpret_cast<const __half2*>(&l.x));
        const float2 l1 = __half22float2(*reinterpret_cast<const __half2*>(&l.y));
        return make_float4(h0.x + l0.x, h0.y + l0.y, h1.x + l1.x, h1.y + l1.y);
    }
    float4 v = *reinterpret_cast<const float4*>(x.hi + e);
    if (x.lo) {
        const float4 l = *reinterpret_cast<const float4*>(x.lo + e);
        v.x += l.x;
        v.y += l.y;
        v.z += l.z;
        v.w += l.w;
    }
    return v;
}

__global__ void __launch_bounds__(TW * TH, 3)
    k_conv_last(const Opnd x, const float* __restrict__ w, const float* __restrict__ bias, float* __restrict__ out,
                const Geo g) {
    extern __shared__ float4 sm4[];
    float4* wsm = sm4 + SH * SW * (PS / 4);  // [tap][ci / 4][co][4]
    const int x0 = blockIdx.x * TW, y0 = g.y_lo + blockIdx.y * TH;
    for (int i = threadIdx.x; i < NW; i += TW * TH) {
        const int co = i / (CL_CIN * 9), r = i - co * CL_CIN * 9, ci = r / 9, tap = r - ci * 9;  // [co][ci][ky][kx]
        reinterpret_cast<float*>(wsm)[((tap * (CL_CIN / 4) + ci / 4) * 3 + co) * 4 + (ci & 3)] = w[i];
    }
    const int tx = threadIdx.x % TW, ty = threadIdx.x / TW;
    const int oy = y0 + ty, ox = x0 + tx;
    float a0 = bias[0], a1 = bias[1], a2 = bias[2];
#pragma unroll 1
    for (int c0 = 0; c0 < CL_CIN; c0 += CH) {
        // Stage channels [c0, c0 + CH) of the input tile: pixel (r, c) of the tile is view pixel
        // (y0 - 1 + r, x0 - 1 + c). Each thread issues a round's loads before any of its stores.
        constexpr int PIECES = SH * SW * (CH / 4), PER = (PIECES + TW * TH - 1) / (TW * TH), RND = (PER + 1) / 2;
        if (c0) __syncthreads();  // the previous channels' arithmetic is done with the tile
#pragma unroll 1
        for (int r0 = 0; r0 < PER; r0 += RND) {
            float4 v[RND];
#pragma unroll
            for (int u = 0; u < RND; ++u) {
                const int i = threadIdx.x + (r0 + u) * TW * TH;
                const int pix = i / (CH / 4), c4 = i % (CH / 4);
                const int r = pix / SW, c = pix % SW;
                const int gy = y0 - 1 + r, gx = x0 - 1 + c;
                v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (i < PIECES && gy >= 0 && gy < g.hgt && gx >= 0 && gx < g.wid)
                    v[u] = load4(x, ((long)gy * g.wid + gx) * CL_CIN + c0 + 4 * c4);
            }
#pragma unroll
            for (int u = 0; u < RND; ++u) {
                const int i = threadIdx.x + (r0 + u) * TW * TH;
                if (i < PIECES) sm4[(i / (CH / 4)) * (PS / 4) + i % (CH / 4)] = v[u];
            }
        }
        __syncthreads();
        if (oy < g.y_hi && ox < g.wid) {
#pragma unroll
            for (int ky = 0; ky < 3; ++ky)
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const float4* px = sm4 + ((ty + ky) * SW + tx + kx) * (PS / 4);
                    const float4* wt = wsm + ((ky * 3 + kx) * (CL_CIN / 4) + c0 / 4) * 3;
#pragma unroll 4
                    for (int c4 = 0; c4 < CH / 4; ++c4) {
                        const float4 v = px[c4], w0 = wt[3 * c4], w1 = wt[3 * c4 + 1], w2 = wt[3 * c4 + 2];
                        a0 = fmaf(v.x, w0.x, fmaf(v.y, w0.y, fmaf(v.z, w0.z, fmaf(v.w, w0.w, a0))));
                        a1 = fmaf(v.x, w1.x, fmaf(v.y, w1.y, fmaf(v.z, w1.z, fmaf(v.w, w1.w, a1))));
                        a2 = fmaf(v.x, w2.x, fmaf(v.y, w2.y, fmaf(v.z, w2.z, fmaf(v.w, w2.w, a2))));
                    }
                }
        }
    }
    if (oy >= g.y_hi || ox >= g.wid) return;
    const int gy = oy + g.oy0;
    if (gy < 0 || gy >= g.oh || ox >= g.ow) return;
    const long plane = (long)g.oh * g.ow, o = (long)gy * g.ow + ox;
    out[o] = a0 / g.img_range + g.mean[0];
    out[plane + o] = a1 / g.img_range + g.mean[1];
    out[2 * plane + o] = a2 / g.img_range + g.mean[2];
}

}  // namespace

bool conv_last_ok(const Opnd& x, int cin, int cout) {
    if (cin != CL_CIN || cout != 3) return false;
    // 16-byte (fp32 planes) or 8-byte (fp16 pairs) channel loads
    const uintptr_t a = reinterpret_cast<uintptr_t>(x.hi) | reinterpret_cast<uintptr_t>(x.lo);
    return (a & 15) == 0;
}

long launch_conv_last(const Opnd& x, const float* w, const float* bias, float* out, int hgt, int wid, const Epi& e,
                      cudaStream_t st) {
    Geo g;
    g.hgt = hgt;
    g.wid = wid;
    g.y_lo = e.y_hi > 0 ? e.y_lo : 0;  // y_hi == 0: every row
    g.y_hi = e.y_hi > 0 ? e.y_hi : hgt;
    g.oh = e.oh;
    g.ow = e.ow;
    g.oy0 = e.oy0;
    g.img_range = e.img_range;
    for (int i = 0; i < 3; ++i) g.mean[i] = e.mean[i];
    if (g.y_hi <= g.y_lo) return 0;
    allow_dyn_smem(k_conv_last, SMEM);
    dim3 grid((unsigned)((wid + TW - 1) / TW), (unsigned)((g.y_hi - g.y_lo + TH - 1) / TH));
    k_conv_last<<<grid, TW * TH, SMEM, st>>>(x, w, bias, out, g);
    HAT_CUDA(cudaGetLastError());
    count_launch();
    return 0;
}

}  // namespace hat
