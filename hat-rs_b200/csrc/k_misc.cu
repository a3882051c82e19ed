// Bandwidth-bound kernels of the HAT forward: the input adjustment, LayerNorm over
// the channel axis, the conv weight reorder, and the channel-attention head.
#include "common.cuh"

namespace hat {

thread_local uint64_t* g_launch_counter = nullptr;

// ---------------------------------------------------------------- pre
// Pre::adjust (src/backend.rs:71-89): edge replication to the padded plane, then
// `(x - mean) * img_range`, written token-major [rows][wp][3]; local row i is padded row
// gy0 + i (rows outside the padded plane, a strip's halo at the image edge, are filled
// by the same clamping and never read as data).
__global__ void k_pre(const float* __restrict__ in, float* __restrict__ out, int h, int w, int rows,
                      int wp, int gy0, float m0, float m1, float m2, float range) {
    long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    long n = (long)rows * wp;
    if (i >= n) return;
    int y = gy0 + (int)(i / wp), x = (int)(i % wp);
    int sy = max(0, min(y, h - 1)), sx = min(x, w - 1);
    long src = (long)sy * w + sx, plane = (long)h * w;
    out[i * 3 + 0] = (in[src] - m0) * range;
    out[i * 3 + 1] = (in[plane + src] - m1) * range;
    out[i * 3 + 2] = (in[2 * plane + src] - m2) * range;
}

void launch_pre(const float* in, float* out, const Plan& p, const float mean[3], float img_range,
                cudaStream_t st) {
    long n = p.tokens();
    k_pre<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(in, out, p.h, p.w, p.rows, p.wp, p.gy0(), mean[0],
                                                       mean[1], mean[2], img_range);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

// ---------------------------------------------------------------- tap sum
// The CAB's first conv (c -> c/compress, 3x3, then GELU; hat_arch.py:50-53) when its
// output is narrow: a linear to 9*cout per-tap partial outputs reads the input plane
// once, and this kernel adds each pixel's nine neighbours' taps. One thread per pixel.
template <int CMAX>
__global__ void k_tapsum_gelu(const float* __restrict__ taps, int ldt, const float* __restrict__ bias, Dst out,
                              int ldo, int cout, int hp, int wp, int ylo, int yhi) {
    const long p = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= (long)hp * wp) return;
    const int y = (int)(p / wp), x = (int)(p - (long)y * wp);
    float acc[CMAX];
#pragma unroll
    for (int co = 0; co < CMAX; ++co) acc[co] = co < cout ? bias[co] : 0.f;
    const bool pairs = cout % 2 == 0 && ldt % 2 == 0;  // 8-byte loads of two channels
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
        const int yy = y + tap / 3 - 1, xx = x + tap % 3 - 1;
        if (yy < ylo || yy >= yhi || xx < 0 || xx >= wp) continue;
        const float* row = taps + ((long)yy * wp + xx) * ldt + tap * cout;
        if (pairs) {
#pragma unroll
            for (int co = 0; co < CMAX; co += 2)
                if (co < cout) {
                    const float2 t2 = *reinterpret_cast<const float2*>(row + co);
                    acc[co] += t2.x;
                    acc[co + 1] += t2.y;
                }
        } else {
#pragma unroll
            for (int co = 0; co < CMAX; ++co)
                if (co < cout) acc[co] += row[co];
        }
    }
    if (out.lo && out.h16 && ldo == 2 * CMAX) {
        // an fp16 pair plane of 2 * CMAX channels: the pixel's channels as 16-byte stores
        uint32_t hw[CMAX], lw[CMAX];
        bool big = false;
#pragma unroll
        for (int i = 0; i < CMAX; ++i) {
            float v2[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int co = 2 * i + k;
                const float a = co < CMAX ? acc[co < CMAX ? co : 0] : 0.f;
                v2[k] = co < cout ? gelu_fast(a) : 0.f;
                big |= beyond_h16(v2[k]);
            }
            split_h16x2(v2[0], v2[1], hw[i], lw[i]);
        }
        if (big && out.err) atomicCAS(out.err, 0, ERR_RANGE_GEMM);
        uint4* dh = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(out.hi) + p * ldo);
        uint4* dl = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(out.lo) + p * ldo);
#pragma unroll
        for (int i = 0; i < CMAX / 4; ++i) {
            dh[i] = make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
            dl[i] = make_uint4(lw[4 * i], lw[4 * i + 1], lw[4 * i + 2], lw[4 * i + 3]);
        }
        return;
    }
    // channels cout..ldo-1 (ldo <= 2 * CMAX) are written as zeros
#pragma unroll
    for (int co = 0; co < 2 * CMAX; ++co) {
        if (co >= ldo) break;
        const float a = co < CMAX ? acc[co < CMAX ? co : 0] : 0.f;
        const float v = co < cout ? gelu_fast(a) : 0.f;
        put(out, p * ldo + co, v);
    }
}

void launch_tapsum_gelu(const float* taps, int ldt, const float* bias, Dst out, int ldo, int cout, int hp, int wp,
                        int ylo, int yhi, cudaStream_t st) {
    if (cout > 8 || ldo > 16 || ldt < 9 * cout) throw Error(1, "tapsum: at most 8 output channels (16 stored)");
    const long n = (long)hp * wp;
    k_tapsum_gelu<8><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(taps, ldt, bias, out, ldo, cout, hp, wp, ylo, yhi);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

// ---------------------------------------------------------------- channel sums
// sum[c] = the `rows` partial rows [rows][c] added in row order (a strip's part of the
// channel-attention pool, before the sum over strips).
__global__ void k_rowsum(const float* __restrict__ partial, long rows, int c, float* __restrict__ sum) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < c; j += gridDim.x * blockDim.x) {
        float s = 0.f;
#pragma unroll 8
        for (long r = 0; r < rows; ++r) s += partial[r * c + j];
        sum[j] = s;
    }
}

void launch_rowsum(const float* partial, long rows, int c, float* sum, cudaStream_t st) {
    k_rowsum<<<(c + 127) / 128, 128, 0, st>>>(partial, rows, c, sum);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

// ---------------------------------------------------------------- layernorm
// One warp per token; the row stays in registers: the mean first, then the biased
// variance of the centred values (src/cpu.rs:563-581), eps 1e-5.
template <int MAXV>
__global__ void k_layernorm(const float* __restrict__ x, const float* __restrict__ g,
                            const float* __restrict__ b, Dst y, long m, int c) {
    long row = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (row >= m) return;
    const float* xr = x + row * c;
    float v[MAXV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        int ch = i * 32 + lane;
        v[i] = ch < c ? xr[ch] : 0.f;
        s += v[i];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    float mean = s / (float)c;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        int ch = i * 32 + lane;
        float d = ch < c ? v[i] - mean : 0.f;
        q += d * d;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    float rstd = 1.f / sqrtf(q / (float)c + 1e-5f);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        int ch = i * 32 + lane;
        if (ch < c) put(y, row * c + ch, (v[i] - mean) * rstd * g[ch] + b[ch]);
    }
}


// Half a warp per token: lanes 0-15 one token, 16-31 the next; lane l holds channels
// l, l+16, ... (MAXV of them), so each load instruction covers 64 bytes of each token.
template <int MAXV>
__global__ void k_layernorm16(const float* __restrict__ x, const float* __restrict__ g,
                              const float* __restrict__ b, Dst y, long m, int c) {
    const int lane = threadIdx.x & 31, hl = lane & 15;
    const long row = ((long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * 2 + (lane >> 4);
    const bool live = row < m;
    const float* xr = x + (live ? row : 0) * c;
    float v[MAXV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int ch = i * 16 + hl;
        v[i] = live && ch < c ? xr[ch] : 0.f;
        s += v[i];
    }
#pragma unroll
    for (int o = 8; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)c;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int ch = i * 16 + hl;
        const float d = ch < c ? v[i] - mean : 0.f;
        q += d * d;
    }
#pragma unroll
    for (int o = 8; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = 1.f / sqrtf(q / (float)c + 1e-5f);
    if (!live) return;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int ch = i * 16 + hl;
        if (ch < c) put(y, row * c + ch, (v[i] - mean) * rstd * g[ch] + b[ch]);
    }
}

// The fp16-pair LayerNorm by bulk copies: a persistent CTA moves tiles of LN_TOK tokens with
// one asynchronous bulk load each (double-buffered, completion on an mbarrier), normalises
// them from shared memory with half a warp per token, and writes the tile's hi and lo rows
// with two bulk stores. Few instructions and many bytes in flight per SM. c a multiple of 8
// and at most 144 (9 channels a lane). Waits are bounded; on expiry error 30 is recorded and
// the CTA stops.
constexpr int LN_TOK = 32;
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__global__ void __launch_bounds__(256) k_layernorm_bulk(const float* __restrict__ x, const float* __restrict__ g,
                                                        const float* __restrict__ b, Dst y, long m, int c,
                                                        int* err) {
    extern __shared__ __align__(128) uint8_t lsm[];
    __shared__ __align__(8) uint64_t full[2];
    float* in0 = reinterpret_cast<float*>(lsm);
    const int tile_f = LN_TOK * c;  // floats of one input tile
    __half* oh = reinterpret_cast<__half*>(lsm + 2 * tile_f * 4);
    __half* ol = oh + tile_f;
    const int lane = threadIdx.x & 31, hl = lane & 15, slot = threadIdx.x >> 4;  // 16 tokens a round
    const long ntiles = (m + LN_TOK - 1) / LN_TOK;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&full[i])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    auto issue = [&](long t, int buf) {
        const long rows = min((long)LN_TOK, m - t * LN_TOK);
        const uint32_t bytes = (uint32_t)(rows * c * 4);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&full[buf])),
                     "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(smem_addr(in0 + buf * tile_f)), "l"(x + t * LN_TOK * c), "r"(bytes),
                     "r"(smem_addr(&full[buf]))
                     : "memory");
    };
    float gg[9], bb[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) {
        const int ch = hl + 16 * k;
        gg[k] = ch < c ? g[ch] : 0.f;
        bb[k] = ch < c ? b[ch] : 0.f;
    }
    if (threadIdx.x == 0 && (long)blockIdx.x < ntiles) issue(blockIdx.x, 0);
    bool big = false;
    uint32_t i = 0;
    for (long t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (threadIdx.x == 0 && t + gridDim.x < ntiles) issue(t + gridDim.x, buf ^ 1);
        // this tile's rows have landed
        {
            uint32_t ok = 0;
            const long long t0 = clock64();
            while (!ok) {
                asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                             " selp.u32 %0, 1, 0, p;\n}\n"
                             : "=r"(ok) : "r"(smem_addr(&full[buf])), "r"((i >> 1) & 1) : "memory");
                if (!ok && clock64() - t0 > 4000000000ll) break;
            }
            if (!__syncthreads_and(ok)) {
                if (threadIdx.x == 0) {
                    atomicCAS(err, 0, 30);
                    // let the loads in flight (this tile's and the next one's) land first
                    for (int k = 0; k < 2; ++k) {
                        const int bf = buf ^ k;
                        const uint32_t par = ((i + k) >> 1) & 1;
                        uint32_t done = 0;
                        const long long t1 = clock64();
                        while (!done && clock64() - t1 < 4000000000ll)
                            asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                                         " selp.u32 %0, 1, 0, p;\n}\n"
                                         : "=r"(done) : "r"(smem_addr(&full[bf])), "r"(par) : "memory");
                    }
                }
                break;
            }
        }
        // the previous tile's stores have read the output rows
        if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncthreads();
        const long rows = min((long)LN_TOK, m - t * LN_TOK);
        const float* tin = in0 + buf * tile_f;
#pragma unroll 1
        for (int r = 0; r < LN_TOK; r += 16) {
            const int tok = r + slot;
            const bool live = tok < rows;
            float v[9];
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                const int ch = hl + 16 * k;
                v[k] = live && ch < c ? tin[tok * c + ch] : 0.f;
                s += v[k];
            }
#pragma unroll
            for (int o = 8; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            const float mean = s / (float)c;
            float q = 0.f;
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                const int ch = hl + 16 * k;
                const float d = ch < c ? v[k] - mean : 0.f;
                q += d * d;
            }
#pragma unroll
            for (int o = 8; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
            const float rstd = 1.f / sqrtf(q / (float)c + 1e-5f);
            if (live) {
#pragma unroll
                for (int k = 0; k < 9; ++k) {
                    const int ch = hl + 16 * k;
                    if (ch < c) {
                        const float o = (v[k] - mean) * rstd * gg[k] + bb[k];
                        __half h, l;
                        split_h16(o, h, l);
                        oh[tok * c + ch] = h;
                        ol[tok * c + ch] = l;
                        big |= beyond_h16(o);
                    }
                }
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (threadIdx.x == 0) {
            const uint32_t bytes = (uint32_t)(rows * c * 2);
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                         ::"l"(reinterpret_cast<__half*>(y.hi) + t * LN_TOK * c), "r"(smem_addr(oh)), "r"(bytes)
                         : "memory");
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                         ::"l"(reinterpret_cast<__half*>(y.lo) + t * LN_TOK * c), "r"(smem_addr(ol)), "r"(bytes)
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
    }
    if (big && y.err) atomicCAS(y.err, 0, ERR_RANGE_GEMM);
    if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

void launch_layernorm(const float* x, const float* g, const float* b, Dst y, long m, int c, cudaStream_t st) {
    if (c > 256) throw Error(1, "layernorm: c > 256 is not supported");
    int* err = y.err;  // the engine's device error word (timeouts, fp16 range)
    if (y.lo && y.h16 && err && c % 8 == 0 && c <= 144 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(y.hi) & 15) == 0 && (reinterpret_cast<uintptr_t>(y.lo) & 15) == 0) {
        const size_t smem = (size_t)LN_TOK * c * (2 * 4 + 2 * 2);
        int dev = 0, sms = 0;
        HAT_CUDA(cudaGetDevice(&dev));
        HAT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        allow_dyn_smem(k_layernorm_bulk, smem);
        const long ntiles = (m + LN_TOK - 1) / LN_TOK;
        const long grid = std::min<long>(ntiles, 4L * sms);  // four 55 KB CTAs per SM
        k_layernorm_bulk<<<(unsigned)grid, 256, smem, st>>>(x, g, b, y, m, c, err);
        HAT_CUDA(cudaGetLastError());
        count_launch();
        return;
    }
    if (c <= 144) {
        k_layernorm16<9><<<(unsigned)((m + 15) / 16), 256, 0, st>>>(x, g, b, y, m, c);
        HAT_CUDA(cudaGetLastError());
        count_launch();
        return;
    }
    unsigned grid = (unsigned)((m + 7) / 8);
    if (c <= 160)
        k_layernorm<5><<<grid, 256, 0, st>>>(x, g, b, y, m, c);
    else
        k_layernorm<8><<<grid, 256, 0, st>>>(x, g, b, y, m, c);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

// ---------------------------------------------------------------- split
__global__ void k_split(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo, long n) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        float h, l;
        split_tf32(x[i], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

void launch_split(const float* x, float* hi, float* lo, long n, cudaStream_t st) {
    k_split<<<1184, 256, 0, st>>>(x, hi, lo, n);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

// ---------------------------------------------------------------- channel attention
// ChannelAttention after the pool (hat_arch.py:40-57): `sums` holds the per-channel
// sums of the CAB's second conv over the plane; one CTA computes the gate.
__global__ void k_ca_gate(const float* __restrict__ partial, long rows, float inv_count,
                          const float* __restrict__ w1, const float* __restrict__ b1, const float* __restrict__ w2,
                          const float* __restrict__ b2, float* __restrict__ gate, int c, int sq, const CabFold f) {
    // c <= 256: lanes cover channels (coalesced rows), warps stride the partial rows, and
    // the per-warp sums are combined in warp order, so the result is identical every run.
    __shared__ float red[32][257];
    __shared__ float mean[256], hid[64];
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll 4
    for (long r = warp; r < rows; r += 32) {  // four rows' loads in flight a warp
        const float* row = partial + r * c;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (lane + 32 * j < c) acc[j] += row[lane + 32 * j];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (lane + 32 * j < c) red[warp][lane + 32 * j] = acc[j];
    __syncthreads();
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
        float a = 0.f;
        for (int w = 0; w < 32; ++w) a += red[w][i];
        mean[i] = a * inv_count;
    }
    __syncthreads();
    for (int j = warp; j < sq; j += 32) {
        float a = 0.f;
        for (int i = lane; i < c; i += 32) a += w1[(long)j * c + i] * mean[i];
#pragma unroll
        for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) hid[j] = fmaxf(a + b1[j], 0.f);
    }
    __syncthreads();
    __shared__ float gs[256];
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
        float a = b2[i];
        for (int j = 0; j < sq; ++j) a += w2[(long)i * sq + j] * hid[j];
        gs[i] = 1.f / (1.f + expf(-a));
        gate[i] = gs[i];
    }
    if (!f.hi) return;
    __syncthreads();
    // The gate folded into the CAB conv's weight rows and proj's bias (k_proj_cab):
    // W'[n][tap * cinp + ci] = conv_scale * gate[n] * w[n][ci][tap], times proj's factor.
    for (int i = threadIdx.x; i < c; i += blockDim.x) f.bias[i] = f.bp[i] + f.cs * gs[i] * f.b2[i];
    const int per = f.cc * 9;
    bool big = false;
    for (int i = threadIdx.x; i < c * per; i += blockDim.x) {
        const int n = i / per, r = i - n * per, ci = r / 9, tap = r - ci * 9;
        const float v = f.cs * gs[n] * f.w[i] * f.factor;  // w: [c][cc][3][3]
        const long o = (long)n * f.k_pad + tap * f.cinp + ci;
        if (f.h16) {
            __half h, l;
            split_h16(v, h, l);
            reinterpret_cast<__half*>(f.hi)[o] = h;
            reinterpret_cast<__half*>(f.lo)[o] = l;
            big |= beyond_h16(v);
        } else {
            float h, l;
            split_tf32(v, h, l);
            f.hi[o] = h;
            f.lo[o] = l;
        }
    }
    if (big && f.err) atomicCAS(f.err, 0, ERR_RANGE_GEMM);
}

// ---------------------------------------------------------------- CAB pool, analytically
// The channel-attention pool needs the sum over the output pixels of the CAB's second conv
// (src/gpu.rs:435; hat_arch.py:40-57). As that conv is folded into proj (k_proj_cab), its
// output is never written; the sum is taken from its input instead:
//   sum_p conv(x)[p][n] = P * b[n] + sum_{tap, ci} w[n][ci][tap] * T[tap][ci],
//   T[tap][ci] = sum over the output pixels p of x[p + tap offset][ci] (zero outside),
// and T follows from per-row sums of x and its first and last columns: a tap shifted by
// dy sums the rows [y0 + dy, y1 + dy) of the view, one shifted by dx = -1 (+1) leaves out
// the last (first) column.

// One CTA per view row r in [r_lo, r_hi): stat[r - r_lo] = {row sum, first, last}[cc].
// The row is read as 16-byte vectors (8 fp16 or 4 fp32 channels of one pixel); thread t
// takes the vectors t, t + nt, ..., all of one channel group since nt is a multiple of the
// vectors per pixel, and the threads of a group are added in thread order.
template <int VEC>
__global__ void k_cab_rowstat(Opnd x, int ld, int cc, int wid, int r_lo, float* __restrict__ stat) {
    __shared__ float part[256][VEC + 1];
    const int vp = ld / VEC, nt = blockDim.x / vp * vp, t = threadIdx.x;
    const long row = (long)(r_lo + blockIdx.x) * wid * ld;
    const long nv = (long)wid * vp;
    float a[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) a[j] = 0.f;
    if (t < nt) {
        if (VEC == 8) {
            const uint4* hv = reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(x.hi) + row);
            const uint4* lv = reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(x.lo) + row);
#pragma unroll 4
            for (long v = t; v < nv; v += nt) {
                const uint4 h = hv[v], l = lv[v];
                const __half2* h2 = reinterpret_cast<const __half2*>(&h);
                const __half2* l2 = reinterpret_cast<const __half2*>(&l);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 fh = __half22float2(h2[j]), fl = __half22float2(l2[j]);
                    a[2 * j] += fh.x + fl.x;
                    a[2 * j + 1] += fh.y + fl.y;
                }
            }
        } else {
            const float4* hv = reinterpret_cast<const float4*>(x.hi + row);
            const float4* lv = x.lo ? reinterpret_cast<const float4*>(x.lo + row) : nullptr;
#pragma unroll 4
            for (long v = t; v < nv; v += nt) {
                float4 h = hv[v];
                if (lv) {
                    const float4 l = lv[v];
                    h.x += l.x;
                    h.y += l.y;
                    h.z += l.z;
                    h.w += l.w;
                }
                a[0] += h.x;
                a[1] += h.y;
                a[2] += h.z;
                a[3] += h.w;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) part[t][j] = a[j];
    __syncthreads();
    auto val = [&](long e) {
        if (x.lo && x.h16)
            return __half2float(reinterpret_cast<const __half*>(x.hi)[e]) +
                   __half2float(reinterpret_cast<const __half*>(x.lo)[e]);
        return x.lo ? x.hi[e] + x.lo[e] : x.hi[e];
    };
    float* o = stat + (long)blockIdx.x * 3 * cc;
    for (int ci = t; ci < cc; ci += blockDim.x) {
        const int grp = ci / VEC, j = ci % VEC;
        float s = 0.f;
        for (int u = grp; u < nt; u += vp) s += part[u][j];
        o[ci] = s;
        o[cc + ci] = val(row + ci);
        o[2 * cc + ci] = val(row + (long)(wid - 1) * ld + ci);
    }
}

// sum[n] for the output rows [y0, y1) of a view of `vrows` rows; `stat` holds the rows
// [r_lo, r_hi) = [y0 - 1, y1 + 1) clipped to the view. The rows [y0, y1) are summed in
// parallel (per value, PARTS interleaved partial sums added in order); a tap shifted by dy
// = -1 / +1 then swaps the range's last / first row for the one beyond it.
__global__ void k_cab_pool(const float* __restrict__ stat, int r_lo, int r_hi, int y0, int y1, int cc, int wid,
                           const float* __restrict__ w, const float* __restrict__ b, int c, float* __restrict__ sum) {
    __shared__ float part[1024];
    __shared__ float S[3 * 64], T[9 * 64];
    const int nvals = 3 * cc, parts = blockDim.x / nvals;
    const int t = threadIdx.x, j = t % nvals, pp = t / nvals;
    if (pp < parts) {
        float a = 0.f;
        for (int r = y0 + pp; r < y1; r += parts) a += stat[(long)(r - r_lo) * nvals + j];
        part[t] = a;
    }
    __syncthreads();
    if (t < nvals) {
        float a = 0.f;
        for (int u = 0; u < parts; ++u) a += part[u * nvals + t];
        S[t] = a;
    }
    __syncthreads();
    auto row = [&](int r, int k) { return r >= r_lo && r < r_hi ? stat[(long)(r - r_lo) * nvals + k] : 0.f; };
    for (int i = t; i < 9 * cc; i += blockDim.x) {
        const int tap = i / cc, ci = i - tap * cc, dy = tap / 3 - 1, dx = tap % 3 - 1;
        float v[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {  // row sum, first column, last column over rows [y0 + dy, y1 + dy)
            const int q = k * cc + ci;
            v[k] = S[q];
            if (dy < 0) v[k] = (v[k] - row(y1 - 1, q)) + row(y0 - 1, q);
            if (dy > 0) v[k] = (v[k] - row(y0, q)) + row(y1, q);
        }
        T[i] = v[0] - (dx < 0 ? v[2] : 0.f) - (dx > 0 ? v[1] : 0.f);
    }
    __syncthreads();
    // One warp per output channel: the lanes take the channel's 9 * cc weights in turn
    // (coalesced) and a fixed shuffle tree adds them.
    const float pix = (float)((long)(y1 - y0) * wid);
    const int warp = t >> 5, lane = t & 31, nw = blockDim.x >> 5, K = 9 * cc;
    for (int n = warp; n < c; n += nw) {
        const float* wn = w + (long)n * K;  // [ci][tap]
        float a = 0.f;
        for (int i = lane; i < K; i += 32) {
            const int ci = i / 9, tap = i - ci * 9;
            a += wn[i] * T[tap * cc + ci];
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) sum[n] = pix * b[n] + a;
    }
}

void launch_cab_pool(Opnd x, int ld, int cc, int wid, int vrows, int y0, int y1, float* stat, const float* w,
                     const float* b, int c, float* sum, cudaStream_t st) {
    if (cc > 64) throw Error(1, "cab pool: at most 64 compressed channels");
    const int r_lo = max(0, y0 - 1), r_hi = min(vrows, y1 + 1);
    if (r_hi <= r_lo) throw Error(1, "cab pool: empty row range");
    const bool h16 = x.lo && x.h16;
    const int vec = h16 ? 8 : 4;
    if (ld % vec || ld / vec > 256 || (reinterpret_cast<uintptr_t>(x.hi) & 15) ||
        (x.lo && (reinterpret_cast<uintptr_t>(x.lo) & 15)))
        throw Error(1, "cab pool: the plane's rows must be whole 16-byte vectors");
    if (h16)
        k_cab_rowstat<8><<<(unsigned)(r_hi - r_lo), 256, 0, st>>>(x, ld, cc, wid, r_lo, stat);
    else
        k_cab_rowstat<4><<<(unsigned)(r_hi - r_lo), 256, 0, st>>>(x, ld, cc, wid, r_lo, stat);
    HAT_CUDA(cudaGetLastError());
    count_launch();
    k_cab_pool<<<1, 1024, 0, st>>>(stat, r_lo, r_hi, y0, y1, cc, wid, w, b, c, sum);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

void launch_ca_gate(const float* partial, long rows, float inv_count, const float* w1, const float* b1,
                    const float* w2, const float* b2, float* gate, int c, int sq, cudaStream_t st,
                    const CabFold& fold) {
    if (c > 256 || sq > 64) throw Error(1, "channel attention: c > 256 or squeeze > 64 is not supported");
    k_ca_gate<<<1, 1024, 0, st>>>(partial, rows, inv_count, w1, b1, w2, b2, gate, c, sq, fold);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

}  // namespace hat
