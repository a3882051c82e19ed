// Tensor-core window attention for sm_100a: the HAB's (shifted) 16x16 window attention
// and the OCAB's 16x16-query / 24x24-key overlapping attention (hat_arch.py:165-196,
// 392-438), one fused kernel per launch:
//
//   S = (q*scale) K^T + bias (+ shift mask)      tcgen05.mma, S in tensor memory
//   P = exp(S - running max), row sums            CUDA cores, one thread per query row
//   O += P V                                      tcgen05.mma, O block in tensor memory
//
// Work item = (window, head, half of the window's 256 queries); 128 query rows per
// item, keys streamed in blocks of 32 (8 blocks for 256 keys, 18 for 576). Every
// operand is split into tf32 hi/lo halves on the way into shared memory, and both
// products use the 3-term split (A_lo.B_hi + A_hi.B_lo + A_hi.B_hi) in fp32-parity
// mode; fast mode issues the single A_hi.B_hi. The softmax is the online form: each
// block's P uses the running row max, and O (kept in registers, fp32) is rescaled when
// the max grows, so S never needs more than one block of tensor memory.
//
// The window partition, the cyclic roll, the nn.Unfold of the keys with its zero
// padding, the relative-position bias gather and the shift mask are address
// arithmetic: nothing is materialised.
//
// Warp roles (288 threads): 0 MMA issuer + TMEM owner, 1-4 softmax (TMEM lane quarters
// 1,2,3,0), 5-8 loaders (gather, scale, split, swizzled stores). Every mbarrier wait is
// bounded; on expiry the kernel records an error code, all roles leave, and TMEM is
// released.
#include "common.cuh"

namespace hat {

namespace {

constexpr int TC_THREADS = 288;
constexpr int KBLK = 32;     // keys per block
constexpr int MT = 128;      // query rows per work item
constexpr int KVS = 4;       // K/V pipeline stages
constexpr long long WAIT_CYCLES_A = 4000000000ll;

__device__ __forceinline__ uint32_t su(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void bar_init(uint64_t* b, int n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su(b)), "r"(n));
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t par) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(su(b)), "r"(par)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t par, volatile int* abort, int* err, int code) {
    if (bar_try(b, par)) return true;
    const long long t0 = clock64();
    while (true) {
        if (bar_try(b, par)) return true;
        if (*abort) return false;
        if (clock64() - t0 > WAIT_CYCLES_A) {
            *abort = 1;
            atomicCAS(err, 0, code);
            return false;
        }
    }
}
__device__ __forceinline__ void bar_wait_quiet(uint64_t* b, uint32_t par) {
    const long long t0 = clock64();
    while (!bar_try(b, par))
        if (clock64() - t0 > WAIT_CYCLES_A) return;
}
__device__ __forceinline__ void fence_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tcf_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tcf_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (sm_100 version field), `rowbytes`-wide swizzle atoms
// (128: SWIZZLE_128B, 32: SWIZZLE_32B), core groups of 8 rows `sbo` bytes apart.
__device__ __forceinline__ uint64_t mdesc(uint32_t saddr, int rowbytes, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(sbo >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)(rowbytes == 128 ? 2 : 6) << 61;
    return d;
}
// kind::tf32, f32 accumulate, M = 128, both operands K-major (bmn = 0).
__host__ __device__ constexpr uint32_t idesc_a(int n, int bmn) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)bmn << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su(b))
                 : "memory");
}
__device__ __forceinline__ void tld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of element (row, c), c < 8, in a K-major SWIZZLE_32B tile of 32-byte rows.
__device__ __forceinline__ uint32_t off_sw32(int row, int c) {
    return row * 32 + ((((c >> 2) ^ (row >> 2)) & 1) << 4) + (c & 3) * 4;
}
// Byte offset of element (row, c), c < 32, in a SWIZZLE_128B tile of 128-byte rows.
__device__ __forceinline__ uint32_t off_sw128(int row, int c) {
    return row * 128 + ((((c >> 2) ^ row) & 7) << 4) + (c & 3) * 4;
}

__device__ __forceinline__ int band3(int v, int n, int shift) { return v < n - 16 ? 0 : (v < n - shift ? 1 : 2); }

}  // namespace

// D: head dim (24 or 30); OCA: overlapping attention; TERMS: 3 (parity) or 1 (fast).
template <int D, bool OCA, int TERMS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_attn_tc(const float* __restrict__ qkv, const float* __restrict__ table, Dst out, int hp, int wp, int c,
              int heads, int shift, float scale, long items, int* err) {
    constexpr int KS = (D + 7) / 8;                 // k-steps of the QK^T product
    constexpr int NK = OCA ? 576 : 256;             // keys per window
    constexpr int NBLK = NK / KBLK;
    constexpr int TROWS = OCA ? 39 * 39 : 31 * 31;
    constexpr uint32_t Q_BYTES = KS * 4096;         // 128 rows x 32 B per k-step
    constexpr uint32_t K_BYTES = KS * 1024;         // 32 rows x 32 B per k-step
    constexpr uint32_t V_BYTES = 4096;              // V^T: 32 features x 128 B (32 keys)
    constexpr uint32_t KV_BYTES = 2 * K_BYTES + 2 * V_BYTES;
    constexpr uint32_t P_BYTES = 16384;             // 128 rows x 128 B
    constexpr uint32_t OFF_KV = 2 * Q_BYTES;
    constexpr uint32_t OFF_P = OFF_KV + KVS * KV_BYTES;
    constexpr uint32_t OFF_TAB = OFF_P + 2 * 2 * P_BYTES;
    constexpr uint32_t OFF_KOFF = OFF_TAB + ((TROWS * 4 + 15) / 16) * 16;

    extern __shared__ __align__(1024) uint8_t raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
    float* tab = reinterpret_cast<float*>(sm + OFF_TAB);
    int* koff = reinterpret_cast<int*>(sm + OFF_KOFF);  // OCAB: key (ky, kx) -> ky*39 + kx
    __shared__ uint64_t q_full, q_empty, kv_full[KVS], kv_empty[KVS], s_full[2], p_full[2], o_full[2], o_free[2], drain;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = (int)(blockIdx.x % heads);
    const int nx = wp / 16;
    const long c3 = 3L * c;

    for (int i = threadIdx.x; i < TROWS; i += TC_THREADS) tab[i] = table[(long)i * heads + head];
    if (OCA)
        for (int i = threadIdx.x; i < NK; i += TC_THREADS) koff[i] = (i / 24) * 39 + (i % 24);
    if (threadIdx.x == 0) {
        bar_init(&q_full, 128);
        bar_init(&q_empty, 1);
        for (int s = 0; s < KVS; ++s) {
            bar_init(&kv_full[s], 128);
            bar_init(&kv_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            bar_init(&s_full[s], 1);
            bar_init(&p_full[s], 128);
            bar_init(&o_full[s], 1);
            bar_init(&o_free[s], 128);
        }
        bar_init(&drain, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(su(&tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tcf_before();
    __syncthreads();
    tcf_after();
    const uint32_t tmem = tmem_slot;  // S buffers at columns 0 and 32, O blocks at 64 and 96

    if (warp == 0) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_s = idesc_a(32, 0), id_o = idesc_a(32, 0);
            const uint32_t qh = su(sm), ql = su(sm + Q_BYTES);
            long g = 0;  // global key-block counter
            uint32_t ti = 0;
            bool ok = true;
            for (long w = blockIdx.x; w < items && ok; w += gridDim.x, ++ti) {
                if (!bar_wait(&q_full, ti & 1, &abort_flag, err, 11)) break;
                auto issue_s = [&](long gb) -> bool {
                    const int s = (int)(gb & 1), kvs = (int)(gb % KVS);
                    if (!bar_wait(&kv_full[kvs], (uint32_t)((gb / KVS) & 1), &abort_flag, err, 12)) return false;
                    tcf_after();
                    const uint32_t kb = su(sm + OFF_KV + kvs * KV_BYTES);
                    const uint32_t d = tmem + s * 32;
#pragma unroll
                    for (int k = 0; k < KS; ++k) {
                        const uint64_t aH = mdesc(qh + k * 4096, 32, 256), aL = mdesc(ql + k * 4096, 32, 256);
                        const uint64_t bH = mdesc(kb + k * 1024, 32, 256), bL = mdesc(kb + K_BYTES + k * 1024, 32, 256);
                        if (TERMS == 3) {
                            mma(d, aL, bH, id_s, k ? 1u : 0u);
                            mma(d, aH, bL, id_s, 1u);
                            mma(d, aH, bH, id_s, 1u);
                        } else {
                            mma(d, aH, bH, id_s, k ? 1u : 0u);
                        }
                    }
                    commit(&s_full[s]);
                    return true;
                };
                if (!issue_s(g)) break;
                for (int j = 0; j < NBLK; ++j) {
                    const long gb = g + j;
                    if (j + 1 < NBLK) {
                        if (!issue_s(gb + 1)) {
                            ok = false;
                            break;
                        }
                        // Once the item's last S MMA is issued, Q may be replaced.
                        if (j + 1 == NBLK - 1) commit(&q_empty);
                    }
                    const int s = (int)(gb & 1);
                    const uint32_t ph = (uint32_t)((gb >> 1) & 1);
                    if (!bar_wait(&p_full[s], ph, &abort_flag, err, 13) ||
                        !bar_wait(&o_free[s], ph ^ 1, &abort_flag, err, 14)) {
                        ok = false;
                        break;
                    }
                    tcf_after();
                    const uint32_t pb = su(sm + OFF_P + s * 2 * P_BYTES);
                    const int kvs = (int)(gb % KVS);
                    const uint32_t vb = su(sm + OFF_KV + kvs * KV_BYTES + 2 * K_BYTES);
                    const uint32_t d = tmem + 64 + s * 32;
#pragma unroll
                    for (int k = 0; k < KBLK / 8; ++k) {
                        const uint64_t aH = mdesc(pb + k * 32, 128, 1024), aL = mdesc(pb + P_BYTES + k * 32, 128, 1024);
                        const uint64_t bH = mdesc(vb + k * 32, 128, 1024), bL = mdesc(vb + V_BYTES + k * 32, 128, 1024);
                        if (TERMS == 3) {
                            mma(d, aL, bH, id_o, k ? 1u : 0u);
                            mma(d, aH, bL, id_o, 1u);
                            mma(d, aH, bH, id_o, 1u);
                        } else {
                            mma(d, aH, bH, id_o, k ? 1u : 0u);
                        }
                    }
                    commit(&o_full[s]);
                    commit(&kv_empty[kvs]);
                }
                g += NBLK;
            }
            commit(&drain);
            bar_wait_quiet(&drain, 0);
        }
    } else if (warp <= 4) {
        // ------------------------------------------------------------ softmax
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;
        const uint32_t trow = (uint32_t)(q4 * 32) << 16;
        constexpr float L2E = 1.4426950408889634f;
        long g = 0;
        for (long w = blockIdx.x; w < items; w += gridDim.x) {
            if (__any_sync(0xffffffffu, abort_flag != 0)) break;
            const long rest = w / heads;
            const int win = (int)(rest >> 1), mtile = (int)(rest & 1);
            const int wy = win / nx, wx = win - wy * nx;
            const int qi = mtile * MT + row, qy = qi >> 4, qx = qi & 15;
            const bool masked = !OCA && shift > 0;
            // Bias row of this query: SA index (qy-ky+15)*31 + (qx-kx+15) = A0 - (ky*31+kx);
            // OCAB index (ky*39+kx) - B0, wrapped into the table.
            const int A0 = qy * 31 + qx + 480, B0 = qy * 39 + qx + 280;
            // Shift mask: key column kx is masked against target label t when
            // band(wx*16+kx) != t; one 16-bit mask per possible row band.
            uint32_t cm[3] = {0, 0, 0};
            int lq = 0;
            if (masked) {
                lq = band3(wy * 16 + qy, hp, shift) * 3 + band3(wx * 16 + qx, wp, shift);
#pragma unroll
                for (int kx = 0; kx < 16; ++kx) {
                    const int bx = band3(wx * 16 + kx, wp, shift);
#pragma unroll
                    for (int by = 0; by < 3; ++by)
                        if (by * 3 + bx != lq) cm[by] |= 1u << kx;
                }
            }
            float m = -INFINITY, l = 0.f, a_prev = 1.f;
            float o[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0.f;
            bool ok = true;
            auto o_update = [&](long gb, float a) -> bool {
                const int s = (int)(gb & 1);
                const bool got = bar_wait(&o_full[s], (uint32_t)((gb >> 1) & 1), &abort_flag, err, 15);
                if (!__all_sync(0xffffffffu, got)) return false;
                tcf_after();
                float ob[32];
                tld16(tmem + trow + 64 + s * 32, ob);
                tld16(tmem + trow + 64 + s * 32 + 16, ob + 16);
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] = o[i] * a + ob[i];
                tcf_before();
                bar_arrive(&o_free[s]);
                return true;
            };
            for (int j = 0; j < NBLK; ++j) {
                const long gb = g + j;
                const int s = (int)(gb & 1);
                const bool got = bar_wait(&s_full[s], (uint32_t)((gb >> 1) & 1), &abort_flag, err, 16);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                tcf_after();
                float sv[32];
                tld16(tmem + trow + s * 32, sv);
                tld16(tmem + trow + s * 32 + 16, sv + 16);
                uint32_t mrow0 = 0, mrow1 = 0;
                if (masked) {
                    // the block's two key rows ky = 2j, 2j+1
                    mrow0 = cm[band3(wy * 16 + 2 * j, hp, shift)];
                    mrow1 = cm[band3(wy * 16 + 2 * j + 1, hp, shift)];
                }
                const float* trow_sa = tab + (A0 - 62 * j);  // SA: minus (k>>4)*31 + (k&15)
                float bmax = -INFINITY;
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    float v;
                    if (OCA) {
                        int bi = koff[j * KBLK + k] - B0;
                        bi += bi < 0 ? TROWS : 0;
                        v = sv[k] + tab[bi];
                    } else {
                        v = sv[k] + trow_sa[-((k >> 4) * 31 + (k & 15))];
                        if (masked) {
                            const uint32_t mr = (k >> 4) ? mrow1 : mrow0;
                            if ((mr >> (k & 15)) & 1u) v += -100.f;
                        }
                    }
                    sv[k] = v;
                    bmax = fmaxf(bmax, v);
                }
                const float mn = fmaxf(m, bmax);
                const float a = exp2f((m - mn) * L2E);
                const float nmn = -mn * L2E;
                float psum = 0.f;
                uint8_t* pb = sm + OFF_P + s * 2 * P_BYTES;
#pragma unroll
                for (int k4 = 0; k4 < 8; ++k4) {
                    float p[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        p[u] = exp2f(fmaf(sv[4 * k4 + u], L2E, nmn));
                        psum += p[u];
                    }
                    float4 ph, pl;
                    split_tf32(p[0], ph.x, pl.x);
                    split_tf32(p[1], ph.y, pl.y);
                    split_tf32(p[2], ph.z, pl.z);
                    split_tf32(p[3], ph.w, pl.w);
                    const uint32_t off = off_sw128(row, 4 * k4);
                    *reinterpret_cast<float4*>(pb + off) = ph;
                    if (TERMS == 3) *reinterpret_cast<float4*>(pb + P_BYTES + off) = pl;
                }
                l = l * a + psum;
                m = mn;
                fence_async();
                tcf_before();
                bar_arrive(&p_full[s]);
                if (j > 0 && !o_update(gb - 1, a_prev)) {
                    ok = false;
                    break;
                }
                a_prev = a;
            }
            if (!ok || !o_update(g + NBLK - 1, a_prev)) break;
            // O / l at the query's plane position (the roll of the shifted windows undone).
            const float inv = 1.f / l;
            long qpos;
            if (OCA)
                qpos = (long)(wy * 16 + qy) * wp + wx * 16 + qx;
            else
                qpos = (long)((wy * 16 + qy + shift) % hp) * wp + (wx * 16 + qx + shift) % wp;
            const long ob = qpos * c + (long)head * D;
#pragma unroll
            for (int i = 0; i < D; ++i) put(out, ob + i, o[i] * inv);
            g += NBLK;
        }
    } else {
        // ------------------------------------------------------------ loaders
        // Warps 5-6 load K: lane = key, warp = column half [0,16) / [16,32); each 4-column
        // chunk is one 16-byte store into the K-major SW32 tiles. Warps 7-8 load V: a
        // thread owns a 4-key x 4-feature block, transposes it in registers and writes
        // four 16-byte rows of V^T (K-major SW128: one row of 32 keys per feature). Loads
        // for the next key block are issued before waiting for a free stage.
        constexpr int VW = (D % 4 == 0) ? 4 : 2;  // vector width that keeps the row alignment
        const int t = threadIdx.x - 160;           // 0..127
        const int lw = warp - 5;                   // 0..3
        const bool is_v = lw >= 2;
        const int kk0 = is_v ? (((lw - 2) * 32 + lane) & 7) * 4 : lane;  // first key of this thread
        const int col0 = is_v ? (((lw - 2) * 32 + lane) >> 3) * 4 : lw * 16;
        long g = 0;
        uint32_t ti = 0;
        float buf[16];
        auto key_pos = [&](int wy, int wx, int kk, bool& inside) -> long {
            inside = true;
            if (OCA) {
                const int ky = kk / 24, kx = kk - ky * 24;
                const int Y = wy * 16 - 4 + ky, X = wx * 16 - 4 + kx;
                inside = Y >= 0 && Y < hp && X >= 0 && X < wp;
                return inside ? (long)Y * wp + X : 0;
            }
            const int ky = kk >> 4, kx = kk & 15;
            return (long)((wy * 16 + ky + shift) % hp) * wp + (wx * 16 + kx + shift) % wp;
        };
        // n floats of row `src` from column `cc` (zeros past D or outside the plane)
        auto load_cols = [&](const float* src, int cc, bool inside, float* dst, int n) {
#pragma unroll
            for (int u = 0; u < 16; u += VW) {
                if (u >= n) break;
                const int col = cc + u;
                if (inside && col + VW <= D) {
                    if (VW == 4) {
                        const float4 v = *reinterpret_cast<const float4*>(src + col);
                        dst[u] = v.x;
                        dst[u + 1] = v.y;
                        dst[u + 2] = v.z;
                        dst[u + 3] = v.w;
                    } else {
                        const float2 v = *reinterpret_cast<const float2*>(src + col);
                        dst[u] = v.x;
                        dst[u + 1] = v.y;
                    }
                } else {
#pragma unroll
                    for (int e2 = 0; e2 < VW; ++e2) dst[u + e2] = (inside && col + e2 < D) ? src[col + e2] : 0.f;
                }
            }
        };
        auto fetch = [&](int wy, int wx, int j) {
            if (!is_v) {
                bool inside;
                const long kpos = key_pos(wy, wx, j * KBLK + kk0, inside);
                load_cols(qkv + kpos * c3 + c + (long)head * D, col0, inside, buf, 16);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    bool inside;
                    const long kpos = key_pos(wy, wx, j * KBLK + kk0 + i, inside);
                    load_cols(qkv + kpos * c3 + 2 * c + (long)head * D, col0, inside, buf + 4 * i, 4);
                }
            }
        };
        for (long w = blockIdx.x; w < items; w += gridDim.x, ++ti) {
            if (__any_sync(0xffffffffu, abort_flag != 0)) break;
            const long rest = w / heads;
            const int win = (int)(rest >> 1), mtile = (int)(rest & 1);
            const int wy = win / nx, wx = win - wy * nx;
            fetch(wy, wx, 0);
            // Q: thread t loads query row t of the item, scaled, split into the SW32 tiles.
            {
                const int qi = mtile * MT + t, qy = qi >> 4, qx = qi & 15;
                long qpos;
                if (OCA)
                    qpos = (long)(wy * 16 + qy) * wp + wx * 16 + qx;
                else
                    qpos = (long)((wy * 16 + qy + shift) % hp) * wp + (wx * 16 + qx + shift) % wp;
                const float* src = qkv + qpos * c3 + (long)head * D;
                float qv[KS * 8];
                load_cols(src, 0, true, qv, 16);
                if (KS * 8 > 16) load_cols(src, 16, true, qv + 16, KS * 8 - 16);
                const bool got = bar_wait(&q_empty, (ti & 1) ^ 1, &abort_flag, err, 17);
                if (!__all_sync(0xffffffffu, got)) break;
#pragma unroll
                for (int c4 = 0; c4 < KS * 2; ++c4) {
                    float4 h, lo;
                    split_tf32(qv[4 * c4] * scale, h.x, lo.x);
                    split_tf32(qv[4 * c4 + 1] * scale, h.y, lo.y);
                    split_tf32(qv[4 * c4 + 2] * scale, h.z, lo.z);
                    split_tf32(qv[4 * c4 + 3] * scale, h.w, lo.w);
                    const uint32_t o = (c4 >> 1) * 4096 + t * 32 + ((((c4 & 1) ^ (t >> 2)) & 1) << 4);
                    *reinterpret_cast<float4*>(sm + o) = h;
                    if (TERMS == 3) *reinterpret_cast<float4*>(sm + Q_BYTES + o) = lo;
                }
                fence_async();
                bar_arrive(&q_full);
            }
            bool ok = true;
            for (int j = 0; j < NBLK; ++j) {
                const long gb = g + j;
                const int s = (int)(gb % KVS);
                const bool got = bar_wait(&kv_empty[s], (uint32_t)(((gb / KVS) & 1) ^ 1), &abort_flag, err, 18);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                uint8_t* kvb = sm + OFF_KV + s * KV_BYTES;
                if (!is_v) {
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) {
                        const int cc = col0 + 4 * c4;
                        if (cc < KS * 8) {
                            float4 h, lo;
                            split_tf32(buf[4 * c4], h.x, lo.x);
                            split_tf32(buf[4 * c4 + 1], h.y, lo.y);
                            split_tf32(buf[4 * c4 + 2], h.z, lo.z);
                            split_tf32(buf[4 * c4 + 3], h.w, lo.w);
                            const uint32_t o = (cc >> 3) * 1024 + kk0 * 32 + (((((cc >> 2) & 1) ^ (kk0 >> 2)) & 1) << 4);
                            *reinterpret_cast<float4*>(kvb + o) = h;
                            if (TERMS == 3) *reinterpret_cast<float4*>(kvb + K_BYTES + o) = lo;
                        }
                    }
                } else {
#pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        const int n = col0 + f;  // feature = row of V^T
                        float4 h, lo;
                        split_tf32(buf[f], h.x, lo.x);
                        split_tf32(buf[4 + f], h.y, lo.y);
                        split_tf32(buf[8 + f], h.z, lo.z);
                        split_tf32(buf[12 + f], h.w, lo.w);
                        const uint32_t o = 2 * K_BYTES + off_sw128(n, kk0);
                        *reinterpret_cast<float4*>(kvb + o) = h;
                        if (TERMS == 3) *reinterpret_cast<float4*>(kvb + V_BYTES + o) = lo;
                    }
                }
                fence_async();
                bar_arrive(&kv_full[s]);
                if (j + 1 < NBLK) fetch(wy, wx, j + 1);
            }
            if (!ok) break;
            g += NBLK;
        }
    }

    tcf_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tcf_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem));
    }
}

template <int D, bool OCA, int TERMS>
static void run_tc(const float* qkv, const float* table, Dst out, const Plan& p, int c, int heads, int shift, int* err,
                   cudaStream_t st) {
    constexpr int KS = (D + 7) / 8;
    constexpr int TROWS = OCA ? 1521 : 961;
    constexpr size_t bytes = 2 * KS * 4096 + KVS * (2 * KS * 1024 + 2 * 4096) + 4 * 16384 + ((TROWS * 4 + 15) / 16) * 16 +
                             (OCA ? 576 * 4 : 0) + 1024;
    static unsigned configured = 0;
    int dev = 0;
    HAT_CUDA(cudaGetDevice(&dev));
    if (!(configured & (1u << dev))) {
        HAT_CUDA(cudaFuncSetAttribute(k_attn_tc<D, OCA, TERMS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
        configured |= 1u << dev;
    }
    const long items = (long)p.nw() * heads * 2;
    int sms = 0;
    HAT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // A multiple of the head count, so every CTA keeps one head (and one bias table).
    long grid = std::min<long>(items, (long)(sms / heads) * heads);
    k_attn_tc<D, OCA, TERMS><<<(unsigned)grid, TC_THREADS, bytes, st>>>(qkv, table, out, p.hp, p.wp, c, heads, shift,
                                                                        1.f / sqrtf((float)D), items, err);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

void launch_attention_tc(int mode, bool oca, const float* qkv, const float* table, Dst out, const Plan& p, int c,
                         int heads, int shift, int* err, cudaStream_t st) {
    if (p.win != 16 || p.owin != 24) throw Error(1, "attention: the kernels are built for window 16 / overlap window 24");
    if (heads <= 0 || c % heads) throw Error(1, "attention: c is not divisible by heads");
    const int d = c / heads;
    const bool three = mode == 0;
#define HAT_ATTN_CASE(DD, O)                                                                 \
    if (d == DD && oca == O) {                                                               \
        if (three)                                                                           \
            run_tc<DD, O, 3>(qkv, table, out, p, c, heads, shift, err, st);                  \
        else                                                                                 \
            run_tc<DD, O, 1>(qkv, table, out, p, c, heads, shift, err, st);                  \
        return;                                                                              \
    }
    HAT_ATTN_CASE(24, false)
    HAT_ATTN_CASE(30, false)
    HAT_ATTN_CASE(24, true)
    HAT_ATTN_CASE(30, true)
#undef HAT_ATTN_CASE
    throw Error(1, "attention: head dim " + std::to_string(d) + " is not 24 or 30");
}

}  // namespace hat
