// Tensor-core GEMM for sm_100a: tcgen05.mma (kind::f16 or kind::tf32) with the
// accumulator in tensor memory, operands staged in shared memory by TMA, one persistent
// CTA per SM.
//
//   D[m][n] = sum_k A[m][k] * B[n][k]       A: activations, B: weights (both K-major)
//
// A is either a token plane [M][K] (the HAT linears) or, for a 3x3 convolution as an
// implicit GEMM, an 8x16 pixel patch of an [H][W][C] plane shifted by each tap: the
// K loop runs over (tap, 32-channel chunk) and TMA's zero fill outside the plane is
// the conv's zero padding.
//
// fp32 parity: every operand x arrives split into x_hi + x_lo (the weights are split
// once at upload; every activation plane a GEMM reads is written split by the kernel
// that produces it), and
//   A.B ~= A_hi.B_hi + A_hi.B_lo + A_lo.B_hi,
// which drops only A_lo.B_lo (relative 2^-22). The split is fp16 pairs (H16: kind::f16,
// 16 elements of K per MMA, 2 bytes each) or tf32 pairs (kind::tf32, 8 elements of 4
// bytes); either way one MMA k-step is 32 bytes of each operand row, so the shared
// memory layout is the same. H16 weights carry a power-of-two factor that the epilogue
// takes out (`ascale`). FAST mode issues the single A_hi.B_hi on tf32. The epilogue can
// write its own output split the same way for the next GEMM.
//
// Warp roles (320 threads): 0 TMA producer, 1 MMA issuer + TMEM owner, 2-9 epilogue
// (TMEM -> registers -> fused epilogue -> global). Two epilogue warps share each TMEM
// lane quarter and take alternate 16-column chunks. Two TMEM accumulators (2 x 256
// columns) let the epilogue of one tile overlap the MMAs of the next.
//
// Every mbarrier wait is bounded (about 2 s of SM clock cycles); on expiry the kernel records an
// error code in `err`, every role leaves its loop, in-flight TMA copies and MMAs are
// waited for (again bounded) and TMEM is released before the CTA exits.
#include <cuda.h>

#include "common.cuh"
#include "umma.cuh"

namespace hat {

namespace {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false (with the abort flag raised and the error recorded) on expiry
// or when another role has already aborted. The bound is counted in SM clock cycles
// (clock64 is a cheap register read; the global timer is not, and reading it on every
// poll delayed every hand-off of the pipeline); WAIT_CYCLES is about 2 s at 1.9 GHz.
constexpr long long WAIT_CYCLES = 4000000000ll;
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort, int* err, int code) {
    if (mbar_try(b, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try(b, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > WAIT_CYCLES) {
            *abort = 1;
            atomicCAS(err, 0, code);
            return false;
        }
    }
}
// Bounded wait used on the way out (no abort flag): true when the phase completed.
__device__ __forceinline__ bool mbar_wait_quiet(uint64_t* b, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try(b, parity))
        if (clock64() - t0 > WAIT_CYCLES) return false;
    return true;
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(dst)), "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor: K-major, rows of `rowbytes` (128: SWIZZLE_128B,
// 64: SWIZZLE_64B, 32: SWIZZLE_32B), 8-row core groups `8*rowbytes` apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, int rowbytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
    d |= (uint64_t)1 << 16;                              // leading byte offset (unused here)
    d |= (uint64_t)((8 * rowbytes) >> 4) << 32;          // stride byte offset
    d |= (uint64_t)1 << 46;                              // descriptor version (sm_100)
    d |= (uint64_t)(rowbytes == 128 ? 2 : rowbytes == 64 ? 4 : 6) << 61;  // swizzle mode
    return d;
}
// Instruction descriptor: f32 accumulate, both operands K-major; A/B format 2 (tf32)
// for kind::tf32, 0 (fp16) for kind::f16.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
template <bool H16>
__host__ __device__ constexpr uint32_t idesc_k(int m, int n) {
    return H16 ? idesc_f16(m, n) : idesc_tf32(m, n);
}
__device__ __forceinline__ void mma_tf32(uint32_t dtmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(dtmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_f16(uint32_t dtmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(dtmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
template <bool H16>
__device__ __forceinline__ void mma_k(uint32_t dtmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if (H16)
        mma_f16(dtmem, a, b, idesc, acc);
    else
        mma_tf32(dtmem, a, b, idesc, acc);
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
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

// Bulk tensor stores from shared memory (the epilogue's staging tiles).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                 ::"l"((uint64_t)map), "r"(c0), "r"(c1), "r"(smem_u32(src))
                 : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                 ::"l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the staging tile may be written again (the stores in flight have read it)
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every store issued has completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Column sums of a warp's 32 x 16 values (lane = row, x[j] = column j; x is consumed): a
// transpose-and-add butterfly of 16 shuffles (8 + 4 + 2 + 1 + 1). Returns the sum over the
// 32 rows of column `col`, which the lane pair (l, l ^ 1) share.
__device__ __forceinline__ float colsum16(float* x, int lane, int& col) {
    const int h1 = (lane >> 4) & 1, h2 = (lane >> 3) & 1, h3 = (lane >> 2) & 1, h4 = (lane >> 1) & 1;
    float a8[8], a4[4], a2[2];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float keep = h1 ? x[8 + i] : x[i], give = h1 ? x[i] : x[8 + i];
        a8[i] = keep + __shfl_xor_sync(0xffffffffu, give, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float keep = h2 ? a8[4 + i] : a8[i], give = h2 ? a8[i] : a8[4 + i];
        a4[i] = keep + __shfl_xor_sync(0xffffffffu, give, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float keep = h3 ? a4[2 + i] : a4[i], give = h3 ? a4[i] : a4[2 + i];
        a2[i] = keep + __shfl_xor_sync(0xffffffffu, give, 4);
    }
    const float keep = h4 ? a2[1] : a2[0], give = h4 ? a2[0] : a2[1];
    const float a1 = keep + __shfl_xor_sync(0xffffffffu, give, 2);
    col = 8 * h1 + 4 * h2 + 2 * h3 + h4;
    return a1 + __shfl_xor_sync(0xffffffffu, a1, 1);
}

__device__ __forceinline__ float epi_act(float v, int act) {
    if (act == ACT_GELU) return gelu_fast(v);
    if (act == ACT_LEAKY) return v > 0.f ? v : 0.01f * v;
    return v;
}

}  // namespace

// One launch's geometry.
struct UmmaArgs {
    long M;          // rows (tokens / pixels)
    int N, BN, ntn;  // output columns, columns per tile, tiles along N
    int KB;          // k-blocks per tile
    int ckb;         // bytes of K per k-block row: 128 or 32
    int klast;       // MMA k-steps of a tile's last k-block (linear) / a tap's last chunk (conv)
    float ascale;    // the accumulator's factor (h16 weights: 2^-e; else 1)
    int stages;
    // conv geometry (MODE 1): plane H x W, channel chunks per tap, patch tiles along x
    int H, W, cchunks, tx;
    int ty0;         // conv: first 8-row tile row computed
    long mtiles, ntiles;
    Dst y;
    int ldo;         // row stride of the output plane (channels), for plain stores
    int nstore;      // columns stored (<= ldo)
    int tma_st;      // 1: plain fp32 stores by TMA from the staging tiles (the output's tensor map)
    int* err;
};

// Row `trow` of tile `mt`: its token / pixel index and whether it exists.
template <int MODE>
__device__ __forceinline__ void tile_row(const UmmaArgs& g, long mt, int trow, long& m, bool& valid) {
    if (MODE == 0) {
        m = mt * 128 + trow;
        valid = m < g.M;
    } else {
        const int py = (g.ty0 + (int)(mt / g.tx)) * 8 + trow / 16, px = (int)(mt % g.tx) * 16 + trow % 16;
        m = (long)py * g.W + px;
        valid = py < g.H;
    }
}

// Epilogue kinds, one kernel instantiation each so a kernel carries only its own store
// path (the instruction footprint of all of them together thrashed the instruction
// cache): EK_STORE plain/residual stores by the lanes, EK_TMA plain fp32 stores without a
// residual by TMA, EK_TMA_RES fp32 stores with a residual by TMA, EK_SHUF2 PixelShuffle(2)
// stores, EK_GENERIC everything else (planar output, other shuffle factors, odd strides),
// EK_QKV the qkv linear's attention layout, EK_RING fp32 stores with a residual (and the
// CAB term) whose inputs a second producer lane streams by TMA (below).
enum { EK_STORE = 0, EK_SHUF2 = 1, EK_GENERIC = 2, EK_TMA = 3, EK_TMA_RES = 4, EK_QKV = 5, EK_RING = 6 };

// EK_RING: the residual (and the CAB output) of each 16-column chunk of a tile, all 128
// rows, are loaded by TMA into one of RING_SLOTS shared-memory slots ([128][16] fp32 each,
// 64-byte swizzle) ahead of the epilogue; the epilogue adds the accumulator into the
// slot in place and stores it from there by TMA. The slot maps travel in QkvMaps:
// qkh = the residual, qkl = the CAB output.
constexpr int RING_SLOTS = 4;
// Chunk k's "loaded" barrier is rfull[k % RING_FULL]. The chunks of one slot are consumed by
// different warps in turn, and a warp may reach chunk k while the load of chunk k - 4 (the
// slot's previous chunk, another warp's) is still in flight; with one barrier per slot its
// parity would then read as complete. With twice as many barriers the previous use of
// rfull[k % 8] is chunk k - 8, whose slot had to be released (so its load had landed)
// before chunk k - 4 could be loaded.
constexpr int RING_FULL = 2 * RING_SLOTS;

// Epilogue warps of a k_umma kind. The qkv linear, whose attention-layout epilogue is its
// bound, runs three warps per TMEM lane quarter, each taking every third 16-column chunk;
// the other kinds two.
constexpr int umma_epi_warps(int MODE, int EK) { return MODE == 0 && EK == EK_QKV ? 12 : 8; }
// Warps ahead of the epilogue: the TMA producer, the MMA issuer and, for EK_RING, the
// residual stream's producer (a warp of its own: two lanes of one warp spinning on
// different barriers can starve each other).
constexpr int umma_lead_warps(int EK) { return EK == EK_RING ? 3 : 2; }
constexpr int umma_threads(int MODE, int EK) { return 32 * (umma_lead_warps(EK) + umma_epi_warps(MODE, EK)); }

// The four output maps of EK_QKV (see Epi::qkv_split): q|k hi and lo (SW32 boxes of 16 x
// 32), v^T hi and lo (unswizzled boxes of 32 tokens x 16 features).
struct __align__(64) QkvMaps {
    CUtensorMap qkh, qkl, vth, vtl;
};

// The bias of columns nb .. nb+15 (zeros past N or without a bias).
__device__ __forceinline__ void load_bias16(const UmmaArgs& g, const Epi& e, int nb, float* bv) {
#pragma unroll
    for (int j = 0; j < 16; ++j) bv[j] = 0.f;
    if (e.bias) {
        if (nb + 16 <= g.N) {
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4) {
                const float4 b = __ldg(reinterpret_cast<const float4*>(e.bias + nb) + j4);
                bv[4 * j4] = b.x;
                bv[4 * j4 + 1] = b.y;
                bv[4 * j4 + 2] = b.z;
                bv[4 * j4 + 3] = b.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (nb + j < g.N) bv[j] = __ldg(e.bias + nb + j);
        }
    }
}

// One 16-column chunk of an epilogue warp's 32 rows with a plain (possibly residual)
// store. Phase 1: each thread holds its own row's accumulators (TMEM lane = row), adds
// bias and activation, contributes the channel sums, and parks the values in the
// warp's staging tile. Phase 2: the warp re-reads the tile so that four lanes cover one
// row's 16 columns, and the residual loads and (split) stores are 64-byte row segments.
// `bv` is the chunk's bias, loaded by the caller a chunk ahead.
// SK, how the chunk leaves: 0 the lanes' own stores (phase 2); 1 by TMA straight from
// phase 1 (no residual); 2 by TMA after phase 2 has added the residual in place; 3 the
// qkv attention layout (fp16 pairs by TMA; v transposed), see Epi::qkv_split.
template <int MODE, int SK>
__device__ __forceinline__ void epi_chunk16(const UmmaArgs& g, const Epi& e, uint32_t taddr, int n0, int c0,
                                            long mt, int q, int lane, bool valid_own, float (*stg)[16],
                                            float* cacc, const float* bv, const CUtensorMap* tmy,
                                            const QkvMaps* qm = nullptr) {
    const int nb = n0 + c0;
    if (SK == 3) {
        float v[16];
        tmem_ld16(taddr + c0, v);
        const float qs = nb < e.qcols ? e.qscale : 1.f;
        bool big = false;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            v[j] = (v[j] * g.ascale + bv[j]) * qs;
            big |= beyond_h16(v[j]);
        }
        if (big) atomicCAS(g.err, 0, ERR_RANGE_GEMM);
        const int row0 = (int)(mt * 128 + q * 32);
        const int c2 = 2 * (g.N / 3);  // q|k columns
        __half* th = reinterpret_cast<__half*>(&stg[0][0]);
        __half* tl = th + 512;  // two 1 KB tiles
        // the previous chunk's stores have read the tiles
        if (lane == 0) bulk_wait_read();
        __syncwarp();
        if (nb < c2) {
            // q / k: this lane's row, 16 values as two 16-byte chunks per tile (32-byte rows,
            // the chunk index flipped by (row >> 2) & 1: the 32-byte swizzle of the map)
            uint32_t hp[8], lp[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) split_h16x2(v[2 * i], v[2 * i + 1], hp[i], lp[i]);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int off = lane * 32 + (((c ^ (lane >> 2)) & 1) << 4);
                *reinterpret_cast<uint4*>(reinterpret_cast<char*>(th) + off) =
                    make_uint4(hp[4 * c], hp[4 * c + 1], hp[4 * c + 2], hp[4 * c + 3]);
                *reinterpret_cast<uint4*>(reinterpret_cast<char*>(tl) + off) =
                    make_uint4(lp[4 * c], lp[4 * c + 1], lp[4 * c + 2], lp[4 * c + 3]);
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&qm->qkh, th, nb, row0);
                tma_store_2d(&qm->qkl, tl, nb, row0);
                bulk_commit();
            }
        } else {
            // v, transposed: tile [16 features][32 tokens], token = lane
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                __half h, l;
                split_h16(v[j], h, l);
                th[j * 32 + lane] = h;
                tl[j * 32 + lane] = l;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&qm->vth, th, row0, nb - c2);
                tma_store_2d(&qm->vtl, tl, row0, nb - c2);
                bulk_commit();
            }
        }
        return;
    }
    if (SK == 1) {
        // fp32 output by TMA: each lane finishes its own row (residual loaded row-wise),
        // parks it in the staging tile in the 64-byte-swizzle layout of the output's
        // tensor map, and one lane stores the 32 x 16 tile.
        long m;
        bool vrow;
        tile_row<MODE>(g, mt, q * 32 + lane, m, vrow);
        float4 r4[4], c4[4], g4[4];
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
            const bool in = vrow && nb + 4 * j4 < g.nstore;
            r4[j4] = make_float4(0.f, 0.f, 0.f, 0.f);
            c4[j4] = r4[j4];
            g4[j4] = r4[j4];
            if (in && e.res) r4[j4] = *reinterpret_cast<const float4*>(e.res + m * g.ldo + nb + 4 * j4);
            if (in && e.cx) {
                c4[j4] = *reinterpret_cast<const float4*>(e.cx + m * g.ldo + nb + 4 * j4);
                g4[j4] = *reinterpret_cast<const float4*>(e.gate + nb + 4 * j4);
            }
        }
        float v[16];
        tmem_ld16(taddr + c0, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = v[j] * g.ascale + bv[j];
        if (e.act == ACT_GELU) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = gelu_fast(v[j]);
        } else if (e.act == ACT_LEAKY) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = v[j] > 0.f ? v[j] : 0.01f * v[j];
        }
        if (nb + 16 > g.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (nb + j >= g.N) v[j] = 0.f;
        }
        if (e.colsum) {
            float x[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) x[j] = valid_own ? v[j] : 0.f;
            int col;
            const float sm = colsum16(x, lane, col);
            if (!(lane & 1) && nb + col < g.N) cacc[nb + col] += sm;
        }
        float o[16];
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
            const float rr[4] = {r4[j4].x, r4[j4].y, r4[j4].z, r4[j4].w};
            const float cc[4] = {c4[j4].x, c4[j4].y, c4[j4].z, c4[j4].w};
            const float gg[4] = {g4[j4].x, g4[j4].y, g4[j4].z, g4[j4].w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = 4 * j4 + u;
                o[j] = e.cx ? (rr[u] + v[j]) + (cc[u] * gg[u]) * e.cscale : (e.res ? rr[u] + v[j] : v[j]);
            }
        }
        // the previous chunk's store has read the tile
        if (lane == 0) bulk_wait_read();
        __syncwarp();
#pragma unroll
        for (int qq = 0; qq < 4; ++qq)
            *reinterpret_cast<float4*>(&stg[lane][4 * (qq ^ ((lane >> 1) & 3))]) =
                make_float4(o[4 * qq], o[4 * qq + 1], o[4 * qq + 2], o[4 * qq + 3]);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
            if (MODE == 0) {
                tma_store_2d(tmy, &stg[0][0], nb, (int)(mt * 128 + q * 32));
            } else {
                const int py = (g.ty0 + (int)(mt / g.tx)) * 8 + 2 * q, px = (int)(mt % g.tx) * 16;
                tma_store_3d(tmy, &stg[0][0], nb, px, py);
            }
            bulk_commit();
        }
        return;
    }
    // Phase-2 geometry and the residual loads first, so their latency overlaps the TMEM
    // load and the register work of phase 1.
    const int lr = lane >> 2, lc = (lane & 3) * 4;
    const int n = nb + lc;
    long base[4];
    bool ok[4];
    float4 rs[4], cx[4];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        long m;
        bool valid;
        tile_row<MODE>(g, mt, q * 32 + it * 8 + lr, m, valid);
        ok[it] = valid && n < g.nstore;
        base[it] = m * g.ldo + n;
        rs[it] = make_float4(0.f, 0.f, 0.f, 0.f);
        cx[it] = rs[it];
        if (ok[it] && e.res) rs[it] = *reinterpret_cast<const float4*>(e.res + base[it]);
        if (ok[it] && e.cx) cx[it] = *reinterpret_cast<const float4*>(e.cx + base[it]);
    }
    float4 gt = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e.cx && n < g.nstore) gt = *reinterpret_cast<const float4*>(e.gate + n);
    float v[16];
    tmem_ld16(taddr + c0, v);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = v[j] * g.ascale + bv[j];
    if (e.act == ACT_GELU) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = gelu_fast(v[j]);
    } else if (e.act == ACT_LEAKY) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = v[j] > 0.f ? v[j] : 0.01f * v[j];
    }
    if (nb + 16 > g.N) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (nb + j >= g.N) v[j] = 0.f;
    }
    if (e.colsum) {
        float x[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = valid_own ? v[j] : 0.f;
        int col;
        const float sm = colsum16(x, lane, col);
        if (!(lane & 1) && nb + col < g.N) cacc[nb + col] += sm;
    }
    // Staging tile rows of 16 floats, the four 16-byte chunks of row r rotated by
    // (r >> 1) & 3: both the row-per-lane stores here and the 4-lanes-per-row loads
    // below are free of bank conflicts.
    if (SK == 2) {
        // the previous chunk's store has read the tile
        if (lane == 0) bulk_wait_read();
        __syncwarp();
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
        *reinterpret_cast<float4*>(&stg[lane][4 * (q ^ ((lane >> 1) & 3))]) =
            make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        if (!ok[it]) continue;
        const int r = it * 8 + lr;
        float4 o = *reinterpret_cast<const float4*>(&stg[r][4 * ((lc >> 2) ^ ((r >> 1) & 3))]);
        if (e.cx) {
            o.x = (rs[it].x + o.x) + (cx[it].x * gt.x) * e.cscale;
            o.y = (rs[it].y + o.y) + (cx[it].y * gt.y) * e.cscale;
            o.z = (rs[it].z + o.z) + (cx[it].z * gt.z) * e.cscale;
            o.w = (rs[it].w + o.w) + (cx[it].w * gt.w) * e.cscale;
        } else if (e.res) {
            o.x = rs[it].x + o.x;
            o.y = rs[it].y + o.y;
            o.z = rs[it].z + o.z;
            o.w = rs[it].w + o.w;
        }
        if (SK == 2)
            *reinterpret_cast<float4*>(&stg[r][4 * ((lc >> 2) ^ ((r >> 1) & 3))]) = o;  // back in place
        else
            put4(g.y, base[it], o);
    }
    if (SK == 2) {
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
            if (MODE == 0) {
                tma_store_2d(tmy, &stg[0][0], nb, (int)(mt * 128 + q * 32));
            } else {
                const int py = (g.ty0 + (int)(mt / g.tx)) * 8 + 2 * q, px = (int)(mt % g.tx) * 16;
                tma_store_3d(tmy, &stg[0][0], nb, px, py);
            }
            bulk_commit();
        }
        return;
    }
    __syncwarp();
}

template <int MODE, int TERMS, int EK, bool H16>
__global__ void __launch_bounds__(umma_threads(MODE, EK), 1)
    k_umma(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
           const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl, const UmmaArgs g,
           const Epi e, const __grid_constant__ CUtensorMap tmY, const __grid_constant__ QkvMaps qm) {
    constexpr int EW = umma_epi_warps(MODE, EK), LEAD = umma_lead_warps(EK), NT = umma_threads(MODE, EK);
    constexpr int PARTS = EW / 4;
    extern __shared__ __align__(1024) uint8_t smraw[];
    __shared__ uint64_t full[6], empty[6], acc_full[2], acc_empty[2], drain;
    __shared__ uint64_t rfull[RING_FULL], rempty[RING_SLOTS];
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    constexpr bool RING = EK == EK_RING;
    // The channel-attention pool: per TMEM lane quarter, column sums accumulated over
    // every tile this CTA owns (in its fixed tile order), written once at the end. The
    // quarter's two epilogue warps own disjoint columns.
    constexpr int CA = (EK == EK_QKV || EK == EK_RING) ? 1 : 256;  // kinds without channel sums
    __shared__ float colacc[4][CA];
    // Per epilogue warp: a 32 x 16 staging tile (swizzled) for the coalesced store; the
    // rotation is the 64-byte swizzle of the TMA store path, whose pattern needs the
    // tiles 512-byte aligned.
    __shared__ __align__(1024) float stg[EK == EK_RING ? 1 : EW][32][16];

    uint8_t* sm = (uint8_t*)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    const int S = g.stages;
    const uint32_t a_bytes = 128 * g.ckb, b_bytes = g.BN * g.ckb;
    // per stage: A hi | A lo | B hi | B lo
    const uint32_t st_bytes = 2 * a_bytes + 2 * b_bytes;
    auto sAh = [&](int s) { return sm + s * st_bytes; };
    auto sAl = [&](int s) { return sm + s * st_bytes + a_bytes; };
    auto sBh = [&](int s) { return sm + s * st_bytes + 2 * a_bytes; };
    auto sBl = [&](int s) { return sm + s * st_bytes + 2 * a_bytes + b_bytes; };
    // EK_RING: the slots after the stages (each the residual chunk, then the CAB chunk),
    // then the CAB gate
    float* ring = reinterpret_cast<float*>(sm + ((S * st_bytes + 1023) & ~1023u));
    const int rstride = e.cx ? 4096 : 2048;  // floats per slot
    float* gsm = ring + RING_SLOTS * rstride;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < 4 * CA; i += NT) (&colacc[0][0])[i] = 0.f;
    if (RING && e.cx)
        for (int i = threadIdx.x; i < g.BN * g.ntn; i += NT) gsm[i] = i < g.N ? e.gate[i] : 0.f;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 32 * EW);
        }
        mbar_init(&drain, 1);
        for (int r = 0; r < RING_FULL; ++r) mbar_init(&rfull[r], 1);
        for (int r = 0; r < RING_SLOTS; ++r) mbar_init(&rempty[r], 4);  // the four lane-quarter warps that take the chunk
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const long ntiles = g.ntiles;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            const uint32_t tx = TERMS == 3 ? 2 * a_bytes + 2 * b_bytes : a_bytes + b_bytes;
            for (long t = blockIdx.x; t < ntiles && !abort_flag; t += gridDim.x) {
                const long mt = t / g.ntn;
                const int nt = (int)(t % g.ntn);
                for (int kb = 0; kb < g.KB; ++kb, ++it) {
                    const int s = it % S;
                    if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, &abort_flag, g.err, 1)) break;
                    mbar_expect_tx(&full[s], tx);
                    constexpr int ES = H16 ? 2 : 4;      // bytes per element
                    const int kel = kb * (g.ckb / ES);  // K offset in elements
                    if (MODE == 0) {
                        tma_2d(sAh(s), &tmAh, kel, (int)(mt * 128), &full[s]);
                        if (TERMS == 3) tma_2d(sAl(s), &tmAl, kel, (int)(mt * 128), &full[s]);
                    } else {
                        const int tap = kb / g.cchunks, cc = kb - tap * g.cchunks;
                        const int py = g.ty0 + (int)(mt / g.tx), px = (int)(mt % g.tx);
                        const int c0 = cc * (g.ckb / ES), x0 = px * 16 + tap % 3 - 1, y0 = py * 8 + tap / 3 - 1;
                        tma_3d(sAh(s), &tmAh, c0, x0, y0, &full[s]);
                        if (TERMS == 3) tma_3d(sAl(s), &tmAl, c0, x0, y0, &full[s]);
                    }
                    tma_2d(sBh(s), &tmBh, kel, nt * g.BN, &full[s]);
                    if (TERMS == 3) tma_2d(sBl(s), &tmBl, kel, nt * g.BN, &full[s]);
                }
            }
            if (abort_flag) {
                // Let the copies already issued land before the CTA can exit.
                for (uint32_t j = (it > (uint32_t)S ? it - S : 0); j < it; ++j) mbar_wait_quiet(&full[j % S], (j / S) & 1);
            }
        }
    } else if (RING && warp == 2) {
        if (lane == 0) {
            // the residual stream: chunk k of this CTA's tile sequence into slot k % RING_SLOTS
            uint32_t k = 0;
            const uint32_t tx = e.cx ? 16384u : 8192u;
            const int nc = g.BN / 16;
            bool ok = true;
            for (long t = blockIdx.x; t < ntiles && ok && !abort_flag; t += gridDim.x) {
                const int row0 = (int)(t / g.ntn * 128), n0 = (int)(t % g.ntn) * g.BN;
                for (int c = 0; c < nc; ++c, ++k) {
                    const int s = (int)(k % RING_SLOTS);
                    if (!mbar_wait(&rempty[s], ((k / RING_SLOTS) & 1) ^ 1, &abort_flag, g.err, 6)) {
                        ok = false;
                        break;
                    }
                    uint64_t* fb = &rfull[k % RING_FULL];
                    mbar_expect_tx(fb, tx);
                    float* slot = ring + s * rstride;
                    tma_2d(slot, &qm.qkh, n0 + 16 * c, row0, fb);
                    if (e.cx) tma_2d(slot + 2048, &qm.qkl, n0 + 16 * c, row0, fb);
                }
            }
            if (abort_flag) {
                for (uint32_t j = (k > (uint32_t)RING_SLOTS ? k - RING_SLOTS : 0); j < k; ++j)
                    mbar_wait_quiet(&rfull[j % RING_FULL], (j / RING_FULL) & 1);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t it = 0, tl = 0;
            const uint32_t idesc = idesc_k<H16>(128, g.BN);
            const int ksteps = g.ckb / 32;  // one MMA k-step = 32 bytes (8 tf32 or 16 fp16)
            for (long t = blockIdx.x; t < ntiles && !abort_flag; t += gridDim.x, ++tl) {
                const int a = tl & 1;
                if (!mbar_wait(&acc_empty[a], ((tl >> 1) & 1) ^ 1, &abort_flag, g.err, 2)) break;
                tc_fence_after();
                const uint32_t d = tmem + a * 256;
                bool ok = true;
                for (int kb = 0; kb < g.KB; ++kb, ++it) {
                    const int s = it % S;
                    if (!mbar_wait(&full[s], (it / S) & 1, &abort_flag, g.err, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ah = smem_u32(sAh(s)), al = smem_u32(sAl(s));
                    const uint32_t bh = smem_u32(sBh(s)), bl = smem_u32(sBl(s));
                    // k-steps past K (the last k-block of a row / of a tap) are skipped
                    const bool last = MODE == 0 ? kb == g.KB - 1 : (kb % g.cchunks) == g.cchunks - 1;
                    const int kst = last ? g.klast : ksteps;
#pragma unroll 1
                    for (int k = 0; k < kst; ++k) {
                        const uint32_t off = k * 32;
                        const uint32_t acc0 = (kb | k) ? 1u : 0u;
                        if (TERMS == 3) {
                            // small terms first, so they are added while the sum is small
                            mma_k<H16>(d, smem_desc(al + off, g.ckb), smem_desc(bh + off, g.ckb), idesc, acc0);
                            mma_k<H16>(d, smem_desc(ah + off, g.ckb), smem_desc(bl + off, g.ckb), idesc, 1u);
                            mma_k<H16>(d, smem_desc(ah + off, g.ckb), smem_desc(bh + off, g.ckb), idesc, 1u);
                        } else {
                            mma_k<H16>(d, smem_desc(ah + off, g.ckb), smem_desc(bh + off, g.ckb), idesc, acc0);
                        }
                    }
                    mma_commit(&empty[s]);
                }
                if (!ok) break;
                mma_commit(&acc_full[a]);
            }
            // Every MMA issued so far completes before TMEM can be released.
            mma_commit(&drain);
            mbar_wait_quiet(&drain, 0);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;          // TMEM lane quarter this warp may read
        const int row = q * 32 + lane;   // tile row of this thread
        const int ew = warp - LEAD;      // 0..EW-1 within the epilogue group
        const int part = ew >> 2;        // which of the quarter's PARTS interleaved chunk sets
        uint32_t tl = 0;
        for (long t = blockIdx.x; t < ntiles; t += gridDim.x, ++tl) {
            if (__any_sync(0xffffffffu, abort_flag != 0)) break;
            const int a = tl & 1;
            const bool got = mbar_wait(&acc_full[a], (tl >> 1) & 1, &abort_flag, g.err, 5);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const long mt = t / g.ntn;
            const int nt = (int)(t % g.ntn);
            long m;
            bool valid;
            int py = 0, px = 0;
            if (MODE == 0) {
                m = mt * 128 + row;
                valid = m < g.M;
            } else {
                py = (g.ty0 + (int)(mt / g.tx)) * 8 + row / 16;
                px = (int)(mt % g.tx) * 16 + row % 16;
                m = (long)py * g.W + px;
                valid = py < g.H;
            }
            const int n0 = nt * g.BN;
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + a * 256;
            if constexpr (RING) {
                // Each lane finishes its own row in the slot (64-byte swizzle: the 16-byte
                // piece qq of row r sits at qq ^ ((r >> 1) & 3)), then one lane stores the
                // warp's 32 rows. A slot is released once the store has read it.
                const int sw = (lane >> 1) & 3;
                const int nc = g.BN / 16;
                float bcur[16], bnext[16];
                load_bias16(g, e, n0 + 16 * part, bcur);
                int pend = -1;
                bool rok = true;
#pragma unroll 1
                for (int c0 = 16 * part; c0 < g.BN; c0 += 16 * PARTS) {
                    if (c0 + 16 * PARTS < g.BN) load_bias16(g, e, n0 + c0 + 16 * PARTS, bnext);
                    const uint32_t k = tl * nc + (c0 >> 4);
                    const int s = (int)(k % RING_SLOTS);
                    const bool in = mbar_wait(&rfull[k % RING_FULL], (k / RING_FULL) & 1, &abort_flag, g.err, 7);
                    if (!__all_sync(0xffffffffu, in)) {
                        rok = false;
                        break;
                    }
                    float v[16];
                    tmem_ld16(taddr + c0, v);
                    float* rt = ring + s * rstride + q * 512;  // this warp's 32 rows of the chunk
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq) {
                        float4* p = reinterpret_cast<float4*>(rt + lane * 16 + 4 * (qq ^ sw));
                        float4 r = *p;
                        const float o0 = v[4 * qq] * g.ascale + bcur[4 * qq];
                        const float o1 = v[4 * qq + 1] * g.ascale + bcur[4 * qq + 1];
                        const float o2 = v[4 * qq + 2] * g.ascale + bcur[4 * qq + 2];
                        const float o3 = v[4 * qq + 3] * g.ascale + bcur[4 * qq + 3];
                        if (e.cx) {
                            const float4 cx = *reinterpret_cast<const float4*>(rt + 2048 + lane * 16 + 4 * (qq ^ sw));
                            const float4 gt = *reinterpret_cast<const float4*>(gsm + n0 + c0 + 4 * qq);
                            r.x = (r.x + o0) + (cx.x * gt.x) * e.cscale;
                            r.y = (r.y + o1) + (cx.y * gt.y) * e.cscale;
                            r.z = (r.z + o2) + (cx.z * gt.z) * e.cscale;
                            r.w = (r.w + o3) + (cx.w * gt.w) * e.cscale;
                        } else {
                            r.x = r.x + o0;
                            r.y = r.y + o1;
                            r.z = r.z + o2;
                            r.w = r.w + o3;
                        }
                        *p = r;
                    }
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmY, rt, n0 + c0, (int)(mt * 128 + q * 32));
                        bulk_commit();
                        if (pend >= 0) {
                            // the previous chunk's store has read its slot
                            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                            mbar_arrive(&rempty[pend]);
                        }
                    }
                    pend = s;
#pragma unroll
                    for (int j = 0; j < 16; ++j) bcur[j] = bnext[j];
                }
                if (lane == 0 && pend >= 0) {
                    bulk_wait_read();
                    mbar_arrive(&rempty[pend]);
                }
                __syncwarp();
                tc_fence_before();
                mbar_arrive(&acc_empty[a]);
                if (!rok) break;
                continue;
            }
            if (EK == EK_SHUF2) {
                // PixelShuffle(2) store: channel n = 4c + 2i + j goes to channel c of output
                // pixel (2y + i, 2x + j). 32 columns give 8 consecutive output channels for
                // each of the 4 sub-pixels: two float4 stores per sub-pixel.
                const int cout = g.N / 4;
                for (int c0 = 32 * part; c0 < g.BN; c0 += 32 * PARTS) {
                    float bv[32];  // bias first, so its latency overlaps the TMEM loads
#pragma unroll
                    for (int j = 0; j < 32; ++j) bv[j] = e.bias ? __ldg(e.bias + n0 + c0 + j) : 0.f;
                    float v[32];
                    tmem_ld16(taddr + c0, v);
                    tmem_ld16(taddr + c0 + 16, v + 16);
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = epi_act(v[j] * g.ascale + bv[j], e.act);
                    if (valid) {
                        const int cb = (n0 + c0) / 4;
#pragma unroll
                        for (int sub = 0; sub < 4; ++sub) {
                            const long oy = 2L * py + (sub >> 1), ox = 2L * px + (sub & 1);
                            const long o = (oy * (2L * g.W) + ox) * cout + cb;
                            put4(g.y, o, make_float4(v[sub], v[4 + sub], v[8 + sub], v[12 + sub]));
                            put4(g.y, o + 4, make_float4(v[16 + sub], v[20 + sub], v[24 + sub], v[28 + sub]));
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&acc_empty[a]);
                continue;
            }
            if (EK == EK_STORE || EK == EK_TMA || EK == EK_TMA_RES || EK == EK_QKV) {
                // each chunk's bias is loaded while the chunk before it is processed
                float bcur[16], bnext[16];
                load_bias16(g, e, n0 + 16 * part, bcur);
#pragma unroll 1
                for (int c0 = 16 * part; c0 < g.BN; c0 += 16 * PARTS) {
                    if (c0 + 16 * PARTS < g.BN) load_bias16(g, e, n0 + c0 + 16 * PARTS, bnext);
                    epi_chunk16<MODE, EK == EK_TMA ? 1 : EK == EK_TMA_RES ? 2 : EK == EK_QKV ? 3 : 0>(
                        g, e, taddr, n0, c0, mt, q, lane, valid, stg[ew], colacc[q], bcur, &tmY, &qm);
#pragma unroll
                    for (int j = 0; j < 16; ++j) bcur[j] = bnext[j];
                }
                tc_fence_before();
                mbar_arrive(&acc_empty[a]);
                continue;
            }
            for (int c0 = 16 * part; c0 < g.BN; c0 += 16 * PARTS) {
                float v[16];
                tmem_ld16(taddr + c0, v);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int n = n0 + c0 + j;
                    v[j] = n < g.N ? epi_act(v[j] * g.ascale + (e.bias ? e.bias[n] : 0.f), e.act) : 0.f;
                }
                // Every loop over v[] is fully unrolled with guards rather than breaks,
                // so v stays in registers (a dynamically indexed v would live in local
                // memory, which misses in the small L1 this kernel leaves beside its
                // shared memory).
                if (valid) {
                    if (e.planar_out) {
                        const int wid = MODE == 0 ? 1 : g.W;
                        const int yy = (int)(m / wid), xx = (int)(m % wid);
                        const bool inside = yy + e.oy0 >= 0 && yy + e.oy0 < e.oh && xx < e.ow;
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int n = n0 + c0 + j;
                            if (inside && n < g.N)
                                g.y.hi[((long)n * e.oh + yy + e.oy0) * e.ow + xx] =
                                    v[j] / e.img_range + (n == 0 ? e.mean[0] : n == 1 ? e.mean[1] : e.mean[2]);
                        }
                    } else if (e.shuffle) {
                        const int r = e.shuffle, cout = g.N / (r * r);
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int n = n0 + c0 + j;
                            if (n < g.N) {
                                const int c = n / (r * r), rem = n - c * r * r, i = rem / r, jj = rem - i * r;
                                const long oy = (long)py * r + i, ox = (long)px * r + jj;
                                put(g.y, (oy * ((long)g.W * r) + ox) * cout + c, v[j]);
                            }
                        }
                    } else {
                        const long base = m * g.ldo + n0 + c0;
                        if (n0 + c0 + 16 <= g.nstore && (g.ldo % 4) == 0) {
#pragma unroll
                            for (int j4 = 0; j4 < 4; ++j4) {
                                float4 o = make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
                                if (e.cx) {
                                    const float4 r = *reinterpret_cast<const float4*>(e.res + base + 4 * j4);
                                    const float4 cx = *reinterpret_cast<const float4*>(e.cx + base + 4 * j4);
                                    const int n = n0 + c0 + 4 * j4;
                                    o.x = (r.x + o.x) + (cx.x * e.gate[n]) * e.cscale;
                                    o.y = (r.y + o.y) + (cx.y * e.gate[n + 1]) * e.cscale;
                                    o.z = (r.z + o.z) + (cx.z * e.gate[n + 2]) * e.cscale;
                                    o.w = (r.w + o.w) + (cx.w * e.gate[n + 3]) * e.cscale;
                                } else if (e.res) {
                                    const float4 r = *reinterpret_cast<const float4*>(e.res + base + 4 * j4);
                                    o.x = r.x + o.x;
                                    o.y = r.y + o.y;
                                    o.z = r.z + o.z;
                                    o.w = r.w + o.w;
                                }
                                put4(g.y, base + 4 * j4, o);
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                const int n = n0 + c0 + j;
                                if (n < g.nstore) {
                                    float o = v[j];
                                    if (e.cx)
                                        o = (e.res[base + j] + o) + (e.cx[base + j] * e.gate[n]) * e.cscale;
                                    else if (e.res)
                                        o = e.res[base + j] + o;
                                    put(g.y, base + j, o);
                                }
                            }
                        }
                    }
                }
                if (e.colsum) {
                    // Column sums of this warp's 32 rows, reduced in a fixed order and
                    // accumulated per warp across this CTA's tiles.
                    float x[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) x[j] = valid ? v[j] : 0.f;
                    int col;
                    const float sm = colsum16(x, lane, col);
                    const int n = n0 + c0 + col;
                    if (!(lane & 1) && n < g.N) colacc[q][n] += sm;
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[a]);
        }
        if (e.colsum) {
            __syncwarp();
            // Each warp writes the columns it owns (its chunk parity within a tile).
            for (int n = lane; n < g.N; n += 32)
                if (((n % g.BN) >> 4) % PARTS == part) e.colsum[((long)blockIdx.x * 4 + q) * g.N + n] = colacc[q][n];
        }
    }

    // The epilogue's bulk stores complete before the CTA (and its staging tiles) go away.
    if ((EK == EK_TMA || EK == EK_TMA_RES || EK == EK_QKV || EK == EK_RING) && warp >= LEAD && lane == 0) bulk_wait_all();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

// ------------------------------------------------------------------ fused MLP
// The HAB / OCAB MLP in one launch (hat_arch.py:252-263 with the residual of :309):
//
//   out = res + b2 + W2 . GELU(W1 . n + b1)        n: the LayerNorm output, split hi/lo
//
// per 128-row tile. The hidden activations never leave the SM: the hidden width runs in
// chunks of MLP_HC = 96 columns; each chunk's fc1 accumulator (96 TMEM columns) is read
// by the epilogue warps, which add b1, apply GELU, split the result into hi/lo (fp16
// pairs, packed two to a column, for H16; tf32 otherwise) and write it back into TMEM,
// where it is the A operand of that chunk's fc2 products (`tcgen05.mma` with A in
// tensor memory), accumulated into the tile's fc2 accumulator. The tile's last chunk
// done, the epilogue adds b2 and the residual and stores, like the GEMM's plain-store
// epilogue. TMEM columns: fc2 accumulator [0, CP), fc1 chunk [CP, CP+96), hidden hi
// [CP+96, CP+96+HW), hidden lo [CP+96+HW, CP+96+2HW), HW = 48 (H16) or 96.
//
// Order of the MMA issuer per tile (each fc1 chunk needs the previous chunk's
// accumulator read; each fc2 chunk needs that chunk's hidden values written):
//   fc1(0); for h: { fc1(h+1) if any; fc2(h) }
// and the TMA producer loads the operands in exactly that order through the same ring.
constexpr int MLP_HC = 96;
constexpr int MLP_MAXH = 768;  // the largest padded hidden width the fused MLP takes

struct MlpArgs {
    int C, HID, NCH, CP, KB1, stages;
    int klast1;       // MMA k-steps of fc1's last k-block
    float s1;         // fc1 accumulator factor (H16 weight scale; fc2's is st.ascale)
    long mtiles;
    const float* b1;  // [HID]
    UmmaArgs st;      // the final store's geometry (N = C, BN = CP, one column tile)
};

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
          "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
          "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
          "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
          "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
          "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ void mma_tf32_ts(uint32_t dtmem, uint32_t atmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(dtmem), "r"(atmem), "l"(b), "r"(idesc), "r"(acc));
}
// A in tensor memory as fp16 pairs: column j holds k = 2j (low half) and 2j + 1.
__device__ __forceinline__ void mma_f16_ts(uint32_t dtmem, uint32_t atmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(dtmem), "r"(atmem), "l"(b), "r"(idesc), "r"(acc));
}
template <bool H16>
__device__ __forceinline__ void mma_k_ts(uint32_t dtmem, uint32_t atmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    if (H16)
        mma_f16_ts(dtmem, atmem, b, idesc, acc);
    else
        mma_tf32_ts(dtmem, atmem, b, idesc, acc);
}
__device__ __forceinline__ void tmem_st8u(uint32_t taddr, const uint32_t* r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

// SK as for epi_chunk16 (0, 1, 2), or MLP_RT: the producer warp loads the tile's residual
// rows by TMA into a shared-memory tile ([CP/16 chunks][128 rows][16], 64-byte swizzle)
// while the hidden chunks run; the final epilogue adds fc2 + bias into that tile in place
// and stores it by TMA, so no global load sits on the epilogue's critical path.
constexpr int MLP_RT = 4;
// Epilogue warps of a k_mlp variant: the fp16-pair, residual-tile one (whose GELU phase bounds
// it) runs three per TMEM lane quarter, each taking 32 of a hidden chunk's 96 columns; the
// others two (48 columns each).
constexpr int mlp_epi_warps(bool H16, int SK) { return H16 && SK == MLP_RT ? 12 : 8; }
template <int TERMS, bool H16, int SK>
__global__ void __launch_bounds__(64 + 32 * mlp_epi_warps(H16, SK), 1)
    k_mlp(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
          const __grid_constant__ CUtensorMap tmW1h, const __grid_constant__ CUtensorMap tmW1l,
          const __grid_constant__ CUtensorMap tmW2h, const __grid_constant__ CUtensorMap tmW2l, const MlpArgs g,
          const Epi e, const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmR) {
    constexpr bool RT = SK == MLP_RT;
    constexpr int EW = mlp_epi_warps(H16, SK), NT = 64 + 32 * EW, PARTS = EW / 4;
    constexpr int CW = MLP_HC / PARTS;  // hidden columns of a chunk per epilogue warp
    static_assert(CW % 16 == 0, "whole 16-column TMEM loads per warp");
    extern __shared__ __align__(1024) uint8_t smraw[];
    __shared__ uint64_t full[6], empty[6], d1_full, d1_free, h_full, h_empty, d2_full, d2_free, drain;
    __shared__ uint64_t res_full, res_empty;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    __shared__ __align__(1024) float stg[RT ? 1 : EW][32][16];
    __shared__ float no_colsum[256];
    __shared__ float b1s[MLP_MAXH];  // fc1 bias, zero past HID (read by every chunk)

    uint8_t* sm = (uint8_t*)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    const int S = g.stages;
    const uint32_t A_B = 128 * 128, W1_B = MLP_HC * 128, W2_B = (uint32_t)g.CP * 128;
    for (int i = threadIdx.x; i < MLP_MAXH; i += NT) b1s[i] = i < g.HID ? g.b1[i] : 0.f;
    const uint32_t st_bytes = max(2 * A_B + 2 * W1_B, 2 * W2_B);
    float* rtile = reinterpret_cast<float*>(sm + S * st_bytes);  // MLP_RT: the residual / output tile
    int* gerr = g.st.err;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&d1_full, 1);
        mbar_init(&d1_free, 32 * EW);
        mbar_init(&h_full, 32 * EW);
        mbar_init(&h_empty, 1);
        mbar_init(&d2_full, 1);
        mbar_init(&d2_free, 32 * EW);
        mbar_init(&drain, 1);
        mbar_init(&res_full, 1);
        mbar_init(&res_empty, EW);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    constexpr uint32_t HW = H16 ? MLP_HC / 2 : MLP_HC;  // TMEM columns of one hidden half (hi or lo)
    constexpr int KEL = H16 ? 64 : 32;                   // K elements per 128-byte k-block row
    constexpr int NKB2 = (MLP_HC + KEL - 1) / KEL;       // fc2 k-blocks per hidden chunk
    const uint32_t T_D2 = 0, T_D1 = (uint32_t)g.CP, T_HH = T_D1 + MLP_HC, T_HL = T_HH + HW;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            auto stage = [&](uint32_t bytes) -> int {
                const int s = (int)(it % S);
                if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, &abort_flag, gerr, 21)) return -1;
                mbar_expect_tx(&full[s], bytes);
                return s;
            };
            auto load_fc1 = [&](long t, int h) {
                for (int kb = 0; kb < g.KB1 && ok; ++kb, ++it) {
                    const int s = stage(TERMS == 3 ? 2 * A_B + 2 * W1_B : A_B + W1_B);
                    if (s < 0) {
                        ok = false;
                        break;
                    }
                    uint8_t* b = sm + s * st_bytes;
                    tma_2d(b, &tmAh, kb * KEL, (int)(t * 128), &full[s]);
                    if (TERMS == 3) tma_2d(b + A_B, &tmAl, kb * KEL, (int)(t * 128), &full[s]);
                    tma_2d(b + 2 * A_B, &tmW1h, kb * KEL, h * MLP_HC, &full[s]);
                    if (TERMS == 3) tma_2d(b + 2 * A_B + W1_B, &tmW1l, kb * KEL, h * MLP_HC, &full[s]);
                }
            };
            auto load_fc2 = [&](int h) {
                for (int kb = 0; kb < NKB2 && ok; ++kb, ++it) {
                    const int s = stage(TERMS == 3 ? 2 * W2_B : W2_B);
                    if (s < 0) {
                        ok = false;
                        break;
                    }
                    uint8_t* b = sm + s * st_bytes;
                    tma_2d(b, &tmW2h, h * MLP_HC + kb * KEL, 0, &full[s]);
                    if (TERMS == 3) tma_2d(b + W2_B, &tmW2l, h * MLP_HC + kb * KEL, 0, &full[s]);
                }
            };
            uint32_t rn = 0;  // residual tiles issued
            auto load_res = [&](long t) {
                // the previous tile's output stores have read the tile
                if (!mbar_wait(&res_empty, (rn & 1) ^ 1, &abort_flag, gerr, 31)) {
                    ok = false;
                    return;
                }
                mbar_expect_tx(&res_full, (uint32_t)g.CP * 512);
                for (int c = 0; c < g.CP / 16; ++c) tma_2d(rtile + c * 2048, &tmR, c * 16, (int)(t * 128), &res_full);
                ++rn;
            };
            for (long t = blockIdx.x; t < g.mtiles && ok && !abort_flag; t += gridDim.x) {
                load_fc1(t, 0);
                for (int h = 0; h < g.NCH && ok; ++h) {
                    if (h + 1 < g.NCH) load_fc1(t, h + 1);
                    load_fc2(h);
                    // Issued once the tile's first chunk is under way: by then the epilogue
                    // has finished the previous tile, so the wait above does not hold up
                    // the weight loads.
                    if (RT && h == 0 && ok) load_res(t);
                }
            }
            if (abort_flag) {
                for (uint32_t j = (it > (uint32_t)S ? it - S : 0); j < it; ++j) mbar_wait_quiet(&full[j % S], (j / S) & 1);
                if (RT && rn) mbar_wait_quiet(&res_full, (rn - 1) & 1);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t it = 0, qn = 0, tl = 0;  // ring position, next fc1 chunk, local tile
            const uint32_t id1 = idesc_k<H16>(128, MLP_HC), id2 = idesc_k<H16>(128, g.CP);
            bool ok = true;
            auto fc1 = [&]() {
                // D1 free: the epilogue has read the previous chunk's accumulator.
                if (!mbar_wait(&d1_free, (qn & 1) ^ 1, &abort_flag, gerr, 22)) {
                    ok = false;
                    return;
                }
                tc_fence_after();
                const uint32_t d = tmem + T_D1;
                for (int kb = 0; kb < g.KB1; ++kb, ++it) {
                    const int s = (int)(it % S);
                    if (!mbar_wait(&full[s], (it / S) & 1, &abort_flag, gerr, 23)) {
                        ok = false;
                        return;
                    }
                    tc_fence_after();
                    const uint32_t ah = smem_u32(sm + s * st_bytes), al = ah + A_B;
                    const uint32_t bh = ah + 2 * A_B, bl = bh + W1_B;
                    const int kst = kb == g.KB1 - 1 ? g.klast1 : 4;
#pragma unroll 1
                    for (int k = 0; k < kst; ++k) {
                        const uint32_t off = k * 32, acc0 = (kb | k) ? 1u : 0u;
                        if (TERMS == 3) {
                            mma_k<H16>(d, smem_desc(al + off, 128), smem_desc(bh + off, 128), id1, acc0);
                            mma_k<H16>(d, smem_desc(ah + off, 128), smem_desc(bl + off, 128), id1, 1u);
                            mma_k<H16>(d, smem_desc(ah + off, 128), smem_desc(bh + off, 128), id1, 1u);
                        } else {
                            mma_k<H16>(d, smem_desc(ah + off, 128), smem_desc(bh + off, 128), id1, acc0);
                        }
                    }
                    mma_commit(&empty[s]);
                }
                mma_commit(&d1_full);
                ++qn;
            };
            for (long t = blockIdx.x; t < g.mtiles && ok && !abort_flag; t += gridDim.x, ++tl) {
                const uint32_t q0 = qn;
                fc1();
                for (int h = 0; h < g.NCH && ok; ++h) {
                    const uint32_t q = q0 + h;
                    if (h + 1 < g.NCH) {
                        fc1();
                        if (!ok) break;
                    }
                    // This chunk's hidden values written; for the tile's first chunk, the
                    // previous tile's fc2 accumulator read.
                    if (!mbar_wait(&h_full, q & 1, &abort_flag, gerr, 24)) {
                        ok = false;
                        break;
                    }
                    if (h == 0 && !mbar_wait(&d2_free, (tl & 1) ^ 1, &abort_flag, gerr, 25)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + T_D2;
                    for (int kb = 0; kb < NKB2; ++kb, ++it) {
                        const int s = (int)(it % S);
                        if (!mbar_wait(&full[s], (it / S) & 1, &abort_flag, gerr, 26)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t bh = smem_u32(sm + s * st_bytes), bl = bh + W2_B;
                        // k-steps of this k-block inside the chunk (H16: 64 + 32 of 96)
                        const int kst = (MLP_HC - kb * KEL) / (KEL / 4) < 4 ? (MLP_HC - kb * KEL) / (KEL / 4) : 4;
#pragma unroll 1
                        for (int k = 0; k < kst; ++k) {
                            // TMEM column of this k-step's A: one per element (tf32), one per pair (fp16)
                            const uint32_t col = H16 ? (uint32_t)((kb * KEL + k * 16) / 2) : (uint32_t)(kb * 32 + k * 8);
                            const uint32_t off = k * 32;
                            const uint32_t acc0 = (h | kb | k) ? 1u : 0u;
                            if (TERMS == 3) {
                                mma_k_ts<H16>(d, tmem + T_HL + col, smem_desc(bh + off, 128), id2, acc0);
                                mma_k_ts<H16>(d, tmem + T_HH + col, smem_desc(bl + off, 128), id2, 1u);
                                mma_k_ts<H16>(d, tmem + T_HH + col, smem_desc(bh + off, 128), id2, 1u);
                            } else {
                                mma_k_ts<H16>(d, tmem + T_HH + col, smem_desc(bh + off, 128), id2, acc0);
                            }
                        }
                        mma_commit(&empty[s]);
                    }
                    if (!ok) break;
                    mma_commit(&h_empty);
                }
                if (!ok) break;
                mma_commit(&d2_full);
            }
            mma_commit(&drain);
            mbar_wait_quiet(&drain, 0);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;
        const int ew = warp - 2;
        const int part = ew >> 2;  // which of the quarter's PARTS column sets
        const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
        uint32_t qc = 0, tl = 0;
        for (long t = blockIdx.x; t < g.mtiles; t += gridDim.x, ++tl) {
            if (__any_sync(0xffffffffu, abort_flag != 0)) break;
            bool ok = true;
            for (int h = 0; h < g.NCH; ++h, ++qc) {
                const bool got = mbar_wait(&d1_full, qc & 1, &abort_flag, gerr, 27);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // This warp's CW columns of the chunk.
                float v[CW];
#pragma unroll
                for (int i = 0; i < CW / 16; ++i) tmem_ld16(tmem + lanes + T_D1 + part * CW + 16 * i, v + 16 * i);
                tc_fence_before();
                mbar_arrive(&d1_free);
                const int nb = h * MLP_HC + part * CW;
#pragma unroll
                for (int j = 0; j < CW; ++j) {
                    const float x = v[j] * g.s1 + b1s[nb + j];
                    v[j] = gelu_fast(x);
                }
                // The hidden buffer is free once the previous chunk's fc2 has run.
                const bool freed = mbar_wait(&h_empty, (qc & 1) ^ 1, &abort_flag, gerr, 28);
                if (!__all_sync(0xffffffffu, freed)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (H16) {
                    // CW values -> CW/2 packed pairs of hi and of lo (columns part*CW/2 ..)
                    uint32_t hp[CW / 2], lp[CW / 2];
#pragma unroll
                    for (int j = 0; j < CW / 2; ++j) split_h16x2(v[2 * j], v[2 * j + 1], hp[j], lp[j]);
#pragma unroll
                    for (int i = 0; i < CW / 16; ++i) {
                        tmem_st8u(tmem + lanes + T_HH + part * (CW / 2) + 8 * i, hp + 8 * i);
                        if (TERMS == 3) tmem_st8u(tmem + lanes + T_HL + part * (CW / 2) + 8 * i, lp + 8 * i);
                    }
                } else {
#pragma unroll
                    for (int g16 = 0; g16 < CW / 16; ++g16) {
                        float hi[16], lo[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            if (TERMS == 3) {
                                split_tf32(v[16 * g16 + j], hi[j], lo[j]);
                            } else {
                                hi[j] = tf32_rna(v[16 * g16 + j]);
                                lo[j] = 0.f;
                            }
                        }
                        tmem_st16(tmem + lanes + T_HH + part * CW + 16 * g16, hi);
                        if (TERMS == 3) tmem_st16(tmem + lanes + T_HL + part * CW + 16 * g16, lo);
                    }
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                mbar_arrive(&h_full);
            }
            if (!ok) break;
            const bool got = mbar_wait(&d2_full, tl & 1, &abort_flag, gerr, 29);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            if constexpr (RT) {
                const bool rg = mbar_wait(&res_full, tl & 1, &abort_flag, gerr, 32);
                if (!__all_sync(0xffffffffu, rg)) break;
                const int sw = (lane >> 1) & 3;  // this row's 16-byte chunk rotation (64-byte swizzle)
                float bcur[16], bnext[16];
                load_bias16(g.st, e, 16 * part, bcur);
#pragma unroll 1
                for (int c0 = 16 * part; c0 < g.CP; c0 += 16 * PARTS) {
                    if (c0 + 16 * PARTS < g.CP) load_bias16(g.st, e, c0 + 16 * PARTS, bnext);
                    float v[16];
                    tmem_ld16(tmem + lanes + T_D2 + c0, v);
                    float* tile = rtile + (c0 >> 4) * 2048 + q4 * 512;  // this warp's 32 rows of the chunk
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq) {
                        float4* p = reinterpret_cast<float4*>(tile + lane * 16 + 4 * (qq ^ sw));
                        float4 r = *p;
                        r.x = r.x + (v[4 * qq] * g.st.ascale + bcur[4 * qq]);
                        r.y = r.y + (v[4 * qq + 1] * g.st.ascale + bcur[4 * qq + 1]);
                        r.z = r.z + (v[4 * qq + 2] * g.st.ascale + bcur[4 * qq + 2]);
                        r.w = r.w + (v[4 * qq + 3] * g.st.ascale + bcur[4 * qq + 3]);
                        *p = r;
                    }
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmY, tile, c0, (int)(t * 128 + q4 * 32));
                        bulk_commit();
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) bcur[j] = bnext[j];
                }
                tc_fence_before();
                mbar_arrive(&d2_free);
                if (lane == 0) {
                    bulk_wait_read();
                    mbar_arrive(&res_empty);
                }
                __syncwarp();
            } else {
                const long m = t * 128 + row;
                const bool valid = m < g.st.M;
                float bcur[16], bnext[16];
                load_bias16(g.st, e, 16 * part, bcur);
#pragma unroll 1
                for (int c0 = 16 * part; c0 < g.CP; c0 += 16 * PARTS) {
                    if (c0 + 16 * PARTS < g.CP) load_bias16(g.st, e, c0 + 16 * PARTS, bnext);
                    epi_chunk16<0, SK>(g.st, e, tmem + lanes + T_D2, 0, c0, t, q4, lane, valid, stg[ew], no_colsum,
                                       bcur, &tmY);
#pragma unroll
                    for (int j = 0; j < 16; ++j) bcur[j] = bnext[j];
                }
                tc_fence_before();
                mbar_arrive(&d2_free);
            }
        }
    }

    if (SK != 0 && warp >= 2 && lane == 0) bulk_wait_all();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

// ------------------------------------------------------------------ proj + CAB conv2
// The HAB's proj linear with the CAB's second conv folded into the same accumulator
// (hat_arch.py:299-309: x = shortcut + attn_x + conv_x * conv_scale, conv_x = the CAB's
// 3x3 conv cc -> c times its channel-attention gate):
//
//   out = res + bias' + Wp . attn + W2' (*) cmid       W2'[n] = conv_scale * gate[n] * W2[n]
//                                                      bias'  = bp + conv_scale * gate * b2
//
// The gate scales whole output channels, so it folds into the conv's weight rows (written
// for each block by the gate kernel, k_ca_gate) and the conv's output never exists as a
// plane: no c-channel fp32 plane is written by the conv and read back by proj. The tiles
// are the conv's 8 x 16 pixel patches of the [rows][W][*] planes; a tile's K loop runs
// first over the attention output's channel chunks at the patch itself (128-byte k-block
// rows), then over (tap, channel chunk) of the cmid view (`ckb_b`-byte rows, the patch
// shifted by the tap, TMA's zero fill outside the view as the conv's zero padding). Both
// weight parts carry proj's power-of-two factor, so one accumulator serves both. The
// With 32-byte conv rows, four of the conv's k-blocks share one pipeline stage (a stage is
// sized for 128-byte rows), so the short conv steps do not each wait out a load. The
// epilogue is the residual ring of k_umma (EK_RING) on patches: a producer warp streams
// the residual's 16-column chunks of the patch by TMA, the epilogue adds bias' and the
// accumulator in place and stores two pixel rows per warp by TMA.
struct ProjCabArgs {
    int N, BN, ntn;
    int KBa, klast_a;               // proj: k-blocks of 64-byte rows, k-steps of the last
    int ckb_b, cchunks_b, klast_b;  // conv: bytes per k-block row, chunks per tap, k-steps of a tap's last
    int tx, ty0, yoff_b;            // patches along x, first patch row, cmid view row of plane row 0
    long ntiles;
    float ascale;
    int stages;
    int slots;          // residual ring slots (at most PC_SLOTS_MAX)
    const float* bias;  // bias' [N]
    int* err;
};

// Pipeline stages of k_proj_cab hold 64-byte k-block rows (a 128-byte row per stage left
// room for two stages only, and the K loop waited out every load); the residual ring
// takes PC_SLOTS of 16-column chunks.
constexpr int PC_SLOTS_MAX = 12, PC_SLOTS = 6;

template <int TERMS, bool H16>
__global__ void __launch_bounds__(32 * 11, 1)
    k_proj_cab(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
               const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
               const __grid_constant__ CUtensorMap tmCh, const __grid_constant__ CUtensorMap tmCl,
               const __grid_constant__ CUtensorMap tmDh, const __grid_constant__ CUtensorMap tmDl,
               const __grid_constant__ CUtensorMap tmR, const __grid_constant__ CUtensorMap tmY,
               const ProjCabArgs g) {
    constexpr int LEAD = 3, EW = 8, NT = 32 * (LEAD + EW), PARTS = EW / 4;
    constexpr int ES = H16 ? 2 : 4;  // bytes per element
    extern __shared__ __align__(1024) uint8_t smraw[];
    __shared__ uint64_t full[6], empty[6], acc_full[2], acc_empty[2], drain;
    __shared__ uint64_t rfull[2 * PC_SLOTS_MAX], rempty[PC_SLOTS_MAX];
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;

    uint8_t* sm = (uint8_t*)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    const int S = g.stages;
    // per stage, sized for 64-byte rows: A hi | A lo | B hi | B lo
    const uint32_t a_max = 128 * 64, b_max = (uint32_t)g.BN * 64;
    const uint32_t st_bytes = 2 * a_max + 2 * b_max;
    float* ring = reinterpret_cast<float*>(sm + S * st_bytes);  // RS x [128][16] fp32
    const int RS = g.slots, RF = 2 * RS;  // slots, and "loaded" barriers as in EK_RING
    // Pipeline steps of a tile: KBa proj k-blocks, then the conv's k-blocks G to a step.
    const int KBb = 9 * g.cchunks_b, G = 64 / g.ckb_b;
    const int NSTEP = g.KBa + (KBb + G - 1) / G;
    const uint32_t a_sub = 128u * (uint32_t)g.ckb_b, b_sub = (uint32_t)g.BN * (uint32_t)g.ckb_b;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 32 * EW);
        }
        mbar_init(&drain, 1);
        for (int r = 0; r < RF; ++r) mbar_init(&rfull[r], 1);
        for (int r = 0; r < RS; ++r) mbar_init(&rempty[r], 4);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (long t = blockIdx.x; t < g.ntiles && ok && !abort_flag; t += gridDim.x) {
                const long mt = t / g.ntn;
                const int nt = (int)(t % g.ntn);
                const int py = g.ty0 + (int)(mt / g.tx), px = (int)(mt % g.tx);
                for (int st = 0; st < NSTEP; ++st, ++it) {
                    const int s = it % S;
                    const bool seg_a = st < g.KBa;
                    const int kb0 = seg_a ? 0 : (st - g.KBa) * G, cnt = seg_a ? 1 : min(G, KBb - kb0);
                    const uint32_t bytes = seg_a ? a_max + b_max : (uint32_t)cnt * (a_sub + b_sub);
                    if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, &abort_flag, g.err, 41)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full[s], TERMS == 3 ? 2 * bytes : bytes);
                    uint8_t* b = sm + s * st_bytes;
                    if (seg_a) {
                        const int kel = st * (64 / ES);
                        tma_3d(b, &tmAh, kel, px * 16, py * 8, &full[s]);
                        if (TERMS == 3) tma_3d(b + a_max, &tmAl, kel, px * 16, py * 8, &full[s]);
                        tma_2d(b + 2 * a_max, &tmBh, kel, nt * g.BN, &full[s]);
                        if (TERMS == 3) tma_2d(b + 2 * a_max + b_max, &tmBl, kel, nt * g.BN, &full[s]);
                    } else {
                        const int cke = g.ckb_b / ES;
                        for (int i = 0; i < cnt; ++i) {
                            const int kb2 = kb0 + i, tap = kb2 / g.cchunks_b, cc = kb2 - tap * g.cchunks_b;
                            const int x0 = px * 16 + tap % 3 - 1, y0 = py * 8 + tap / 3 - 1 + g.yoff_b;
                            tma_3d(b + i * a_sub, &tmCh, cc * cke, x0, y0, &full[s]);
                            if (TERMS == 3) tma_3d(b + a_max + i * a_sub, &tmCl, cc * cke, x0, y0, &full[s]);
                            tma_2d(b + 2 * a_max + i * b_sub, &tmDh, kb2 * cke, nt * g.BN, &full[s]);
                            if (TERMS == 3)
                                tma_2d(b + 2 * a_max + b_max + i * b_sub, &tmDl, kb2 * cke, nt * g.BN, &full[s]);
                        }
                    }
                }
            }
            if (abort_flag) {
                for (uint32_t j = (it > (uint32_t)S ? it - S : 0); j < it; ++j) mbar_wait_quiet(&full[j % S], (j / S) & 1);
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ residual stream
        if (lane == 0) {
            uint32_t k = 0;
            const int nc = g.BN / 16;
            bool ok = true;
            for (long t = blockIdx.x; t < g.ntiles && ok && !abort_flag; t += gridDim.x) {
                const long mt = t / g.ntn;
                const int n0 = (int)(t % g.ntn) * g.BN;
                const int py = g.ty0 + (int)(mt / g.tx), px = (int)(mt % g.tx);
                for (int c = 0; c < nc; ++c, ++k) {
                    const int s = (int)(k % RS);
                    if (!mbar_wait(&rempty[s], ((k / RS) & 1) ^ 1, &abort_flag, g.err, 42)) {
                        ok = false;
                        break;
                    }
                    uint64_t* fb = &rfull[k % RF];
                    mbar_expect_tx(fb, 8192u);
                    tma_3d(ring + s * 2048, &tmR, n0 + 16 * c, px * 16, py * 8, fb);
                }
            }
            if (abort_flag) {
                for (uint32_t j = (k > (uint32_t)RS ? k - RS : 0); j < k; ++j) mbar_wait_quiet(&rfull[j % RF], (j / RF) & 1);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t it = 0, tl = 0;
            const uint32_t idesc = idesc_k<H16>(128, g.BN);
            for (long t = blockIdx.x; t < g.ntiles && !abort_flag; t += gridDim.x, ++tl) {
                const int a = tl & 1;
                if (!mbar_wait(&acc_empty[a], ((tl >> 1) & 1) ^ 1, &abort_flag, g.err, 43)) break;
                tc_fence_after();
                const uint32_t d = tmem + a * 256;
                bool ok = true;
                for (int st = 0; st < NSTEP; ++st, ++it) {
                    const int s = it % S;
                    if (!mbar_wait(&full[s], (it / S) & 1, &abort_flag, g.err, 44)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const bool seg_a = st < g.KBa;
                    const int ckb = seg_a ? 64 : g.ckb_b;
                    const int kb0 = seg_a ? 0 : (st - g.KBa) * G, cnt = seg_a ? 1 : min(G, KBb - kb0);
                    const uint32_t base = smem_u32(sm + s * st_bytes);
#pragma unroll 1
                    for (int i = 0; i < cnt; ++i) {
                        int kst;
                        if (seg_a)
                            kst = st == g.KBa - 1 ? g.klast_a : 2;
                        else
                            kst = (kb0 + i) % g.cchunks_b == g.cchunks_b - 1 ? g.klast_b : ckb / 32;
                        const uint32_t ah = base + (seg_a ? 0u : i * a_sub), al = ah + a_max;
                        const uint32_t bh = base + 2 * a_max + (seg_a ? 0u : i * b_sub), bl = bh + b_max;
#pragma unroll 1
                        for (int k = 0; k < kst; ++k) {
                            const uint32_t off = k * 32;
                            const uint32_t acc0 = (st | i | k) ? 1u : 0u;
                            if (TERMS == 3) {
                                mma_k<H16>(d, smem_desc(al + off, ckb), smem_desc(bh + off, ckb), idesc, acc0);
                                mma_k<H16>(d, smem_desc(ah + off, ckb), smem_desc(bl + off, ckb), idesc, 1u);
                                mma_k<H16>(d, smem_desc(ah + off, ckb), smem_desc(bh + off, ckb), idesc, 1u);
                            } else {
                                mma_k<H16>(d, smem_desc(ah + off, ckb), smem_desc(bh + off, ckb), idesc, acc0);
                            }
                        }
                    }
                    mma_commit(&empty[s]);
                }
                if (!ok) break;
                mma_commit(&acc_full[a]);
            }
            mma_commit(&drain);
            mbar_wait_quiet(&drain, 0);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;
        const int ew = warp - LEAD;
        const int part = ew >> 2;
        const int sw = (lane >> 1) & 3;
        const int nc = g.BN / 16;
        uint32_t tl = 0;
        for (long t = blockIdx.x; t < g.ntiles; t += gridDim.x, ++tl) {
            if (__any_sync(0xffffffffu, abort_flag != 0)) break;
            const int a = tl & 1;
            const bool got = mbar_wait(&acc_full[a], (tl >> 1) & 1, &abort_flag, g.err, 45);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const long mt = t / g.ntn;
            const int n0 = (int)(t % g.ntn) * g.BN;
            const int py = g.ty0 + (int)(mt / g.tx), px = (int)(mt % g.tx);
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + a * 256;
            float bcur[16], bnext[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) bcur[j] = n0 + 16 * part + j < g.N ? __ldg(g.bias + n0 + 16 * part + j) : 0.f;
            int pend = -1;
            bool rok = true;
#pragma unroll 1
            for (int c0 = 16 * part; c0 < g.BN; c0 += 16 * PARTS) {
                if (c0 + 16 * PARTS < g.BN) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = n0 + c0 + 16 * PARTS + j;
                        bnext[j] = n < g.N ? __ldg(g.bias + n) : 0.f;
                    }
                }
                const uint32_t k = tl * nc + (c0 >> 4);
                const int s = (int)(k % RS);
                const bool in = mbar_wait(&rfull[k % RF], (k / RF) & 1, &abort_flag, g.err, 46);
                if (!__all_sync(0xffffffffu, in)) {
                    rok = false;
                    break;
                }
                float v[16];
                tmem_ld16(taddr + c0, v);
                float* rt = ring + s * 2048 + q * 512;  // this warp's 32 rows (two pixel rows) of the chunk
#pragma unroll
                for (int qq = 0; qq < 4; ++qq) {
                    float4* p = reinterpret_cast<float4*>(rt + lane * 16 + 4 * (qq ^ sw));
                    float4 r = *p;
                    r.x = r.x + (v[4 * qq] * g.ascale + bcur[4 * qq]);
                    r.y = r.y + (v[4 * qq + 1] * g.ascale + bcur[4 * qq + 1]);
                    r.z = r.z + (v[4 * qq + 2] * g.ascale + bcur[4 * qq + 2]);
                    r.w = r.w + (v[4 * qq + 3] * g.ascale + bcur[4 * qq + 3]);
                    *p = r;
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&tmY, rt, n0 + c0, px * 16, py * 8 + 2 * q);
                    bulk_commit();
                    if (pend >= 0) {
                        asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                        mbar_arrive(&rempty[pend]);
                    }
                }
                pend = s;
#pragma unroll
                for (int j = 0; j < 16; ++j) bcur[j] = bnext[j];
            }
            if (lane == 0 && pend >= 0) {
                bulk_wait_read();
                mbar_arrive(&rempty[pend]);
            }
            __syncwarp();
            tc_fence_before();
            mbar_arrive(&acc_empty[a]);
            if (!rok) break;
        }
    }

    if (warp >= LEAD && lane == 0) bulk_wait_all();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

// ------------------------------------------------------------------ host side

// cuTensorMapEncodeTiled, fetched from the driver through the runtime so the library
// does not link libcuda itself.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        HAT_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p) throw Error(3, "cuTensorMapEncodeTiled is unavailable");
        fn = (EncodeTiledFn)p;
    }
    return fn;
}

static CUtensorMap make_map(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                            const uint32_t* box, int rowbytes, bool h16 = false) {
    CUtensorMap m;
    uint32_t es[5] = {1, 1, 1, 1, 1};
    CUresult r = encode_fn()(&m, h16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank,
                             const_cast<void*>(base), dims,
                             strides_bytes, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             rowbytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                             : rowbytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                             : rowbytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(3, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return m;
}

CUtensorMap tensor_map(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                       const uint32_t* box, int rowbytes, bool h16) {
    return make_map(base, rank, dims, strides_bytes, box, rowbytes, h16);
}

static int num_sms() {
    static int n[64] = {0};
    int dev = 0;
    HAT_CUDA(cudaGetDevice(&dev));
    if (!n[dev & 63]) HAT_CUDA(cudaDeviceGetAttribute(&n[dev & 63], cudaDevAttrMultiProcessorCount, dev));
    return n[dev & 63];
}

// Dynamic shared memory at most: the 227 KB per CTA less the static arrays (channel
// sums 4 KB, staging tiles 17 KB, barriers) and some slack. Three stages of a 144-wide
// tile (3 x 68 KB) still fit.
static const long SMEM_CAP = 232448 - 22528;

// EK_RING: the stages, rounded to 1 KB, then the slots and the gate.
static size_t ring_smem(const UmmaArgs& g, const Epi& e) {
    const size_t st = ((size_t)g.stages * (2 * 128 * g.ckb + 2 * g.BN * g.ckb) + 1023) & ~(size_t)1023;
    return st + (size_t)RING_SLOTS * (e.cx ? 16384 : 8192) + (e.cx ? 4 * (size_t)g.BN * g.ntn : 0) + 1024;
}

// The dynamic shared memory a k_umma instantiation may take: the 227 KB a CTA can have,
// less its static shared memory (staging tiles and channel sums vary with the kind).
// The static size is a property of the compiled kernel (the same on every device), so it
// is read once; the shared-memory allowance is set on the current device at every call.
template <int MODE, int TERMS, int EK, bool H16>
static long umma_smem_cap() {
    static const long cap = [] {
        cudaFuncAttributes fa;
        HAT_CUDA(cudaFuncGetAttributes(&fa, k_umma<MODE, TERMS, EK, H16>));
        return 232448 - (long)fa.sharedSizeBytes;
    }();
    allow_dyn_smem(k_umma<MODE, TERMS, EK, H16>, (size_t)cap);
    return cap;
}

template <int MODE, int TERMS, int EK, bool H16>
static void launch_ek(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh, const CUtensorMap& bl,
                      const UmmaArgs& g0, const Epi& e, const CUtensorMap& ty, const QkvMaps& qm, cudaStream_t st) {
    const long cap = umma_smem_cap<MODE, TERMS, EK, H16>();
    UmmaArgs g = g0;
    const long per = 2L * 128 * g.ckb + 2L * g.BN * g.ckb;
    const long extra = EK == EK_RING ? (long)ring_smem(g, e) - (long)g.stages * per : 1024;
    g.stages = (int)std::min<long>(g.stages, (cap - extra) / per);
    if (g.stages < 1 || (EK == EK_RING && g.stages < 2))
        throw Error(1, "umma: the pipeline stages do not fit in shared memory");
    const size_t smem = EK == EK_RING ? ring_smem(g, e) : (size_t)g.stages * per + 1024;
    const long grid = std::min<long>(g.ntiles, num_sms());
    if (e.colsum && (g.N > 256 || EK == EK_QKV || EK == EK_RING))
        throw Error(1, "umma: channel sums are limited to 256 columns of the plain epilogues");
    constexpr int NT = umma_threads(MODE, EK);
    k_umma<MODE, TERMS, EK, H16><<<(unsigned)grid, NT, smem, st>>>(ah, al, bh, bl, g, e, ty, qm);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

// The epilogue kind for this launch (see EK_*).
static int pick_ek(const UmmaArgs& g, const Epi& e) {
    if (e.planar_out) return EK_GENERIC;
    if (e.shuffle == 2 && g.BN % 32 == 0 && g.N % g.BN == 0) return EK_SHUF2;
    if (e.shuffle) return EK_GENERIC;
    if (g.ldo % 4 == 0 && g.nstore % 4 == 0 && (!e.cx || g.N % 4 == 0)) return EK_STORE;
    return EK_GENERIC;
}

// The output's tensor map for the TMA-store epilogues (plain fp32 stores of EK_STORE) and
// the epilogue kind that goes with it: EK_TMA without a residual, EK_TMA_RES with one (the
// residual is added in the staging tile, where its loads are coalesced), or EK_STORE when
// the launch keeps the lanes' own stores. MODE 0: [M][ldo] rows; MODE 1: the [H][W][ldo]
// plane, a lane quarter's 32 rows being 2 pixel rows of 16.
template <int MODE>
static int store_map(const UmmaArgs& g, const Epi& e, CUtensorMap& ty, bool mlp = false) {
    if (pick_ek(g, e) != EK_STORE || g.y.lo || (reinterpret_cast<uintptr_t>(g.y.hi) & 15) || g.ldo % 4 ||
        g.nstore < 16)
        return EK_STORE;
    if (MODE == 0) {
        if (g.M < 32) return EK_STORE;
        uint64_t dims[2] = {(uint64_t)g.nstore, (uint64_t)g.M};
        uint64_t str[1] = {(uint64_t)g.ldo * 4};
        uint32_t box[2] = {16, 32};
        ty = make_map(g.y.hi, 2, dims, str, box, 64);
    } else {
        if (g.H < 2 || g.W < 16) return EK_STORE;
        uint64_t dims[3] = {(uint64_t)g.nstore, (uint64_t)g.W, (uint64_t)g.H};
        uint64_t str[2] = {(uint64_t)g.ldo * 4, (uint64_t)g.W * g.ldo * 4};
        uint32_t box[3] = {16, 16, 2};
        ty = make_map(g.y.hi, 3, dims, str, box, 64);
    }
    // With a residual only the linears gain (measured: proj faster; the fused MLP and the
    // residual convs slower than with the lanes' stores).
    if (e.res || e.cx) return MODE == 0 && !mlp ? EK_TMA_RES : EK_STORE;
    return EK_TMA;
}

template <int MODE, int TERMS, bool H16>
static void launch_k(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh, const CUtensorMap& bl,
                     UmmaArgs g, const Epi& e, cudaStream_t st) {
    CUtensorMap ty = ah;  // unused unless a TMA-store epilogue runs
    QkvMaps qm{ah, ah, ah, ah};
    if constexpr (MODE == 0 && TERMS == 3 && H16) {
      if (e.qkv_split) {
        // the qkv attention layout (see Epi::qkv_split)
        const int c = g.N / 3;
        if (g.N % 48 || g.M % 8 || (reinterpret_cast<uintptr_t>(e.qkv_split) & 15))
            throw Error(1, "umma_linear: the qkv attention layout needs N a multiple of 48 and M of 8");
        const __half* qkh = reinterpret_cast<const __half*>(e.qkv_split);
        const __half* qkl = qkh + g.M * 2 * c;
        const __half* vth = qkl + g.M * 2 * c;
        const __half* vtl = vth + (long)c * g.M;
        uint64_t dqk[2] = {(uint64_t)(2 * c), (uint64_t)g.M}, sqk[1] = {(uint64_t)(2 * c) * 2};
        uint32_t bqk[2] = {16, 32};
        qm.qkh = make_map(qkh, 2, dqk, sqk, bqk, 32, true);
        qm.qkl = make_map(qkl, 2, dqk, sqk, bqk, 32, true);
        uint64_t dvt[2] = {(uint64_t)g.M, (uint64_t)c}, svt[1] = {(uint64_t)g.M * 2};
        uint32_t bvt[2] = {32, 16};
        qm.vth = make_map(vth, 2, dvt, svt, bvt, 0, true);
        qm.vtl = make_map(vtl, 2, dvt, svt, bvt, 0, true);
        g.tma_st = 1;
        launch_ek<MODE, TERMS, EK_QKV, H16>(ah, al, bh, bl, g, e, ty, qm, st);
        return;
      }
    }
    if (e.qkv_split) throw Error(1, "umma_linear: the qkv attention layout is for fp16 parity mode");
    if constexpr (MODE == 0) {
        // A linear with a residual and a plain fp32 output: the residual stream by TMA.
        auto al16 = [](const void* p) { return !(reinterpret_cast<uintptr_t>(p) & 15); };
        const bool ring = e.res && !e.colsum && e.act == ACT_NONE && pick_ek(g, e) == EK_STORE && !g.y.lo &&
                          !g.y.h16 && al16(g.y.hi) && al16(e.res) && g.ldo % 4 == 0 && g.nstore >= 16 &&
                          g.M >= 128 && g.BN % 16 == 0 && (!e.cx || (al16(e.cx) && e.gate));
        if (ring) {
            UmmaArgs gr = g;
            const long per = 2L * 128 * g.ckb + 2L * g.BN * g.ckb;
            const long extra = (long)RING_SLOTS * (e.cx ? 16384 : 8192) + (e.cx ? 4L * g.BN * g.ntn : 0) + 2048;
            const long cap = umma_smem_cap<MODE, TERMS, EK_RING, H16>();
            gr.stages = (int)std::min<long>(g.stages, (cap - extra) / per);
            if (gr.stages >= 2) {
                uint64_t dims[2] = {(uint64_t)g.nstore, (uint64_t)g.M};
                uint64_t str[1] = {(uint64_t)g.ldo * 4};
                uint32_t ybox[2] = {16, 32}, rbox[2] = {16, 128};
                ty = make_map(g.y.hi, 2, dims, str, ybox, 64);
                qm.qkh = make_map(e.res, 2, dims, str, rbox, 64);
                if (e.cx) qm.qkl = make_map(e.cx, 2, dims, str, rbox, 64);
                gr.tma_st = 1;
                if (ring_smem(gr, e) > (size_t)cap) throw Error(1, "umma_linear: residual ring does not fit");
                launch_ek<MODE, TERMS, EK_RING, H16>(ah, al, bh, bl, gr, e, ty, qm, st);
                return;
            }
        }
    }
    const int sk = store_map<MODE>(g, e, ty);
    g.tma_st = sk != EK_STORE;
    switch (sk != EK_STORE ? sk : pick_ek(g, e)) {
        case EK_TMA: launch_ek<MODE, TERMS, EK_TMA, H16>(ah, al, bh, bl, g, e, ty, qm, st); break;
        case EK_TMA_RES: launch_ek<MODE, TERMS, EK_TMA_RES, H16>(ah, al, bh, bl, g, e, ty, qm, st); break;
        case EK_STORE: launch_ek<MODE, TERMS, EK_STORE, H16>(ah, al, bh, bl, g, e, ty, qm, st); break;
        case EK_SHUF2: launch_ek<MODE, TERMS, EK_SHUF2, H16>(ah, al, bh, bl, g, e, ty, qm, st); break;
        default: launch_ek<MODE, TERMS, EK_GENERIC, H16>(ah, al, bh, bl, g, e, ty, qm, st); break;
    }
}
// parity on fp16 pairs, parity on tf32 pairs, or fast (tf32, one term)
template <int MODE>
static void launch_mode(bool three, bool h16, const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh,
                        const CUtensorMap& bl, const UmmaArgs& g, const Epi& e, cudaStream_t st) {
    if (three && h16)
        launch_k<MODE, 3, true>(ah, al, bh, bl, g, e, st);
    else if (three)
        launch_k<MODE, 3, false>(ah, al, bh, bl, g, e, st);
    else
        launch_k<MODE, 1, false>(ah, al, bh, bl, g, e, st);
}

static long colsum_rows(const UmmaArgs& g) { return std::min<long>(g.ntiles, num_sms()) * 4; }

static int pick_stages(int BN, int ckb) {
    const long per = 2L * 128 * ckb + 2L * BN * ckb;
    const long budget = SMEM_CAP - 1024;
    return (int)std::max(1L, std::min(6L, budget / per));
}

static void fill_common(UmmaArgs& g, const GemmW& w, Dst y, const Epi& e, int* err) {
    g.N = w.n;
    g.BN = w.bn;
    g.ntn = w.n_pad / w.bn;
    g.y = y;
    g.ldo = e.ldo ? e.ldo : w.n;
    g.nstore = e.ldo ? e.ldo : w.n;
    g.err = err;
}

long umma_linear(int mode, Opnd x, const GemmW& w, Dst y, long m, const Epi& e, int* err, cudaStream_t st) {
    const int ckb = 128;
    const bool three = mode == 0;
    if (three && !x.lo) throw Error(1, "umma_linear: fp32-parity mode needs a split operand");
    const bool h16 = three && w.h16;
    if (three && x.h16 != w.h16) throw Error(1, "umma_linear: operand and weight split kinds differ");
    const int es = h16 ? 2 : 4, kel = ckb / es, kstep = 32 / es;  // elements per k-block / k-step
    uint64_t adims[2] = {(uint64_t)w.k, (uint64_t)m};
    uint64_t astr[1] = {(uint64_t)w.k * es};
    uint32_t abox[2] = {(uint32_t)kel, 128};
    CUtensorMap tah = make_map(x.hi, 2, adims, astr, abox, ckb, h16);
    CUtensorMap tal = make_map(three ? x.lo : x.hi, 2, adims, astr, abox, ckb, h16);
    uint64_t bdims[2] = {(uint64_t)w.k_pad, (uint64_t)w.n_pad};
    uint64_t bstr[1] = {(uint64_t)w.k_pad * es};
    uint32_t bbox[2] = {(uint32_t)kel, (uint32_t)w.bn};
    CUtensorMap tbh = make_map(w.hi, 2, bdims, bstr, bbox, ckb, h16);
    CUtensorMap tbl = make_map(three ? w.lo : w.hi, 2, bdims, bstr, bbox, ckb, h16);
    UmmaArgs g{};
    fill_common(g, w, y, e, err);
    g.M = m;
    g.KB = (w.k + kel - 1) / kel;  // k-blocks holding real K (the rest of k_pad is zeros)
    g.klast = (w.k - (g.KB - 1) * kel + kstep - 1) / kstep;
    g.ascale = h16 ? w.scale : 1.f;
    g.ckb = ckb;
    g.stages = pick_stages(w.bn, ckb);
    g.mtiles = (m + 127) / 128;
    g.ntiles = g.mtiles * g.ntn;
    launch_mode<0>(three, h16, tah, tal, tbh, tbl, g, e, st);
    return colsum_rows(g);  // colsum: one partial row per (CTA, epilogue warp)
}

long umma_conv3x3(int mode, Opnd x, const GemmW& w, Dst y, int hgt, int wid, const Epi& e, int* err,
                  cudaStream_t st) {
    const bool three = mode == 0;
    if (three && !x.lo) throw Error(1, "umma_conv3x3: fp32-parity mode needs a split operand");
    const bool h16 = three && w.h16;
    if (three && x.h16 != w.h16) throw Error(1, "umma_conv3x3: operand and weight split kinds differ");
    const int ckb = w.ckb;
    const int es = h16 ? 2 : 4, cke = ckb / es, kstep = 32 / es;  // channels per chunk / per k-step
    uint64_t adims[3] = {(uint64_t)w.cin_plane, (uint64_t)wid, (uint64_t)hgt};
    uint64_t astr[2] = {(uint64_t)w.cin_plane * es, (uint64_t)wid * w.cin_plane * es};
    uint32_t abox[3] = {(uint32_t)cke, 16, 8};
    CUtensorMap tah = make_map(x.hi, 3, adims, astr, abox, ckb, h16);
    CUtensorMap tal = make_map(three ? x.lo : x.hi, 3, adims, astr, abox, ckb, h16);
    uint64_t bdims[2] = {(uint64_t)w.k_pad, (uint64_t)w.n_pad};
    uint64_t bstr[1] = {(uint64_t)w.k_pad * es};
    uint32_t bbox[2] = {(uint32_t)cke, (uint32_t)w.bn};
    CUtensorMap tbh = make_map(w.hi, 2, bdims, bstr, bbox, ckb, h16);
    CUtensorMap tbl = make_map(three ? w.lo : w.hi, 2, bdims, bstr, bbox, ckb, h16);
    UmmaArgs g{};
    fill_common(g, w, y, e, err);
    g.M = (long)hgt * wid;
    g.cchunks = (w.cin + cke - 1) / cke;  // chunks holding real channels (cinp - cin are zeros)
    g.klast = (w.cin - (g.cchunks - 1) * cke + kstep - 1) / kstep;
    g.ascale = h16 ? w.scale : 1.f;
    g.KB = 9 * g.cchunks;
    g.ckb = ckb;
    g.stages = pick_stages(w.bn, ckb);
    g.H = hgt;
    g.W = wid;
    g.tx = wid / 16;
    const int ylo = e.y_hi > 0 ? e.y_lo : 0, yhi = e.y_hi > 0 ? e.y_hi : hgt;
    if (ylo % 8 || yhi % 8 || ylo < 0 || yhi > hgt || ylo >= yhi) throw Error(1, "umma_conv3x3: bad output row range");
    g.ty0 = ylo / 8;
    g.mtiles = (long)((yhi - ylo) / 8) * g.tx;
    g.ntiles = g.mtiles * g.ntn;
    launch_mode<1>(three, h16, tah, tal, tbh, tbl, g, e, st);
    return colsum_rows(g);
}


bool umma_proj_cab_ok(const GemmW& wp, const GemmW& w2) {
    if (!wp.umma || !w2.umma || wp.conv || !w2.conv || wp.h16 != w2.h16) return false;
    // the kernel's conv chunk (64-byte rows at most) must tile the weight's K layout per tap
    const int es = wp.h16 ? 2 : 4, cke = std::min(w2.ckb, 64) / es;
    return wp.n == w2.n && wp.bn == w2.bn && wp.n_pad == w2.n_pad && wp.bn % 16 == 0 && wp.bn <= 256 &&
           wp.n % 4 == 0 && (w2.ckb == 128 || w2.ckb == 32) && w2.cinp == (w2.cin + cke - 1) / cke * cke &&
           w2.cin_plane % (16 / es) == 0;
}

template <int TERMS, bool H16>
static void launch_proj_cab(const CUtensorMap* m, const ProjCabArgs& g0, cudaStream_t st) {
    static const long cap = [] {
        cudaFuncAttributes fa;
        HAT_CUDA(cudaFuncGetAttributes(&fa, k_proj_cab<TERMS, H16>));
        return 232448 - (long)fa.sharedSizeBytes;
    }();
    allow_dyn_smem(k_proj_cab<TERMS, H16>, (size_t)cap);
    ProjCabArgs g = g0;
    const long per = 2L * 128 * 64 + 2L * g.BN * 64;
    g.slots = PC_SLOTS;
    g.stages = (int)std::min<long>(6, (cap - 1024 - (long)g.slots * 8192) / per);
    if (g.stages < 2) throw Error(1, "umma_proj_cab: the pipeline does not fit in shared memory");
    const size_t smem = (size_t)g.stages * per + (size_t)g.slots * 8192 + 1024;
    const long grid = std::min<long>(g.ntiles, num_sms());
    k_proj_cab<TERMS, H16><<<(unsigned)grid, 32 * 11, smem, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7],
                                                                    m[8], m[9], g);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

long umma_proj_cab(int mode, Opnd attn, const GemmW& wp, Opnd cmid, int cm_ld, int cm_rows, int cm_lo,
                   const GemmW& w2, const float* w2hi, const float* w2lo, const float* bias, const float* res,
                   float* out, int rows, int wid, int y_lo, int y_hi, int* err, cudaStream_t st) {
    if (!umma_proj_cab_ok(wp, w2)) throw Error(1, "umma_proj_cab: weights not in the fused layout");
    const bool three = mode == 0;
    if (three && (!attn.lo || !cmid.lo)) throw Error(1, "umma_proj_cab: fp32-parity mode needs split operands");
    const bool h16 = three && wp.h16;
    if (three && (attn.h16 != h16 || cmid.h16 != h16)) throw Error(1, "umma_proj_cab: operand split kinds differ");
    if (wid % 16 || y_lo % 8 || y_hi % 8 || y_lo < 0 || y_hi > rows || y_lo >= y_hi || cm_lo < 0 ||
        cm_lo + cm_rows > rows || cm_ld < w2.cin)
        throw Error(1, "umma_proj_cab: bad geometry");
    auto a16 = [](const void* p) { return !(reinterpret_cast<uintptr_t>(p) & 15); };
    if (!a16(res) || !a16(out) || !a16(attn.hi) || !a16(cmid.hi) || (three && (!a16(attn.lo) || !a16(cmid.lo))))
        throw Error(1, "umma_proj_cab: planes must be 16-byte aligned");
    // 64-byte k-block rows for both parts (32 fp16 or 16 tf32 elements); the conv's chunk
    // of a tap is its weight layout's chunk, or half of it for 128-byte chunks.
    const int ckb_b = std::min(w2.ckb, 64);
    const int es = h16 ? 2 : 4, kel = 64 / es, kstep = 32 / es, cke = ckb_b / es;
    const int c = wp.k, N = wp.n;
    CUtensorMap m[10];
    {   // attention output [rows][wid][c], patches of 16 x 8 pixels, 128-byte k-block rows
        uint64_t d[3] = {(uint64_t)c, (uint64_t)wid, (uint64_t)rows};
        uint64_t s2[2] = {(uint64_t)c * es, (uint64_t)wid * c * es};
        uint32_t b[3] = {(uint32_t)kel, 16, 8};
        m[0] = make_map(attn.hi, 3, d, s2, b, 64, h16);
        m[1] = make_map(three ? attn.lo : attn.hi, 3, d, s2, b, 64, h16);
    }
    {   // proj weight [n_pad][k_pad]
        uint64_t d[2] = {(uint64_t)wp.k_pad, (uint64_t)wp.n_pad}, s1[1] = {(uint64_t)wp.k_pad * es};
        uint32_t b[2] = {(uint32_t)kel, (uint32_t)wp.bn};
        m[2] = make_map(wp.hi, 2, d, s1, b, 64, h16);
        m[3] = make_map(three ? wp.lo : wp.hi, 2, d, s1, b, 64, h16);
    }
    {   // the cmid view [cm_rows][wid][cm_ld]
        uint64_t d[3] = {(uint64_t)cm_ld, (uint64_t)wid, (uint64_t)cm_rows};
        uint64_t s2[2] = {(uint64_t)cm_ld * es, (uint64_t)wid * cm_ld * es};
        uint32_t b[3] = {(uint32_t)cke, 16, 8};
        m[4] = make_map(cmid.hi, 3, d, s2, b, ckb_b, h16);
        m[5] = make_map(three ? cmid.lo : cmid.hi, 3, d, s2, b, ckb_b, h16);
    }
    {   // the folded conv weight [n_pad][9 * cinp]
        uint64_t d[2] = {(uint64_t)w2.k_pad, (uint64_t)w2.n_pad}, s1[1] = {(uint64_t)w2.k_pad * es};
        uint32_t b[2] = {(uint32_t)cke, (uint32_t)w2.bn};
        m[6] = make_map(w2hi, 2, d, s1, b, ckb_b, h16);
        m[7] = make_map(three ? w2lo : w2hi, 2, d, s1, b, ckb_b, h16);
    }
    {   // residual (patches, 16-column chunks) and output (two pixel rows per warp), fp32
        uint64_t d[3] = {(uint64_t)N, (uint64_t)wid, (uint64_t)rows};
        uint64_t s2[2] = {(uint64_t)N * 4, (uint64_t)wid * N * 4};
        uint32_t br[3] = {16, 16, 8}, by[3] = {16, 16, 2};
        m[8] = make_map(res, 3, d, s2, br, 64);
        m[9] = make_map(out, 3, d, s2, by, 64);
    }
    ProjCabArgs g{};
    g.N = N;
    g.BN = wp.bn;
    g.ntn = wp.n_pad / wp.bn;
    g.KBa = (c + kel - 1) / kel;
    g.klast_a = (c - (g.KBa - 1) * kel + kstep - 1) / kstep;
    g.ckb_b = ckb_b;
    g.cchunks_b = (w2.cin + cke - 1) / cke;
    g.klast_b = (w2.cin - (g.cchunks_b - 1) * cke + kstep - 1) / kstep;
    g.tx = wid / 16;
    g.ty0 = y_lo / 8;
    g.yoff_b = -cm_lo;
    g.ntiles = (long)((y_hi - y_lo) / 8) * g.tx * g.ntn;
    g.ascale = h16 ? wp.scale : 1.f;
    g.bias = bias;
    g.err = err;
    if (three && h16)
        launch_proj_cab<3, true>(m, g, st);
    else if (three)
        launch_proj_cab<3, false>(m, g, st);
    else
        launch_proj_cab<1, false>(m, g, st);
    return 0;
}

}  // namespace hat

namespace hat {

bool umma_mlp_ok(const GemmW& w1, const GemmW& w2) {
    return w1.umma && w2.umma && !w1.conv && !w2.conv && w1.h16 == w2.h16 && w2.n == w1.k && w2.k == w1.n &&
           w1.n_pad % MLP_HC == 0 && w2.k_pad >= w1.n_pad && w1.n_pad <= MLP_MAXH &&
           w2.n_pad % 16 == 0 && w2.n_pad + 3 * MLP_HC <= 512 && w1.k % (w1.h16 ? 8 : 4) == 0;
}

long umma_mlp(int mode, Opnd x, const GemmW& w1, const float* b1, const GemmW& w2, const float* b2, const float* res,
              Dst y, long m, int* err, cudaStream_t st) {
    if (!umma_mlp_ok(w1, w2)) throw Error(1, "umma_mlp: weights not in the fused-MLP layout");
    const bool three = mode == 0;
    if (three && !x.lo) throw Error(1, "umma_mlp: fp32-parity mode needs a split operand");
    const bool h16 = three && w1.h16;
    if (three && x.h16 != w1.h16) throw Error(1, "umma_mlp: operand and weight split kinds differ");
    const int es = h16 ? 2 : 4, kel = 128 / es, kstep = 32 / es;
    const int C = w1.k;
    uint64_t adims[2] = {(uint64_t)C, (uint64_t)m};
    uint64_t astr[1] = {(uint64_t)C * es};
    uint32_t abox[2] = {(uint32_t)kel, 128};
    CUtensorMap tah = make_map(x.hi, 2, adims, astr, abox, 128, h16);
    CUtensorMap tal = make_map(three ? x.lo : x.hi, 2, adims, astr, abox, 128, h16);
    uint64_t d1[2] = {(uint64_t)w1.k_pad, (uint64_t)w1.n_pad};
    uint64_t s1[1] = {(uint64_t)w1.k_pad * es};
    uint32_t b1box[2] = {(uint32_t)kel, (uint32_t)MLP_HC};
    CUtensorMap t1h = make_map(w1.hi, 2, d1, s1, b1box, 128, h16);
    CUtensorMap t1l = make_map(three ? w1.lo : w1.hi, 2, d1, s1, b1box, 128, h16);
    uint64_t d2[2] = {(uint64_t)w2.k_pad, (uint64_t)w2.n_pad};
    uint64_t s2[1] = {(uint64_t)w2.k_pad * es};
    uint32_t b2box[2] = {(uint32_t)kel, (uint32_t)w2.n_pad};
    CUtensorMap t2h = make_map(w2.hi, 2, d2, s2, b2box, 128, h16);
    CUtensorMap t2l = make_map(three ? w2.lo : w2.hi, 2, d2, s2, b2box, 128, h16);

    MlpArgs g{};
    g.C = C;
    g.HID = w1.n;
    g.NCH = w1.n_pad / MLP_HC;
    g.CP = w2.n_pad;
    g.KB1 = (C + kel - 1) / kel;
    g.klast1 = (C - (g.KB1 - 1) * kel + kstep - 1) / kstep;
    g.s1 = h16 ? w1.scale : 1.f;
    g.mtiles = (m + 127) / 128;
    g.b1 = b1;
    const long st_bytes = std::max(2L * 128 * 128 + 2L * MLP_HC * 128, 2L * g.CP * 128);
    g.stages = (int)std::max(2L, std::min(6L, (SMEM_CAP - 1024) / st_bytes));
    // The residual-tile epilogue (MLP_RT): an fp32 output with a residual, both 16-byte
    // aligned, whole 128-row tiles of the tensor maps, and two pipeline stages beside the
    // CP x 128 fp32 tile.
    const long rt_bytes = (long)g.CP * 512;
    const bool rt = res && !y.lo && !y.h16 && !(reinterpret_cast<uintptr_t>(y.hi) & 15) &&
                    !(reinterpret_cast<uintptr_t>(res) & 15) && C % 4 == 0 && C >= 16 && m >= 128 &&
                    g.CP % 16 == 0 && 2 * st_bytes + rt_bytes + 1024 <= SMEM_CAP;
    if (rt) g.stages = 2;
    UmmaArgs& u = g.st;
    u.M = m;
    u.N = C;
    u.BN = g.CP;
    u.ntn = 1;
    u.y = y;
    u.ldo = C;
    u.nstore = C;
    u.err = err;
    u.mtiles = g.mtiles;
    u.ntiles = g.mtiles;
    u.ascale = h16 ? w2.scale : 1.f;
    Epi e;
    e.bias = b2;
    e.res = res;
    if (C % 4) throw Error(1, "umma_mlp: the width must be a multiple of 4");
    const size_t smem = (size_t)g.stages * st_bytes + (rt ? rt_bytes : 0) + 1024;
    CUtensorMap ty = tah;  // the output's tensor map when the final store goes by TMA
    CUtensorMap tr = tah;  // MLP_RT: the residual's
    int skx;
    if (rt) {
        uint64_t dims[2] = {(uint64_t)C, (uint64_t)m};
        uint64_t str[1] = {(uint64_t)C * 4};
        uint32_t ybox[2] = {16, 32}, rbox[2] = {16, 128};
        ty = make_map(y.hi, 2, dims, str, ybox, 64);
        tr = make_map(res, 2, dims, str, rbox, 64);
        u.tma_st = true;
        skx = 3;
    } else {
        const int sk = store_map<0>(u, e, ty, true);
        u.tma_st = sk != EK_STORE;
        skx = sk == EK_TMA ? 1 : sk == EK_TMA_RES ? 2 : 0;
    }
    const int which = (h16 ? 2 : three ? 0 : 1) * 4 + skx;
    using KFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, MlpArgs, Epi,
                         CUtensorMap, CUtensorMap);
    const KFn table[12] = {k_mlp<3, false, 0>, k_mlp<3, false, 1>, k_mlp<3, false, 2>, k_mlp<3, false, MLP_RT>,
                           k_mlp<1, false, 0>, k_mlp<1, false, 1>, k_mlp<1, false, 2>, k_mlp<1, false, MLP_RT>,
                           k_mlp<3, true, 0>,  k_mlp<3, true, 1>,  k_mlp<3, true, 2>,  k_mlp<3, true, MLP_RT>};
    const KFn kern = table[which];
    allow_dyn_smem(kern, (size_t)SMEM_CAP);
    const long grid = std::min<long>(g.mtiles, num_sms());
    const int nt = 64 + 32 * mlp_epi_warps(h16, skx == 3 ? MLP_RT : skx);
    kern<<<(unsigned)grid, nt, smem, st>>>(tah, tal, t1h, t1l, t2h, t2l, g, e, ty, tr);
    HAT_CUDA(cudaGetLastError());
    count_launch();
    return 0;
}

}  // namespace hat
