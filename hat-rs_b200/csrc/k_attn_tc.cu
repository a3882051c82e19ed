// Tensor-core window attention for sm_100a: the HAB's (shifted) 16x16 window attention
// and the OCAB's 16x16-query / 24x24-key overlapping attention (hat_arch.py:165-196,
// 392-438), one fused kernel per launch:
//
//   S = (q*scale) K^T + bias (+ shift mask)      tcgen05.mma, S in tensor memory
//   P = exp(S - m), row sums                      CUDA cores, one thread per query row
//   O += P V                                      tcgen05.mma, P and O in tensor memory
//
// Work item = (window, head, half of the window's 256 queries); 128 query rows per
// item, keys streamed in blocks of 32 (8 blocks for 256 keys, 18 for 576). Every
// operand is split into fp16 hi/lo halves (hi = fp16(x), lo = fp16(x - hi): 22
// significant bits, the same as a tf32 pair), and both products use the 3-term split
// (A_lo.B_hi + A_hi.B_lo + A_hi.B_hi) of `tcgen05.mma.kind::f16` with fp32 accumulation
// in fp32-parity mode; fast mode issues the single A_hi.B_hi. A kind::f16 MMA takes 16
// elements of K for the cost of 8 in kind::tf32, so QK^T (head dim 24 or 30, padded to
// 32) is 2 k-steps and PV over a 32-key block 2 k-steps. Values below fp16's normal
// range keep an absolute error of at most 2^-25 per element; |q|, |k|, |v| of 65504 or
// more would overflow, so the loaders check the range and stop the kernel with an
// error code instead.
//
// Softmax: P is written back into tensor memory as packed fp16 pairs (P_hi in the first
// 16 of the block's 32 S columns, P_lo in the other 16) and the PV product reads its A
// operand from there. O accumulates in tensor memory across the item's key blocks. Each
// row keeps a reference max m: P = exp(S - m) with the row sum l accumulated against the
// same m, so O / l is exact whatever m is. m is the first block's max and moves only
// when a later block's max exceeds it by more than RESCALE_LOG2 (in log2 units, so every
// P stays below 2^RESCALE_LOG2); then the row's O in tensor memory and l are scaled by
// exp(m_old - m_new) first. With RESCALE_LOG2 = 8 that is rare, so O is read once per
// item, not once per key block. P and l carry a factor 2^P_SHIFT (P below 2^14), which
// keeps more of P's split above fp16's subnormals and cancels in O / l. S, the bias
// table and the shift mask are in log2 units (q is scaled by scale * log2(e)), so P is
// one ex2 per key.
//
// The window partition, the cyclic roll, the nn.Unfold of the keys with its zero
// padding, the relative-position bias gather and the shift mask are address
// arithmetic: nothing is materialised. The bias table is staged in shared memory with
// rows 48 floats apart, which puts the two half-warps (two query rows of the window)
// on disjoint banks.
//
// Warp roles: 0 MMA issuer + TMEM owner, 1-4 softmax (TMEM lane quarters 1,2,3,0), then the
// loaders: 4 warps (gathering, splitting loaders, or copies on the pre-split layout for the
// OCAB; 288 threads, two CTAs per SM) or, for the window attention on the pre-split layout,
// 2 warps of 16-byte copies (224 threads, three CTAs per SM).
// Every mbarrier wait is bounded; on expiry the kernel records an error code, all roles
// leave, and TMEM is released.
#include <cuda_fp16.h>

#include <cstring>

#include "common.cuh"
#include "umma.cuh"

namespace hat {

namespace {

// H2 (window attention on the pre-split layout): a work item is a whole window of one head,
// both 128-query halves, so its keys and values are loaded once for 256 queries; eight softmax
// warps (four per half, each half's S, P and O in tensor memory of its own), one loader warp
// (TMA, and copies for the windows that wrap around the plane), 320 threads, two CTAs per SM
// (96 registers a thread). Otherwise a work item is one
// half: four softmax warps, four loader warps, 288 threads, two CTAs per SM (96 registers).
template <bool H2>
struct AttnShape {
    static constexpr int halves = H2 ? 2 : 1;           // query halves per work item
    static constexpr int loaders = H2 ? 1 : 4;          // loader warps
    static constexpr int softmax = 4 * halves;          // softmax warps
    static constexpr int threads = 32 * (1 + softmax + loaders);
    static constexpr int ctas = 2;                      // CTAs per SM
};
constexpr int KBLK = 32;     // keys per block
constexpr int MT = 128;      // query rows per work item
constexpr int KVS = 4;       // K/V pipeline stages
// The window attention's table is kept as four copies, copy c shifted left by c floats,
// rows SA_TS floats apart and copies SA_CS floats apart: the 16 biases a query meets in one
// key row are then four aligned 16-byte loads from copy (qx mod 4), and SA_CS = 8 mod 32
// puts the eight lanes of a load phase on distinct 16-byte bank groups.
constexpr int SA_TS = 32, SA_CS = 1000;
// The OCAB's 39 x 39 table the same way: rows OCA_TS apart, copies OCA_CS (= 8 mod 32) apart;
// a block's 32 keys are four runs of 8 keys within one key row, two aligned loads each.
constexpr int OCA_TS = 40, OCA_CS = 1576;
template <bool OCA>
constexpr int tab_floats() { return OCA ? 4 * OCA_CS : 4 * SA_CS; }
constexpr float RESCALE_LOG2 = 8.f;
constexpr float P_SHIFT = 6.f;
constexpr float F16_LIMIT = 65504.f;  // the largest finite fp16
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
// kind::f16 with fp16 A and B (format 0), f32 accumulate, M = 128, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_h(int n) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
// D (tmem) (+)= A (smem) . B (smem)
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// D (tmem) (+)= A (tmem: lane = row, column j = the fp16 pair k = 2j, 2j+1) . B (smem)
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(d), "r"(a), "l"(b), "r"(idesc), "r"(acc));
}
// 2^x by the PTX ex2.approx instruction (relative error about 2^-22; subnormal results
// flush to zero, which P never needs).
// max of three (sm_100's three-input max)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
constexpr float L2E = 1.4426950408889634f;  // log2(e): S, the bias and the mask in log2 units
__device__ __forceinline__ void commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su(b))
                 : "memory");
}
// 32 consecutive columns of this warp's 32 TMEM lanes (one row per thread).
__device__ __forceinline__ void tld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tst32(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
          "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
          "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
          "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
          "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
          "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
          "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
          "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
          "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
          "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
          "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tst16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tst_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TMA tile loads into shared memory (no multicast), completing on `bar`'s transaction count.
__device__ __forceinline__ void tma3(uint32_t dst, const CUtensorMap* m, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(dst), "l"((uint64_t)m), "r"(c0), "r"(c1), "r"(c2), "r"(su(bar))
        : "memory");
}
__device__ __forceinline__ void tma4(uint32_t dst, const CUtensorMap* m, int c0, int c1, int c2, int c3, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];"
        ::"r"(dst), "l"((uint64_t)m), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(su(bar))
        : "memory");
}
__device__ __forceinline__ void tma4_store(const CUtensorMap* m, uint32_t src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];"
                 ::"l"((uint64_t)m), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(src)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// named barrier 1 or 2 (a query half's softmax warps) over 128 threads
__device__ __forceinline__ void half_sync(int hh) {
    if (hh == 0)
        asm volatile("bar.sync 1, 128;" ::: "memory");
    else
        asm volatile("bar.sync 2, 128;" ::: "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su(b)), "r"(bytes) : "memory");
}

// Byte offset of the 16-byte chunk q (0 or 1) of row `row` in a SWIZZLE_32B tile of
// 32-byte rows (16 fp16 values of K per row).
__device__ __forceinline__ uint32_t off_sw32(int row, int q) { return row * 32 + (((q ^ (row >> 2)) & 1) << 4); }

__device__ __forceinline__ int band3(int v, int n, int shift) { return v < n - 16 ? 0 : (v < n - shift ? 1 : 2); }

}  // namespace

// Where a launch's windows lie in its plane (the whole padded plane, or one strip of it
// with halo rows). Window (wy, wx), wy < nwy, holds plane rows (oy + 16wy + y + sy) mod
// rows and columns (16wx + x + sx) mod wp for y, x < 16 (SA), or the 16x16 queries at
// (oy + 16wy + y, 16wx + x) with the 24x24 keys 4 rows / columns further out (OCAB,
// zero outside padded rows 0..ghp-1, local row i being padded row gy0 + i). The shift
// mask (mshift > 0) labels a query or key by the rolled-frame position
// ((yr0 + 16wy + y) mod ghp, 16wx + x) against the bands of the ghp x wp plane. Only
// queries on plane rows [olo, ohi) are written.
struct AttnGeom {
    int rows, wp, nwy, oy, sy, sx, ghp, yr0, gy0, olo, ohi, mshift;
};

// D: head dim (24 or 30); OCA: overlapping attention; TERMS: 3 (parity) or 1 (fast);
// PRE: q, k and v arrive as fp16 pairs in the qkv linear's attention layout (q|k hi and lo
// [P][2c], v^T hi and lo [c][P], q already scaled by scale * log2(e); see Epi::qkv_split),
// so the loaders only copy 16-byte pieces (window attention, D = 24, parity mode).
template <int D, bool OCA, int TERMS, bool PRE>
__global__ void __launch_bounds__(AttnShape<PRE && !OCA>::threads, AttnShape<PRE && !OCA>::ctas)
    k_attn_tc(const float* __restrict__ qkv, const float* __restrict__ table, Dst out, const AttnGeom gm, int c,
              int heads, float scale, long items, int* err, const __grid_constant__ CUtensorMap tqh,
              const __grid_constant__ CUtensorMap tql, const __grid_constant__ CUtensorMap tkh,
              const __grid_constant__ CUtensorMap tkl, const __grid_constant__ CUtensorMap tvh,
              const __grid_constant__ CUtensorMap tvl, const __grid_constant__ CUtensorMap toh,
              const __grid_constant__ CUtensorMap tol) {
    const int wp = gm.wp;
    constexpr int KH = (D + 15) / 16;               // k-steps of the QK^T product (16 fp16 each)
    constexpr int NK = OCA ? 576 : 256;             // keys per window
    constexpr int NBLK = NK / KBLK;
    constexpr int TR = OCA ? 39 : 31;               // bias-table rows (and columns)
    constexpr int TW = OCA ? 39 : 31;               // the checkpoint table's row length
    constexpr uint32_t Q_BYTES = KH * 4096;         // 128 rows x 32 B per k-step
    constexpr uint32_t K_BYTES = KH * 1024;         // 32 keys x 32 B per k-step
    constexpr uint32_t V_BYTES = 2 * 1024;          // V^T: 32 features x 32 B per 16-key k-step
    constexpr uint32_t KV_BYTES = 2 * K_BYTES + 2 * V_BYTES;
    using Shape = AttnShape<PRE && !OCA>;
    constexpr int HV = Shape::halves;               // query halves of a work item
    // Q buffers. One: a second (the next item's Q loading while this item's last key blocks
    // run) measured no faster with three K/V stages, and with four it left room for only one
    // CTA per SM (12.3 ms per pass -> 18.6 ms).
    constexpr int QB = 1;
    constexpr uint32_t Q_REGION = HV * 2 * Q_BYTES;  // one buffer: every half, hi and lo
    constexpr uint32_t OFF_KV = QB * Q_REGION;
    constexpr uint32_t OFF_TAB = OFF_KV + KVS * KV_BYTES;
    // The window kernel's output staging: per half, 128 rows of 24 fp16 (48 bytes), hi then lo,
    // stored by TMA (see the softmax's output).
    constexpr uint32_t OFF_OST = (OFF_TAB + tab_floats<OCA>() * 4 + 1023) & ~1023u;
    constexpr uint32_t OST_BYTES = 128 * 48;

    // TMEM columns: half h's S blocks at 64h and 64h + 32 (fp32); once read, a block's first
    // 16 columns hold P_hi and the next 16 P_lo (fp16 pairs); half h's O (per item parity)
    // at 64 HV + 64h and 64 HV + 64h + 32.
    constexpr uint32_t T_PLO = 16, T_O = 64 * HV;
    constexpr uint32_t TMEM_COLS = 128 * HV;

    extern __shared__ __align__(1024) uint8_t raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
    float* tab = reinterpret_cast<float*>(sm + OFF_TAB);
    __shared__ uint64_t q_full[QB], q_empty[QB], kv_full[KVS], kv_empty[KVS], s_full[HV][2], p_full[HV][2],
        o_done[HV], o_free[HV][2], drain;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = (int)(blockIdx.x % heads);
    const int nx = wp / 16;
    const long c3 = 3L * c;

    // Bias table of this head (in log2 units), as four copies, copy c shifted left by c
    // floats. SA: tab_c[r*SA_TS + s - c] = table[r*31 + s], the bias of (qy - ky + 15,
    // qx - kx + 15). OCAB: tab_c[r*OCA_TS + s - c] is the bias of key - query offset
    // (r - 22, s - 22), i.e. table[((r - 22)*39 + (s - 22)) mod 1521].
    constexpr int NT = Shape::threads, NLT = 32 * Shape::loaders, LW0 = 1 + Shape::softmax;  // first loader warp
    {
        constexpr int TS = OCA ? OCA_TS : SA_TS, CS = OCA ? OCA_CS : SA_CS;
        for (int i = threadIdx.x; i < 4 * CS; i += NT) {
            const int cp = i / CS, at = i - cp * CS + cp, r = at / TS, s = at - r * TS;
            float v = 0.f;
            if (r < TR && s < TR) {
                int src = OCA ? (r - 22) * TW + (s - 22) : r * TW + s;
                if (src < 0) src += TR * TW;
                v = table[(long)src * heads + head] * L2E;
            }
            tab[i] = v;
        }
    }
    if (threadIdx.x == 0) {
        for (int b = 0; b < QB; ++b) {
            bar_init(&q_full[b], NLT);
            bar_init(&q_empty[b], 1);
        }
        for (int s = 0; s < KVS; ++s) {
            bar_init(&kv_full[s], NLT);
            bar_init(&kv_empty[s], 1);
        }
        for (int h = 0; h < HV; ++h) {
            for (int s = 0; s < 2; ++s) {
                bar_init(&s_full[h][s], 1);
                bar_init(&p_full[h][s], 128);
                bar_init(&o_free[h][s], 128);
            }
            bar_init(&o_done[h], 1);
        }
        bar_init(&drain, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su(&tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (PRE) {
        // The head dim's padding (24 -> 32) is never copied: zero it once. Q and K: the second
        // 16-byte piece of k-step 1 of every row; V^T: feature rows 24..31.
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        for (int i = threadIdx.x; i < QB * HV * 2 * MT; i += NT)
            *reinterpret_cast<uint4*>(sm + (i / MT) * Q_BYTES + 4096 + off_sw32(i % MT, 1)) = z;
        for (int i = threadIdx.x; i < KVS * 2 * KBLK; i += NT) {
            const int st = i / (2 * KBLK), lo = (i / KBLK) & 1, key = i % KBLK;
            *reinterpret_cast<uint4*>(sm + OFF_KV + st * KV_BYTES + lo * K_BYTES + 1024 + off_sw32(key, 1)) = z;
        }
        // V^T row 24 of the hi tile is all ones (fp16 1.0) and every other padding row zero: the
        // PV product then leaves the row sum of P in column 24 of O (P_lo.1 + P_hi.1 + P_hi.0),
        // accumulated and rescaled along with O.
        const uint4 one = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
        for (int i = threadIdx.x; i < KVS * 2 * 8 * 4; i += NT) {
            const int st = i / 64, lo = (i / 32) & 1, f = 24 + ((i / 4) & 7), ks = (i / 2) & 1, pc = i & 1;
            *reinterpret_cast<uint4*>(sm + OFF_KV + st * KV_BYTES + 2 * K_BYTES + lo * V_BYTES + ks * 1024 +
                                      off_sw32(f, pc)) = (f == 24 && !lo) ? one : z;
        }
        fence_async();
    }
    tcf_before();
    __syncthreads();
    tcf_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_s = idesc_h(32), id_o = idesc_h(32);
            long g = 0;  // global key-block counter
            uint32_t ti = 0;
            bool ok = true;
            for (long w = blockIdx.x; w < items && ok; w += gridDim.x, ++ti) {
                const int qb = (int)(ti % QB);
                if (!bar_wait(&q_full[qb], (ti / QB) & 1, &abort_flag, err, 11)) break;
                // Each half's O block of this item's parity must have been read by the softmax.
                for (int h = 0; h < HV && ok; ++h)
                    ok = bar_wait(&o_free[h][ti & 1], ((ti >> 1) & 1) ^ 1, &abort_flag, err, 19);
                if (!ok) break;
                // S of key block gb for every half (each into its own buffer gb & 1)
                auto issue_s = [&](long gb) -> bool {
                    const int s = (int)(gb & 1), kvs = (int)(gb % KVS);
                    if (!bar_wait(&kv_full[kvs], (uint32_t)((gb / KVS) & 1), &abort_flag, err, 12)) return false;
                    tcf_after();
                    const uint32_t kb = su(sm + OFF_KV + kvs * KV_BYTES);
#pragma unroll
                    for (int h = 0; h < HV; ++h) {
                        const uint32_t qh = su(sm + qb * Q_REGION + h * 2 * Q_BYTES), ql = qh + Q_BYTES;
                        const uint32_t d = tmem + h * 64 + s * 32;
#pragma unroll
                        for (int k = 0; k < KH; ++k) {
                            const uint64_t aH = mdesc(qh + k * 4096, 32, 256), aL = mdesc(ql + k * 4096, 32, 256);
                            const uint64_t bH = mdesc(kb + k * 1024, 32, 256),
                                           bL = mdesc(kb + K_BYTES + k * 1024, 32, 256);
                            if (TERMS == 3) {
                                mma_ss(d, aL, bH, id_s, k ? 1u : 0u);
                                mma_ss(d, aH, bL, id_s, 1u);
                                mma_ss(d, aH, bH, id_s, 1u);
                            } else {
                                mma_ss(d, aH, bH, id_s, k ? 1u : 0u);
                            }
                        }
                        commit(&s_full[h][s]);
                    }
                    return true;
                };
                if (!issue_s(g)) break;
                for (int j = 0; j < NBLK; ++j) {
                    const long gb = g + j;
                    // S of the next block goes into the other S buffers, whose P the previous
                    // PVs (issued earlier, executed in order) have consumed.
                    if (j + 1 < NBLK) {
                        if (!issue_s(gb + 1)) {
                            ok = false;
                            break;
                        }
                        // Once the item's last S MMAs are issued, Q may be replaced.
                        if (j + 1 == NBLK - 1) commit(&q_empty[qb]);
                    }
                    const int s = (int)(gb & 1);
                    const int kvs = (int)(gb % KVS);
                    const uint32_t vb = su(sm + OFF_KV + kvs * KV_BYTES + 2 * K_BYTES);
                    for (int h = 0; h < HV; ++h) {
                        if (!bar_wait(&p_full[h][s], (uint32_t)((gb >> 1) & 1), &abort_flag, err, 13)) {
                            ok = false;
                            break;
                        }
                        tcf_after();
                        const uint32_t od = tmem + T_O + h * 64 + (ti & 1) * 32;
                        const uint32_t ph = tmem + h * 64 + s * 32, pl = ph + T_PLO;
#pragma unroll
                        for (int k = 0; k < KBLK / 16; ++k) {
                            const uint64_t bH = mdesc(vb + k * 1024, 32, 256),
                                           bL = mdesc(vb + V_BYTES + k * 1024, 32, 256);
                            const uint32_t acc = (j | k) ? 1u : 0u;
                            if (TERMS == 3) {
                                mma_ts(od, pl + k * 8, bH, id_o, acc);
                                mma_ts(od, ph + k * 8, bL, id_o, 1u);
                                mma_ts(od, ph + k * 8, bH, id_o, 1u);
                            } else {
                                mma_ts(od, ph + k * 8, bH, id_o, acc);
                            }
                        }
                        commit(&o_done[h]);
                    }
                    if (!ok) break;
                    commit(&kv_empty[kvs]);
                }
                g += NBLK;
            }
            commit(&drain);
            bar_wait_quiet(&drain, 0);
        }
    } else if (warp <= Shape::softmax) {
        // ------------------------------------------------------------ softmax
        const int q4 = warp & 3;       // TMEM lane quarter (a warp reaches lanes 32 (warp % 4) ..)
        const int hh = (warp - 1) >> 2;  // the query half of the item this warp works on
        const uint32_t th = (uint32_t)hh * 64;
        const int row = q4 * 32 + lane;
        const uint32_t trow = (uint32_t)(q4 * 32) << 16;
        constexpr int VW = (D % 4 == 0) ? 4 : 2;
        long g = 0;
        uint32_t ti = 0;
        for (long w = blockIdx.x; w < items; w += gridDim.x, ++ti) {
            if (__any_sync(0xffffffffu, abort_flag != 0)) break;
            const long rest = w / heads;
            const int win = HV == 2 ? (int)rest : (int)(rest >> 1), mtile = HV == 2 ? hh : (int)(rest & 1);
            const int wy = win / nx, wx = win - wy * nx;
            const int qi = mtile * MT + row, qy = qi >> 4, qx = qi & 15;
            const bool masked = !OCA && gm.mshift > 0;
            const int shift = gm.mshift, ghp = gm.ghp;
            const int yrw = gm.yr0 + wy * 16;  // rolled-frame row of the window's first row (mod ghp)
            // OCAB: the copy whose runs of key biases start 16-byte aligned for this query column
            const int occ = (15 - qx) & 3;
            // Shift mask: key column kx is masked against target label t when
            // band(wx*16+kx) != t; one 16-bit mask per possible row band.
            uint32_t cm[3] = {0, 0, 0};
            if (masked) {
                const int lq = band3((yrw + qy) % ghp, ghp, shift) * 3 + band3(wx * 16 + qx, wp, shift);
#pragma unroll
                for (int kx = 0; kx < 16; ++kx) {
                    const int bx = band3(wx * 16 + kx, wp, shift);
#pragma unroll
                    for (int by = 0; by < 3; ++by)
                        if (by * 3 + bx != lq) cm[by] |= 1u << kx;
                }
            }
            const uint32_t t_o = tmem + trow + T_O + th + (ti & 1) * 32;
            float m = 0.f, l = 0.f;
            bool ok = true;
            for (int j = 0; j < NBLK; ++j) {
                const long gb = g + j;
                const int s = (int)(gb & 1);
                const bool got = bar_wait(&s_full[hh][s], (uint32_t)((gb >> 1) & 1), &abort_flag, err, 16);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                tcf_after();
                float sv[32];
                tld32(tmem + trow + th + s * 32, sv);
                uint32_t mrow0 = 0, mrow1 = 0;
                if (masked) {
                    // the block's two key rows ky = 2j, 2j+1
                    const int b0 = band3((yrw + 2 * j) % ghp, ghp, shift), b1 = band3((yrw + 2 * j + 1) % ghp, ghp, shift);
                    mrow0 = b0 == 0 ? cm[0] : (b0 == 1 ? cm[1] : cm[2]);  // selects: no local memory
                    mrow1 = b1 == 0 ? cm[0] : (b1 == 1 ? cm[1] : cm[2]);
                }
                if (OCA) {
#pragma unroll
                    for (int g8 = 0; g8 < 4; ++g8) {
                        // keys k0 .. k0 + 7 lie in key row ky, columns kx0 .. kx0 + 7 (kx0 a multiple of
                        // 8): biases tab[(ky - qy + 15)*OCA_TS + kx - qx + 15], ascending
                        const int k0 = j * KBLK + 8 * g8, ky = k0 / 24, kx0 = k0 - 24 * ky;
                        const float4* b = reinterpret_cast<const float4*>(
                            tab + occ * OCA_CS + (ky - qy + 15) * OCA_TS + kx0 - qx + 15 - occ);
                        const float4 t0 = b[0], t1 = b[1];
                        sv[8 * g8 + 0] += t0.x;
                        sv[8 * g8 + 1] += t0.y;
                        sv[8 * g8 + 2] += t0.z;
                        sv[8 * g8 + 3] += t0.w;
                        sv[8 * g8 + 4] += t1.x;
                        sv[8 * g8 + 5] += t1.y;
                        sv[8 * g8 + 6] += t1.z;
                        sv[8 * g8 + 7] += t1.w;
                    }
                } else if (!PRE) {
                    // tab[(ky - ... )]: scalar loads from copy 0 (even query rows) or copy 2 (odd
                    // ones), which keeps the two half-warps apart in the banks but for two lanes
                    const int cp = (qy & 1) * 2;
                    const float* t0 = tab + cp * SA_CS + (qy + 15 - 2 * j) * SA_TS + qx + 15 - cp;
#pragma unroll
                    for (int k = 0; k < 32; ++k) {
                        sv[k] += t0[-(k >> 4) * SA_TS - (k & 15)];
                        if (masked) {
                            const uint32_t mr = (k >> 4) ? mrow1 : mrow0;
                            if ((mr >> (k & 15)) & 1u) sv[k] += -100.f * L2E;
                        }
                    }
                } else {
                    // key row ky = 2j + kyl: the biases for kx = 15 .. 0 are 16 consecutive
                    // floats of copy (qx mod 4), four aligned 16-byte loads
                    const float4* b4 = reinterpret_cast<const float4*>(tab + (qx & 3) * SA_CS) +
                                       (qy + 15 - 2 * j) * (SA_TS / 4) + (qx >> 2);
#pragma unroll
                    for (int kyl = 0; kyl < 2; ++kyl)
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float4 t = b4[q - kyl * (SA_TS / 4)];
                            sv[kyl * 16 + 15 - 4 * q] += t.x;
                            sv[kyl * 16 + 14 - 4 * q] += t.y;
                            sv[kyl * 16 + 13 - 4 * q] += t.z;
                            sv[kyl * 16 + 12 - 4 * q] += t.w;
                        }
                    if (masked) {
#pragma unroll
                        for (int k = 0; k < 32; ++k) {
                            const uint32_t mr = (k >> 4) ? mrow1 : mrow0;
                            if ((mr >> (k & 15)) & 1u) sv[k] += -100.f * L2E;
                        }
                    }
                }
                // sv is in log2 units: q carries scale * log2(e), the table log2(e)
                // the block max: 16 three-input maxes
                float bmax = fmaxf(sv[0], sv[1]);
#pragma unroll
                for (int k = 2; k < 32; k += 2) bmax = fmax3(bmax, sv[k], sv[k + 1]);
                // The row's reference max moves only on a large jump (first block: set).
                const bool need = j == 0 || bmax > m + RESCALE_LOG2;
                float a = 1.f;
                if (need) {
                    a = j == 0 ? 0.f : ex2(m - bmax);
                    m = bmax;
                    l *= a;
                }
                // P (times 2^P_SHIFT) as fp16 hi/lo pairs over the block's S columns.
                float psum = 0.f;
                uint32_t ph[16], pl[16];
                const float mo = m - P_SHIFT;
#pragma unroll
                for (int k = 0; k < 32; k += 2) {
                    const float p0 = ex2(sv[k] - mo), p1 = ex2(sv[k + 1] - mo);
                    if (!PRE) psum += p0 + p1;  // PRE: the row sum comes from O's column 24
                    split_h16x2(p0, p1, ph[k >> 1], pl[k >> 1]);
                }
                tst16(tmem + trow + th + s * 32, ph);
                if (TERMS == 3) tst16(tmem + trow + th + s * 32 + T_PLO, pl);
                if (!PRE) l += psum;
                if (j > 0) {
                    // PV of the previous block has finished (this also keeps every
                    // o_done phase consumed in order); a moved max then rescales the
                    // row's O before this block's PV adds to it.
                    const bool done = bar_wait(&o_done[hh], (uint32_t)((gb - 1) & 1), &abort_flag, err, 15);
                    if (!__all_sync(0xffffffffu, done)) {
                        ok = false;
                        break;
                    }
                    if (__any_sync(0xffffffffu, need)) {
                        tcf_after();
                        float ov[32];
                        tld32(t_o, ov);
#pragma unroll
                        for (int i = 0; i < 32; ++i) ov[i] *= a;
                        tst32(t_o, ov);
                    }
                }
                tst_wait();
                tcf_before();
                bar_arrive(&p_full[hh][s]);
            }
            if (!ok) break;
            // O / l at the query's plane position (the roll of the shifted windows undone).
            const bool done = bar_wait(&o_done[hh], (uint32_t)((g + NBLK - 1) & 1), &abort_flag, err, 15);
            if (!__all_sync(0xffffffffu, done)) break;
            tcf_after();
            float ov[32];
            tld32(t_o, ov);
            tcf_before();
            bar_arrive(&o_free[hh][ti & 1]);
            const float inv = 1.f / (PRE ? ov[24] : l);
            if constexpr (PRE && !OCA) {
                const int tx0 = wx * 16 + gm.sx, ty0 = gm.oy + wy * 16 + gm.sy;
                if (tx0 + 16 <= wp && ty0 + 16 <= gm.rows) {
                    // A window that does not wrap: the half's 128 rows of 24 features as fp16 pairs
                    // into the staging tile, then two TMA stores by the half's first thread. (A
                    // strip's shifted windows also write rows of the halo, which no one reads.)
                    uint8_t* stg = sm + OFF_OST + hh * 2 * OST_BYTES;
                    const bool issuer = (warp - 1) % 4 == 0 && lane == 0;
                    if (issuer) bulk_wait_read();  // the half's previous stores have read the tile
                    half_sync(hh);
                    bool big = false;
#pragma unroll
                    for (int i = 0; i < D; i += 8) {
                        uint4 h, lo;
                        split_h16x2(ov[i] * inv, ov[i + 1] * inv, h.x, lo.x);
                        split_h16x2(ov[i + 2] * inv, ov[i + 3] * inv, h.y, lo.y);
                        split_h16x2(ov[i + 4] * inv, ov[i + 5] * inv, h.z, lo.z);
                        split_h16x2(ov[i + 6] * inv, ov[i + 7] * inv, h.w, lo.w);
#pragma unroll
                        for (int u = 0; u < 8; ++u) big |= beyond_h16(ov[i + u] * inv);
                        *reinterpret_cast<uint4*>(stg + row * 48 + 2 * i) = h;
                        *reinterpret_cast<uint4*>(stg + OST_BYTES + row * 48 + 2 * i) = lo;
                    }
                    if (big && out.err) atomicCAS(out.err, 0, ERR_RANGE_GEMM);
                    fence_async();
                    half_sync(hh);
                    if (issuer) {
                        tma4_store(&toh, su(stg), 0, head, tx0, ty0 + 8 * hh);
                        tma4_store(&tol, su(stg + OST_BYTES), 0, head, tx0, ty0 + 8 * hh);
                        bulk_commit();
                    }
                    g += NBLK;
                    continue;
                }
            }
            const int qrow = OCA ? gm.oy + wy * 16 + qy : (gm.oy + wy * 16 + qy + gm.sy) % gm.rows;
            const long qpos = (long)qrow * wp + (OCA ? wx * 16 + qx : (wx * 16 + qx + gm.sx) % wp);
            const long ob = qpos * c + (long)head * D;
            if (qrow >= gm.olo && qrow < gm.ohi) {  // rows outside [olo, ohi) are a neighbour's
                if (D % 8 == 0 && c % 8 == 0 && out.lo && out.h16) {
                    // fp16 pairs, 16 bytes (8 features) a store, one range check
                    bool big = false;
#pragma unroll
                    for (int i = 0; i < D; i += 8) {
                        uint4 h, lo;
                        split_h16x2(ov[i] * inv, ov[i + 1] * inv, h.x, lo.x);
                        split_h16x2(ov[i + 2] * inv, ov[i + 3] * inv, h.y, lo.y);
                        split_h16x2(ov[i + 4] * inv, ov[i + 5] * inv, h.z, lo.z);
                        split_h16x2(ov[i + 6] * inv, ov[i + 7] * inv, h.w, lo.w);
#pragma unroll
                        for (int u = 0; u < 8; ++u) big |= beyond_h16(ov[i + u] * inv);
                        *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(out.hi) + ob + i) = h;
                        *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(out.lo) + ob + i) = lo;
                    }
                    if (big && out.err) atomicCAS(out.err, 0, ERR_RANGE_GEMM);
                } else if (VW == 4) {
#pragma unroll
                    for (int i = 0; i < D; i += 4)
                        put4(out, ob + i, make_float4(ov[i] * inv, ov[i + 1] * inv, ov[i + 2] * inv, ov[i + 3] * inv));
                } else {
#pragma unroll
                    for (int i = 0; i < D; ++i) put(out, ob + i, ov[i] * inv);
                }
            }
            g += NBLK;
        }
        // the output stores have finished before the CTA (and its shared memory) goes away
        if (PRE && !OCA && (warp - 1) % 4 == 0 && lane == 0) bulk_wait_all();
    } else if constexpr (PRE) {
        // ------------------------------------------------------------ loaders (copies)
        // Per item, Q: 128 rows x 3 pieces of 8 dims x (hi, lo) = 6 copies a thread. Per key
        // block, K: 32 keys x 3 x 2 16-byte copies, and V^T: SA, 24 features x 4 pieces of 8
        // keys x 2 (a key block is two window rows, and each 8-key piece is contiguous in
        // the plane: the roll moves windows by 8 columns, so pieces never wrap); OCAB, 24
        // features x 8 pieces of 4 keys x 2 8-byte copies (the key window starts 4 columns
        // left of the query window). OCAB keys outside the image are zeros, a whole piece at
        // a time (the image edges fall on multiples of 4).
        static_assert(D == 24 && TERMS == 3, "the copy loaders are for parity attention, D = 24");
        const int t = threadIdx.x - 32 * LW0;  // 0..NLT-1
        const long P = (long)gm.rows * wp, c2 = 2L * c;
        constexpr int R = 6;  // copies in flight a thread (registers), rounds of R
        const __half* qkh = reinterpret_cast<const __half*>(qkv);
        const __half* qkl = qkh + P * c2;
        const __half* vth = qkl + P * c2;
        const __half* vtl = vth + (long)c * P;
        auto pos = [&](int wy, int wx, int y, int x) -> long {
            return (long)((gm.oy + wy * 16 + y + gm.sy) % gm.rows) * wp + (wx * 16 + x + gm.sx) % wp;
        };
        // OCAB key (ky, kx) of window (wy, wx): its plane index, or -1 outside the image
        auto okey = [&](int wy, int wx, int ky, int kx) -> long {
            const int Y = gm.oy + wy * 16 - 4 + ky, X = wx * 16 - 4 + kx;
            const bool in = Y >= 0 && Y < gm.rows && gm.gy0 + Y >= 0 && gm.gy0 + Y < gm.ghp && X >= 0 && X < wp;
            return in ? (long)Y * wp + X : -1;
        };
        long g = 0;
        uint32_t ti = 0;
        for (long w = blockIdx.x; w < items; w += gridDim.x, ++ti) {
            if (__any_sync(0xffffffffu, abort_flag != 0)) break;
            const long rest = w / heads;
            const int win = HV == 2 ? (int)rest : (int)(rest >> 1), mtile = HV == 2 ? 0 : (int)(rest & 1);
            const int wy = win / nx, wx = win - wy * nx;
            const int qb = (int)(ti % QB);
            // Windows that do not wrap around the plane's edge are loaded by TMA: q|k as 4-D tiles
            // (head dim, head, x, y) whose dims 24..31 come back as the tile's out-of-range zeros,
            // and v^T as 3-D tiles (x, feature, y) whose rows past the head's 24 features are
            // never read back from O. The shifted windows of the last column or row wrap around
            // the plane and are copied by the loader threads instead.
            const int tx0 = wx * 16 + gm.sx, ty0 = gm.oy + wy * 16 + gm.sy;
            const bool tma = !OCA && tx0 + 16 <= wp && ty0 + 16 <= gm.rows;
            if (tma) {
                const bool got = bar_wait(&q_empty[qb], ((ti / QB) & 1) ^ 1, &abort_flag, err, 17);
                if (!__all_sync(0xffffffffu, got)) break;
                if (t == 0) {
                    bar_expect_tx(&q_full[qb], HV * 2 * KH * 4096);
#pragma unroll
                    for (int h = 0; h < HV; ++h)
#pragma unroll
                        for (int k = 0; k < KH; ++k) {
                            const uint32_t d = su(sm + qb * Q_REGION + 2 * h * Q_BYTES + k * 4096);
                            const int y = ty0 + 8 * (mtile + h);
                            tma4(d, &tqh, 16 * k, head, tx0, y, &q_full[qb]);
                            tma4(d + Q_BYTES, &tql, 16 * k, head, tx0, y, &q_full[qb]);
                        }
                } else {
                    bar_arrive(&q_full[qb]);
                }
            } else {
                // Q: 768 copies per half, R at a time per thread (the first round issued before
                // the wait)
                bool got = true;
#pragma unroll 1
                for (int r0 = 0; r0 < 768 * HV; r0 += R * NLT) {
                    uint4 qv[R];
                    uint32_t qd[R];
#pragma unroll
                    for (int u = 0; u < R; ++u) {
                        const int cid0 = r0 + t + NLT * u, half = cid0 / 768, cid = cid0 - 768 * half;
                        const int row = cid / 6, part = cid % 6, lo = part / 3, ch = part % 3;
                        const int qi = (mtile + half) * MT + row;
                        const long qpos = OCA ? (long)(gm.oy + wy * 16 + (qi >> 4)) * wp + wx * 16 + (qi & 15)
                                              : pos(wy, wx, qi >> 4, qi & 15);
                        qv[u] = *reinterpret_cast<const uint4*>((lo ? qkl : qkh) + qpos * c2 + head * D + 8 * ch);
                        qd[u] = qb * Q_REGION + (2 * half + lo) * Q_BYTES + (ch >> 1) * 4096 + off_sw32(row, ch & 1);
                    }
                    if (r0 == 0) {
                        got = bar_wait(&q_empty[qb], ((ti / QB) & 1) ^ 1, &abort_flag, err, 17);
                        if (!__all_sync(0xffffffffu, got)) break;
                    }
#pragma unroll
                    for (int u = 0; u < R; ++u) *reinterpret_cast<uint4*>(sm + qd[u]) = qv[u];
                }
                if (!__all_sync(0xffffffffu, got)) break;
                fence_async();
                bar_arrive(&q_full[qb]);
            }
            bool ok = true;
            for (int j = 0; j < NBLK; ++j) {
                const long gb = g + j;
                const int s = (int)(gb % KVS);
                constexpr int NCOPY = OCA ? 576 : 384;  // 192 K + 384 (OCAB) or 192 V^T copies
                bool got = true;
                uint8_t* kvb = sm + OFF_KV + s * KV_BYTES;
                if (tma) {
                    got = bar_wait(&kv_empty[s], (uint32_t)(((gb / KVS) & 1) ^ 1), &abort_flag, err, 18);
                    if (!__all_sync(0xffffffffu, got)) {
                        ok = false;
                        break;
                    }
                    if (t == 0) {
                        bar_expect_tx(&kv_full[s], 2 * K_BYTES + 4 * 768);
                        const uint32_t kb = su(kvb);
                        const int y = ty0 + 2 * j;  // the block's two key rows
#pragma unroll
                        for (int k = 0; k < KH; ++k) {
                            tma4(kb + k * 1024, &tkh, 16 * k, head, tx0, y, &kv_full[s]);
                            tma4(kb + K_BYTES + k * 1024, &tkl, 16 * k, head, tx0, y, &kv_full[s]);
                        }
                        // v^T: per key row, the head's 24 feature rows of a 16-key k-step (768
                        // bytes); rows 24..31 keep their ones / zeros
#pragma unroll
                        for (int ks = 0; ks < 2; ++ks) {
                            tma3(kb + 2 * K_BYTES + ks * 1024, &tvh, tx0, head * D, y + ks, &kv_full[s]);
                            tma3(kb + 2 * K_BYTES + V_BYTES + ks * 1024, &tvl, tx0, head * D, y + ks, &kv_full[s]);
                        }
                    } else {
                        bar_arrive(&kv_full[s]);
                    }
                    continue;
                }
#pragma unroll 1
                for (int r0 = 0; r0 < NCOPY; r0 += R * NLT) {
                uint4 cv[R];
                uint32_t dst[R];
                bool wide[R];
#pragma unroll
                for (int u = 0; u < R; ++u) {
                    const int cid = r0 + t + NLT * u;
                    cv[u] = make_uint4(0u, 0u, 0u, 0u);
                    dst[u] = 0xffffffffu;
                    wide[u] = true;
                    if (cid >= NCOPY) continue;
                    if (cid < 192) {
                        const int key = cid / 6, part = cid % 6, lo = part / 3, ch = part % 3;
                        const int kk = j * KBLK + key;
                        const long kpos = OCA ? okey(wy, wx, kk / 24, kk % 24) : pos(wy, wx, kk >> 4, kk & 15);
                        if (kpos >= 0)
                            cv[u] = *reinterpret_cast<const uint4*>((lo ? qkl : qkh) + kpos * c2 + c + head * D + 8 * ch);
                        dst[u] = lo * K_BYTES + (ch >> 1) * 1024 + off_sw32(key, ch & 1);
                    } else if (!OCA) {
                        const int v2 = cid - 192, f = v2 >> 3, part = v2 & 7, lo = part >> 2;
                        const int ks = (part >> 1) & 1, pc = part & 1;  // key row 2j + ks, keys 8 pc ..
                        const long kpos = pos(wy, wx, 2 * j + ks, 8 * pc);
                        cv[u] = *reinterpret_cast<const uint4*>((lo ? vtl : vth) + (long)(head * D + f) * P + kpos);
                        dst[u] = 2 * K_BYTES + lo * V_BYTES + ks * 1024 + off_sw32(f, pc);
                    } else {
                        const int v2 = cid - 192, f = v2 >> 4, part = v2 & 15, lo = part >> 3, pc4 = part & 7;
                        const int kb = 4 * pc4, kk = j * KBLK + kb;  // 4 keys kb .. kb+3 of the block
                        const long kpos = okey(wy, wx, kk / 24, kk % 24);
                        if (kpos >= 0) {
                            const uint2 x2 =
                                *reinterpret_cast<const uint2*>((lo ? vtl : vth) + (long)(head * D + f) * P + kpos);
                            cv[u].x = x2.x;
                            cv[u].y = x2.y;
                        }
                        wide[u] = false;
                        dst[u] = 2 * K_BYTES + lo * V_BYTES + (kb >> 4) * 1024 + off_sw32(f, (kb >> 3) & 1) + (kb & 7) * 2;
                    }
                }
                if (r0 == 0) {
                    got = bar_wait(&kv_empty[s], (uint32_t)(((gb / KVS) & 1) ^ 1), &abort_flag, err, 18);
                    if (!__all_sync(0xffffffffu, got)) break;
                }
#pragma unroll
                for (int u = 0; u < R; ++u) {
                    if (dst[u] == 0xffffffffu) continue;
                    if (wide[u])
                        *reinterpret_cast<uint4*>(kvb + dst[u]) = cv[u];
                    else
                        *reinterpret_cast<uint2*>(kvb + dst[u]) = make_uint2(cv[u].x, cv[u].y);
                }
                }
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                fence_async();
                bar_arrive(&kv_full[s]);
            }
            if (!ok) break;
            g += NBLK;
        }
    } else {
        // ------------------------------------------------------------ loaders
        // Warps 5-6 load K: lane = key, warp = k-step (columns [0,16) / [16,32)); each
        // 8-column chunk is one 16-byte store of fp16 into the K-major SW32 tiles. Warps
        // 7-8 load V: a thread owns a 4-key x 4-feature block, transposes it in registers
        // and writes four 8-byte pieces of V^T rows (K-major SW32, one 32-byte row of 16
        // keys per feature and k-step). Loads for the next key block are issued before
        // waiting for a free stage. A value of fp16's range or beyond records error 20.
        constexpr int VW = (D % 4 == 0) ? 4 : 2;  // vector width that keeps the row alignment
        const int t = threadIdx.x - 160;           // 0..127
        const int lw = warp - 5;                   // 0..3
        const bool is_v = lw >= 2;
        const int kk0 = is_v ? (((lw - 2) * 32 + lane) & 7) * 4 : lane;  // first key of this thread
        const int col0 = is_v ? (((lw - 2) * 32 + lane) >> 3) * 4 : lw * 16;
        long g = 0;
        uint32_t ti = 0;
        float buf[16];
        bool range_ok = true;
        // fp16 hi/lo of 8 values as four packed words each (element 2i in the low half).
        auto split8 = [&](const float* x, uint4& hi, uint4& lo) {
            uint32_t h[4], l[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                range_ok &= !(fabsf(x[2 * i]) >= F16_LIMIT) && !(fabsf(x[2 * i + 1]) >= F16_LIMIT);
                split_h16x2(x[2 * i], x[2 * i + 1], h[i], l[i]);
            }
            hi = make_uint4(h[0], h[1], h[2], h[3]);
            lo = make_uint4(l[0], l[1], l[2], l[3]);
        };
        auto key_pos = [&](int wy, int wx, int kk, bool& inside) -> long {
            inside = true;
            if (OCA) {
                const int ky = kk / 24, kx = kk - ky * 24;
                const int Y = gm.oy + wy * 16 - 4 + ky, X = wx * 16 - 4 + kx;
                inside = Y >= 0 && Y < gm.rows && gm.gy0 + Y >= 0 && gm.gy0 + Y < gm.ghp && X >= 0 && X < wp;
                return inside ? (long)Y * wp + X : 0;
            }
            const int ky = kk >> 4, kx = kk & 15;
            return (long)((gm.oy + wy * 16 + ky + gm.sy) % gm.rows) * wp + (wx * 16 + kx + gm.sx) % wp;
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
                const long qpos =
                    OCA ? (long)(gm.oy + wy * 16 + qy) * wp + wx * 16 + qx
                        : (long)((gm.oy + wy * 16 + qy + gm.sy) % gm.rows) * wp + (wx * 16 + qx + gm.sx) % wp;
                const float* src = qkv + qpos * c3 + (long)head * D;
                float qv[KH * 16];
                load_cols(src, 0, true, qv, 16);
                if (KH > 1) load_cols(src, 16, true, qv + 16, 16);
#pragma unroll
                for (int i = 0; i < KH * 16; ++i) qv[i] *= scale * L2E;
                const bool got = bar_wait(&q_empty[0], (ti & 1) ^ 1, &abort_flag, err, 17);
                if (!__all_sync(0xffffffffu, got)) break;
#pragma unroll
                for (int c8 = 0; c8 < KH * 2; ++c8) {
                    uint4 h, lo;
                    split8(qv + 8 * c8, h, lo);
                    const uint32_t o = (c8 >> 1) * 4096 + off_sw32(t, c8 & 1);
                    *reinterpret_cast<uint4*>(sm + o) = h;
                    if (TERMS == 3) *reinterpret_cast<uint4*>(sm + Q_BYTES + o) = lo;
                }
                fence_async();
                bar_arrive(&q_full[0]);
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
                    if (lw < KH) {
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            uint4 h, lo;
                            split8(buf + 8 * q, h, lo);
                            const uint32_t o = lw * 1024 + off_sw32(kk0, q);
                            *reinterpret_cast<uint4*>(kvb + o) = h;
                            if (TERMS == 3) *reinterpret_cast<uint4*>(kvb + K_BYTES + o) = lo;
                        }
                    }
                } else {
#pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        const int n = col0 + f;  // feature = row of V^T
                        const float x[4] = {buf[f], buf[4 + f], buf[8 + f], buf[12 + f]};
                        uint32_t h[2], l[2];
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            range_ok &= !(fabsf(x[2 * i]) >= F16_LIMIT) && !(fabsf(x[2 * i + 1]) >= F16_LIMIT);
                            split_h16x2(x[2 * i], x[2 * i + 1], h[i], l[i]);
                        }
                        const uint32_t o = 2 * K_BYTES + (kk0 >> 4) * 1024 + off_sw32(n, (kk0 >> 3) & 1) + (kk0 & 7) * 2;
                        *reinterpret_cast<uint2*>(kvb + o) = make_uint2(h[0], h[1]);
                        if (TERMS == 3) *reinterpret_cast<uint2*>(kvb + V_BYTES + o) = make_uint2(l[0], l[1]);
                    }
                }
                fence_async();
                bar_arrive(&kv_full[s]);
                if (j + 1 < NBLK) fetch(wy, wx, j + 1);
            }
            if (!ok) break;
            g += NBLK;
        }
        if (!range_ok) atomicCAS(err, 0, ERR_RANGE_ATTN);
    }

    tcf_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tcf_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

template <int D, bool OCA, int TERMS, bool PRE = false>
static void run_tc(const float* qkv, const float* table, Dst out, const Plan& p, int c, int heads, int shift, int* err,
                   cudaStream_t st) {
    constexpr int KH = (D + 15) / 16;
    constexpr int TR = OCA ? 39 : 31;
    using Shape = AttnShape<PRE && !OCA>;
    constexpr int QB = 1;  // Q buffers (see the kernel)
    constexpr size_t tab_end = QB * Shape::halves * 2 * KH * 4096 + KVS * (2 * KH * 1024 + 2 * 2048) +
                               tab_floats<OCA>() * 4;
    // + the window kernel's output staging (1 KB aligned), + 1 KB to align the base
    constexpr size_t bytes = (PRE && !OCA ? ((tab_end + 1023) & ~(size_t)1023) + 2 * Shape::halves * 128 * 48
                                          : tab_end) + 1024;
    allow_dyn_smem(k_attn_tc<D, OCA, TERMS, PRE>, bytes);
    // The windows of this launch (see AttnGeom).
    AttnGeom gm;
    gm.rows = p.rows;
    gm.wp = p.wp;
    gm.ghp = p.hp;
    gm.gy0 = p.gy0();
    gm.olo = p.halo;
    gm.ohi = p.halo + p.own();
    gm.yr0 = 0;
    gm.sy = gm.sx = gm.mshift = 0;
    if (!p.strip()) {
        gm.nwy = p.hp / 16;
        gm.oy = 0;
        if (!OCA) gm.sy = gm.sx = gm.mshift = shift;
    } else if (OCA || shift == 0) {
        gm.nwy = p.own() / 16;  // the strip's own windows
        gm.oy = p.halo;
    } else {
        // Shifted windows overlapping the strip: the rolled frame's window rows start at
        // padded rows 16k + shift; the first one that reaches row r0 starts at r0 - shift.
        if (p.halo < shift) throw Error(1, "attention: a strip's halo is narrower than the window shift");
        gm.nwy = p.own() / 16 + 1;
        gm.oy = p.halo - shift;
        gm.sx = gm.mshift = shift;
        gm.yr0 = ((p.r0 - 2 * shift) % p.hp + p.hp) % p.hp;
    }
    const long items = (long)gm.nwy * p.nx() * heads * (2 / Shape::halves);
    int sms = 0, dev = 0;
    HAT_CUDA(cudaGetDevice(&dev));
    HAT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // AttnShape::ctas CTAs per SM; a multiple of the head count, so every CTA keeps one head
    // (and one bias table).
    long grid = std::min<long>(items, (long)(Shape::ctas * sms / heads) * heads);
    // TMA maps of the pre-split layout for the window kernel (see the loaders): q|k hi / lo as
    // (head dim 24, head, x, y) with 16 x 1 x 16 x {8, 2} boxes, v^T hi / lo as (x, feature,
    // y) with 16 x 32 x 2 boxes; 32-byte swizzled rows, fp16.
    CUtensorMap m[8];
    memset(m, 0, sizeof m);
    if (PRE && !OCA) {
        const long P = (long)p.rows * p.wp;
        const __half* qkh = reinterpret_cast<const __half*>(qkv);
        const __half* qkl = qkh + P * 2 * c;
        const __half* vth = qkl + P * 2 * c;
        const __half* vtl = vth + (long)c * P;
        const uint64_t qdims[4] = {(uint64_t)D, (uint64_t)heads, (uint64_t)p.wp, (uint64_t)p.rows};
        const uint64_t qstr[3] = {(uint64_t)D * 2, (uint64_t)c * 4, (uint64_t)p.wp * c * 4};
        const uint32_t qbox[4] = {16, 1, 16, 8}, kbox[4] = {16, 1, 16, 2};
        m[0] = tensor_map(qkh, 4, qdims, qstr, qbox, 32, true);
        m[1] = tensor_map(qkl, 4, qdims, qstr, qbox, 32, true);
        m[2] = tensor_map(qkh + c, 4, qdims, qstr, kbox, 32, true);
        m[3] = tensor_map(qkl + c, 4, qdims, qstr, kbox, 32, true);
        const uint64_t vdims[3] = {(uint64_t)p.wp, (uint64_t)c, (uint64_t)p.rows};
        const uint64_t vstr[2] = {(uint64_t)P * 2, (uint64_t)p.wp * 2};
        const uint32_t vbox[3] = {16, 24, 1};
        m[4] = tensor_map(vth, 3, vdims, vstr, vbox, 32, true);
        m[5] = tensor_map(vtl, 3, vdims, vstr, vbox, 32, true);
        // the output: fp16 pairs [P][c] as (head dim, head, x, y), 24 x 1 x 16 x 8 boxes
        const uint64_t ostr[3] = {(uint64_t)D * 2, (uint64_t)c * 2, (uint64_t)p.wp * c * 2};
        const uint32_t obox[4] = {(uint32_t)D, 1, 16, 8};
        m[6] = tensor_map(out.hi, 4, qdims, ostr, obox, 0, true);
        m[7] = tensor_map(out.lo, 4, qdims, ostr, obox, 0, true);
    }
    k_attn_tc<D, OCA, TERMS, PRE><<<(unsigned)grid, Shape::threads, bytes, st>>>(
        qkv, table, out, gm, c, heads, 1.f / sqrtf((float)D), items, err, m[0], m[1], m[2], m[3], m[4], m[5], m[6],
        m[7]);
    HAT_CUDA(cudaGetLastError());
    count_launch();
}

void launch_attention_tc(int mode, bool oca, const float* qkv, const float* table, Dst out, const Plan& p, int c,
                         int heads, int shift, int* err, cudaStream_t st, bool pre) {
    if (p.win != 16 || p.owin != 24) throw Error(1, "attention: the kernels are built for window 16 / overlap window 24");
    if (heads <= 0 || c % heads) throw Error(1, "attention: c is not divisible by heads");
    const int d = c / heads;
    const bool three = mode == 0;
    if (pre) {
        if (d != 24 || !three || c % 8 || p.tokens() % 8)
            throw Error(1, "attention: the pre-split qkv layout is for parity attention with head dim 24");
        if (oca)
            run_tc<24, true, 3, true>(qkv, table, out, p, c, heads, shift, err, st);
        else
            run_tc<24, false, 3, true>(qkv, table, out, p, c, heads, shift, err, st);
        return;
    }
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
