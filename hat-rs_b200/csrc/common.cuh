// Shared definitions of the B200 HAT backend: error plumbing, the plane geometry and
// the kernel entry points every layer of the scheduler calls.
#pragma once

#include <cuda_runtime.h>
#ifdef __CUDACC__
#include <cuda_fp16.h>
#endif
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

namespace hat {

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// Codes the kernels leave in the device error word. The bounded pipeline waits use small
// numbers (one per wait site, below 64); these two report an operand that fp16 operand
// pairs cannot hold (|x| >= 65504), which the engine answers by redoing the pass on tf32
// pairs.
constexpr int ERR_RANGE_ATTN = 90;  // an attention operand (q, k or v)
constexpr int ERR_RANGE_GEMM = 91;  // a GEMM operand plane written as fp16 pairs

#define HAT_CUDA(call)                                                                   \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess)                                                           \
            throw ::hat::Error(3, std::string(#call) + ": " + cudaGetErrorString(e_));   \
    } while (0)

// The padded geometry of one pass (src/plan.rs:32-113): the plane is padded to a
// window multiple, `shift = win/2`, the OCAB window is `win + win/2` with `opad` on
// each side.
struct Plan {
    int h = 0, w = 0;    // the caller's image
    int hp = 0, wp = 0;  // padded to window multiples
    int win = 16, shift = 8, owin = 24, opad = 4;
    // Strip sharding (one image over several GPUs): this plan computes the padded rows
    // [r0, r1) and holds `halo` rows of each neighbour above and below them, so its
    // planes have `rows` = r1 - r0 + 2 * halo rows (local row i is padded row
    // r0 - halo + i). Unsharded: r0 = 0, r1 = rows = hp, halo = 0.
    int r0 = 0, r1 = 0, halo = 0, rows = 0;
    bool strip() const { return halo > 0; }
    int own() const { return r1 - r0; }
    int gy0() const { return r0 - halo; }  // padded row of local row 0 (may be negative)
    int nx() const { return wp / win; }
    int ny() const { return hp / win; }
    int nw() const { return nx() * ny(); }
    long tokens() const { return (long)rows * wp; }  // tokens of this plan's planes
    static Plan make(int h, int w, int win) {
        Plan p;
        p.h = h;
        p.w = w;
        p.win = win;
        p.hp = (h + win - 1) / win * win;
        p.wp = (w + win - 1) / win * win;
        p.shift = win / 2;
        p.owin = win + win / 2;
        p.opad = (p.owin - win) / 2;
        p.r0 = 0;
        p.r1 = p.rows = p.hp;
        return p;
    }
    // Rank `rank` of `n`: window-aligned row strips as equal as the window rows allow
    // (the first ny % n ranks take one window row more), each with `halo` rows of its
    // neighbours. Every rank needs at least one window row.
    static Plan make_strip(int h, int w, int win, int rank, int n, int halo) {
        Plan p = make(h, w, win);
        const int ny = p.hp / win, base = ny / n, extra = ny % n;
        const int wy0 = rank * base + (rank < extra ? rank : extra);
        const int wy1 = wy0 + base + (rank < extra ? 1 : 0);
        p.r0 = wy0 * win;
        p.r1 = wy1 * win;
        p.halo = halo;
        p.rows = p.r1 - p.r0 + 2 * halo;
        return p;
    }
    bool operator==(const Plan& o) const {
        return h == o.h && w == o.w && hp == o.hp && wp == o.wp && win == o.win && r0 == o.r0 && r1 == o.r1 &&
               halo == o.halo;
    }
};

// ---------------------------------------------------------------- operands
// A GEMM operand plane. In fp32-parity mode every plane a tensor-core GEMM reads is
// stored pre-split by the kernel that produces it, so the GEMM needs no conversion
// pass. Two split kinds:
//  * `h16`: `hi` and `lo` are fp16 arrays (element i at byte 2i, behind the float
//    pointers): hi = fp16(x), lo = fp16(x - hi), 22 significant bits, read by
//    kind::f16 MMAs. Values under fp16's normal range keep an absolute error of at
//    most 2^-25; |x| >= 65504 does not fit and is reported through `err` (ERR_RANGE_GEMM).
//  * otherwise: fp32 arrays, hi = x rounded to tf32 and lo the rounded remainder (see
//    split_tf32), hi + lo within 2^-22 |x| of x, read by kind::tf32 MMAs.
// `lo == nullptr` marks a plain fp32 plane (fast mode, the CUDA-core path, and planes
// read only by CUDA-core code).
struct Opnd {
    const float* hi = nullptr;
    const float* lo = nullptr;
    bool h16 = false;
};
struct Dst {
    float* hi = nullptr;
    float* lo = nullptr;
    bool h16 = false;
    int* err = nullptr;  // h16: set to 21 when a value is beyond fp16's range
};
// The plane starting `i` elements further on (2 bytes per element for an h16 split).
inline Opnd opnd_at(Opnd o, long i) {
    if (o.lo && o.h16)
        return Opnd{reinterpret_cast<const float*>(reinterpret_cast<const char*>(o.hi) + 2 * i),
                    reinterpret_cast<const float*>(reinterpret_cast<const char*>(o.lo) + 2 * i), true};
    return Opnd{o.hi + i, o.lo ? o.lo + i : nullptr, false};
}
inline Dst dst_at(Dst d, long i) {
    if (d.lo && d.h16)
        return Dst{reinterpret_cast<float*>(reinterpret_cast<char*>(d.hi) + 2 * i),
                   reinterpret_cast<float*>(reinterpret_cast<char*>(d.lo) + 2 * i), true, d.err};
    return Dst{d.hi + i, d.lo ? d.lo + i : nullptr, false, d.err};
}

#ifdef __CUDACC__
// x = hi + lo with hi = x rounded to the nearest tf32 value and lo = (x - hi) rounded
// to tf32 as well: both halves are exact tf32 operands, the split is unbiased, and
// hi + lo is within 2^-22 |x| of x. tf32 keeps 10 of fp32's 23 mantissa bits: adding
// half a unit of the 13th bit to the sign-magnitude pattern and clearing the low 13
// bits rounds the magnitude to nearest (ties away from zero), carrying into the
// exponent when the mantissa overflows.
__device__ __forceinline__ float tf32_rna(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    hi = tf32_rna(x);
    lo = tf32_rna(x - hi);
}
// fp16 split: hi = fp16(x) and lo = fp16(x - hi), both rounded to nearest.
__device__ __forceinline__ void split_h16(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(x - __half2float(hi));
}
// The same for a pair, packed (a in the low half): what kind::f16 operands hold.
__device__ __forceinline__ void split_h16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
__device__ __forceinline__ bool beyond_h16(float v) { return fabsf(v) >= 65504.f; }
// GELU, 0.5 x (1 + erf(x / sqrt 2)), with erf from Abramowitz & Stegun 7.1.26 (Hastings'
// rational approximation; |error| of erf at most 1.5e-7 for z >= 0):
//   erfc(z) = (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2),  t = 1 / (1 + p z),
// with p = 0.3275911, a1..a5 = 0.254829592, -0.284496736, 1.421413741, -1.453152027,
// 1.061405429. 1 + erf(x / sqrt 2) is 2 - erfc(z) for x >= 0 and erfc(z) for x < 0, so the
// negative side has no cancellation. exp and the reciprocal are the PTX approximate
// instructions (ex2.approx, rcp.approx; about 2^-22 relative). Against the exact GELU the
// result is within 1e-6 absolute for every finite x (the CUDA self-test checks it over
// [-10, 10]); large |x| give x or 0.
__device__ __forceinline__ float gelu_fast(float x) {
    const float z = fabsf(x) * 0.70710678118654752f;
    float t, e;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, z, 1.f)));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-(z * z) * 1.4426950408889634f));
    const float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f),
                                        -0.284496736f),
                                0.254829592f);
    const float erfc = poly * e;
    return 0.5f * x * (x >= 0.f ? 2.f - erfc : erfc);
}
// Store v at index i of a destination plane, split when it has a lo half.
__device__ __forceinline__ void put(const Dst& d, long i, float v) {
    if (d.lo && d.h16) {
        __half h, l;
        split_h16(v, h, l);
        reinterpret_cast<__half*>(d.hi)[i] = h;
        reinterpret_cast<__half*>(d.lo)[i] = l;
        if (beyond_h16(v) && d.err) atomicCAS(d.err, 0, ERR_RANGE_GEMM);
    } else if (d.lo) {
        float h, l;
        split_tf32(v, h, l);
        d.hi[i] = h;
        d.lo[i] = l;
    } else {
        d.hi[i] = v;
    }
}
// i a multiple of 4.
__device__ __forceinline__ void put4(const Dst& d, long i, float4 v) {
    if (d.lo && d.h16) {
        uint2 h, l;
        split_h16x2(v.x, v.y, h.x, l.x);
        split_h16x2(v.z, v.w, h.y, l.y);
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(d.hi) + i) = h;
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(d.lo) + i) = l;
        if ((beyond_h16(v.x) || beyond_h16(v.y) || beyond_h16(v.z) || beyond_h16(v.w)) && d.err)
            atomicCAS(d.err, 0, ERR_RANGE_GEMM);
    } else if (d.lo) {
        float4 h, l;
        split_tf32(v.x, h.x, l.x);
        split_tf32(v.y, h.y, l.y);
        split_tf32(v.z, h.z, l.z);
        split_tf32(v.w, h.w, l.w);
        *reinterpret_cast<float4*>(d.hi + i) = h;
        *reinterpret_cast<float4*>(d.lo + i) = l;
    } else {
        *reinterpret_cast<float4*>(d.hi + i) = v;
    }
}
// The fp32 value of element i of an operand plane.
__device__ __forceinline__ float get(const Opnd& o, long i) {
    if (o.lo && o.h16)
        return __half2float(reinterpret_cast<const __half*>(o.hi)[i]) +
               __half2float(reinterpret_cast<const __half*>(o.lo)[i]);
    return o.lo ? o.hi[i] + o.lo[i] : o.hi[i];
}
#endif

// ---------------------------------------------------------------- epilogues
// What a GEMM-shaped kernel does with its fp32 accumulator before the store.
enum Act : int { ACT_NONE = 0, ACT_GELU = 1, ACT_LEAKY = 2 };

struct Epi {
    const float* bias = nullptr;   // [n]
    int act = ACT_NONE;            // applied to acc + bias
    // residual: out = res + v, or the HAB sum out = (res + v) + (cx * gate) * cscale
    const float* res = nullptr;    // [m][ldo] (may alias out)
    const float* cx = nullptr;     // [m][ldo] the CAB output (HAB sum only)
    const float* gate = nullptr;   // [n] channel-attention gate (HAB sum only)
    float cscale = 0.f;
    // Channel sums of the stored value (the channel attention's average pool): one
    // partial row [n] per M tile of the launch, written without atomics so the sum
    // (taken by the gate in tile order) is the same on every run.
    float* colsum = nullptr;       // [partial rows][n]; the conv launcher returns the row count
    // Channel stride of the output plane for plain stores (0: the GEMM's n). Columns in
    // [n, ldo) are left as they are (the tensor-core path writes zeros there).
    int ldo = 0;
    // PixelShuffle(r) on store: channel n = c*r*r + i*r + j of pixel (y, x) goes to
    // channel c of pixel (r*y + i, r*x + j) of a [hgt*r][wid*r][n/(r*r)] plane.
    int shuffle = 0;
    // Final store: crop to (oh, ow), `v / img_range + mean[n]`, planar [n][oh][ow]; plane
    // row y is output row y + oy0 (a strip's offset in the whole output).
    int planar_out = 0;
    int oh = 0, ow = 0, oy0 = 0;
    float img_range = 1.f, mean[3] = {0, 0, 0};
    // 3x3 conv: compute the output rows [y_lo, y_hi) only (multiples of 8; 0, 0 = every
    // row); the input plane is still read over its full height, so rows next to the range
    // are real data, not padding. The CUDA-core conv ignores this and computes every row.
    int y_lo = 0, y_hi = 0;
    // The qkv linear of a HAB in fp16 parity mode writes its output straight in the layout
    // the window attention copies from (fp16 hi/lo pairs, M tokens, c = N / 3): q|k hi
    // [M][2c], q|k lo [M][2c], v^T hi [c][M], v^T lo [c][M], one after the other from
    // `qkv_split`, columns below `qcols` (q) multiplied by `qscale`.
    float* qkv_split = nullptr;
    float qscale = 1.f;
    int qcols = 0;
};

// ---------------------------------------------------------------- kernels (launchers)
// All launchers enqueue on `st` and throw hat::Error on a launch failure. `launches`
// counts kernels issued (the reference's `launched()`, src/cuda.rs:542-555).
// Lets kernel `fn` take `bytes` of dynamic shared memory on the current device. Called
// before every launch instead of being cached per device ordinal: the setting belongs to
// the device's context, which cudaDeviceReset (or a different context) replaces.
template <class F>
inline void allow_dyn_smem(F* fn, size_t bytes) {
    HAT_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

extern thread_local uint64_t* g_launch_counter;
inline void count_launch(int n = 1) {
    if (g_launch_counter) *g_launch_counter += n;
}

// planar [3][h][w] in [0,1] → token-major [hp][wp][3], edge-replicated and
// mean-adjusted (src/backend.rs:71-89).
void launch_pre(const float* in, float* out, const Plan& p, const float mean[3], float img_range,
                cudaStream_t st);

// LayerNorm over the channel axis of a [m][c] token plane (src/cpu.rs:563-581).
void launch_layernorm(const float* x, const float* g, const float* b, Dst y, long m, int c, cudaStream_t st);

// Split a plain fp32 array into tf32 hi/lo halves (for callers that hand in fp32 operands).
void launch_split(const float* x, float* hi, float* lo, long n, cudaStream_t st);

// Window attention of one HAB over the [hp][wp][3c] qkv plane (hat_arch.py:165-196):
// the tensor-core kernel (mode: parity / fast), or the CUDA-core one when `simt`.
// `pre`: the qkv buffer holds the qkv linear's attention layout (Epi::qkv_split).
void launch_window_attention(int mode, bool simt, const float* qkv, const float* table, Dst out, const Plan& p,
                             int c, int heads, int shift, int* err, cudaStream_t st, bool pre = false);

// OCAB attention over the [hp][wp][3c] qkv plane (hat_arch.py:392-438).
void launch_overlap_attention(int mode, bool simt, const float* qkv, const float* table, Dst out, const Plan& p,
                              int c, int heads, int* err, cudaStream_t st, bool pre = false);

// The second half of a 3x3 conv computed as a per-tap linear: `taps` is the [hp][wp][ldt]
// plane of Y[p][tap*cout + co] = sum_ci w[co][ci][tap] x[p][ci] (tap = ky*3 + kx), and
// out[p][co] = gelu(bias[co] + sum_tap Y[p + (ky-1, kx-1)][tap*cout + co]) with zero
// padding; channels cout..ldo-1 of `out` are written as zeros. cout <= 8, ldo <= 16.
void launch_tapsum_gelu(const float* taps, int ldt, const float* bias, Dst out, int ldo, int cout, int hp, int wp,
                        int ylo, int yhi, cudaStream_t st);
// Rows [ylo, yhi) of the plane are data; the taps of rows outside are the conv's zero padding.

// sum[c] = the sum of `rows` partial rows [rows][c], in row order.
void launch_rowsum(const float* partial, long rows, int c, float* sum, cudaStream_t st);

// The gate folded into the CAB's second conv and proj (k_proj_cab), written by the gate
// kernel when `hi` is set: hi/lo[n][tap * cinp + ci] (row stride k_pad) = the split of
// cs * gate[n] * w[n][ci][tap] * factor (fp16 pairs when h16, else tf32 pairs; a value
// beyond fp16's range sets ERR_RANGE_GEMM in `err`), and bias[n] = bp[n] + cs * gate[n] * b2[n].
struct CabFold {
    const float* w = nullptr;   // the conv weight [c][cc][3][3]
    const float* b2 = nullptr;  // its bias [c]
    const float* bp = nullptr;  // proj's bias [c]
    float cs = 0.f, factor = 1.f;
    int cc = 0, cinp = 0, k_pad = 0;
    bool h16 = false;
    float* hi = nullptr;
    float* lo = nullptr;
    float* bias = nullptr;
    int* err = nullptr;
};

// gate[c] = sigmoid(W2 relu(W1 mean + b1) + b2) (hat_arch.py:40-57), where the mean
// over the plane is the sum of `rows` partial rows [rows][c] times `inv_count`.
void launch_ca_gate(const float* partial, long rows, float inv_count, const float* w1, const float* b1,
                    const float* w2, const float* b2, float* gate, int c, int sq, cudaStream_t st,
                    const CabFold& fold = CabFold());

// The sum over the output rows [y0, y1) of a 3x3 conv (weight w [c][cc][3][3], bias b) of
// the view x ([vrows][wid][ld], zero outside), computed from x's row and edge sums without
// the conv's output: sum[c]. `stat` is scratch of 3 * cc * (y1 - y0 + 2) floats.
void launch_cab_pool(Opnd x, int ld, int cc, int wid, int vrows, int y0, int y1, float* stat, const float* w,
                     const float* b, int c, float* sum, cudaStream_t st);

}  // namespace hat
