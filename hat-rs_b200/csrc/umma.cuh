// Weights prepared for the GEMM kernels, and the GEMM launchers (tensor-core and
// CUDA-core).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace hat {

// A Linear or 3x3 Conv2d weight in the layouts the kernels read.
//  * `simt`: linear [n][k]; conv [n][9][cin] (tap-major K).
//  * `hi`/`lo`: the tensor-core B operand [n_pad][k_pad], K-major, zero padded, split
//    the way the operand planes it multiplies are (see Opnd): tf32 pairs, or (`h16`)
//    fp16 pairs of the weight times 2^e, with e chosen so that the largest |w| lands in
//    [2^14, 2^15) and `scale` = 2^-e undoing it in the epilogue (a power of two: exact).
//    For a conv, K = 9 taps x `cinp` channels, `cinp` a multiple of the channel chunk
//    one k-block of a tap covers (`ckb` bytes: 128, or 32 for narrow inputs).
struct GemmW {
    const float* simt = nullptr;
    const float* hi = nullptr;
    const float* lo = nullptr;
    int n = 0, k = 0;       // k = 9 * cin for a conv
    bool conv = false;
    int cin = 0;            // conv input channels
    int cin_plane = 0;      // channel stride of the conv's input plane (>= cin)
    int cinp = 0;           // conv channels per tap in the tensor-core K layout
    int ckb = 128;          // bytes of K per k-block row
    int bn = 0, n_pad = 0, k_pad = 0;
    bool umma = false;      // tensor-core layout present
    bool h16 = false;       // fp16 split (kind::f16) rather than tf32 (kind::tf32)
    float scale = 1.f;      // h16: the accumulator's factor (2^-e)
};


// Columns per tensor-core tile for an output width n: at most 192 (so three pipeline
// stages fit in shared memory for c = 144), a multiple of 16, tiles of equal width.
inline int umma_bn(int n) {
    int tiles = (n + 191) / 192;
    int per = (n + tiles - 1) / tiles;
    return (per + 15) / 16 * 16;
}

// Device-side weight preparation (k_prep.cu). `w` is the PyTorch layout on the device;
// the outputs are allocated by the caller with the sizes `plan_gemm_w` sets.
void plan_gemm_w(GemmW& g, int n, int k_or_cin, bool conv, int cin_plane, bool h16 = false);
// The power of two 2^e that puts max|w| in [2^14, 2^15) (1 for an all-zero weight).
float h16_weight_factor(float max_abs);
size_t gemm_w_floats(const GemmW& g);  // simt + hi + lo floats
void launch_prep_gemm_w(const float* w, float* simt, float* hi, float* lo, const GemmW& g, cudaStream_t st);
// [cout][cin][3][3] conv weights -> the per-tap linear [9*cout][cin] (row tap*cout + co).
void launch_prep_taps(const float* w, float* out, int cout, int cin, cudaStream_t st);

// Tensor-core launchers (`x.lo` required in parity mode, split the same way as the
// weight: `x.h16 == w.h16`); return the number of
// channel-sum partial rows written when `e.colsum` is set.
// cuTensorMapEncodeTiled over `rank` dims (innermost first) with the given byte strides of
// dims 1.., box and swizzle row width (128, 64, 32 or 0 bytes); fp16 elements when h16.
CUtensorMap tensor_map(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                       const uint32_t* box, int rowbytes, bool h16);

long umma_linear(int mode, Opnd x, const GemmW& w, Dst y, long m, const Epi& e, int* err, cudaStream_t st);
long umma_conv3x3(int mode, Opnd x, const GemmW& w, Dst y, int hgt, int wid, const Epi& e, int* err,
                  cudaStream_t st);

// The HAB / OCAB MLP fused into one tensor-core launch: y = res + b2 + w2 . GELU(w1 . x + b1),
// the hidden activations kept on chip (k_umma.cu, k_mlp). `umma_mlp_ok` says whether the
// two weights' tensor-core layouts allow it (hidden width a multiple of 96 after padding,
// output width at most 224); `res` may alias `y.hi`.
bool umma_mlp_ok(const GemmW& w1, const GemmW& w2);
long umma_mlp(int mode, Opnd x, const GemmW& w1, const float* b1, const GemmW& w2, const float* b2, const float* res,
              Dst y, long m, int* err, cudaStream_t st);

// The HAB's proj linear with the CAB's second conv folded in (k_umma.cu, k_proj_cab):
//   out = res + bias + wp . attn + W2' (*) cmid
// over output rows [y_lo, y_hi) of the [rows][wid][*] planes. W2' (`w2hi`/`w2lo`) is
// the conv weight `w2`'s tensor-core layout with each output row scaled by its gate and
// conv_scale and by proj's power-of-two factor (k_ca_gate writes it); `cmid` is the view
// of cm_rows rows starting at plane row cm_lo (zeros outside it), channel stride cm_ld.
bool umma_proj_cab_ok(const GemmW& wp, const GemmW& w2);
long umma_proj_cab(int mode, Opnd attn, const GemmW& wp, Opnd cmid, int cm_ld, int cm_rows, int cm_lo,
                   const GemmW& w2, const float* w2hi, const float* w2lo, const float* bias, const float* res,
                   float* out, int rows, int wid, int y_lo, int y_hi, int* err, cudaStream_t st);

// CUDA-core launchers (read hi + lo when the operand is split); same return value.
long simt_linear(Opnd x, const GemmW& w, Dst y, long m, const Epi& e, cudaStream_t st);
long simt_conv3x3(Opnd x, const GemmW& w, Dst y, int hgt, int wid, const Epi& e, cudaStream_t st);

// What the engine calls: the tensor-core kernel when the shape allows it and
// `simt_only` is false, else the CUDA-core kernel.
struct GemmCtx {
    int mode = 0;
    bool simt_only = false;
    int* err = nullptr;   // device error flag of the tensor-core kernels' bounded waits
};
long gemm_linear(const GemmCtx& c, Opnd x, const GemmW& w, Dst y, long m, const Epi& e, cudaStream_t st);
long gemm_conv3x3(const GemmCtx& c, Opnd x, const GemmW& w, Dst y, int hgt, int wid, const Epi& e,
                  cudaStream_t st);

}  // namespace hat
