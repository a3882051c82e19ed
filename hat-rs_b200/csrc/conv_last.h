// conv_last as a bandwidth kernel (k_conv_last.cu): 64 -> 3 channels, 3x3, fp32 FMAs,
// planar output with the crop and denormalisation of Pre::finish.
#pragma once

#include "common.cuh"

namespace hat {

constexpr int CL_CIN = 64;

// Whether the kernel takes this conv: 64 input channels, 3 outputs, aligned planes.
bool conv_last_ok(const Opnd& x, int cin, int cout);
// The conv over the input view [hgt][wid][64] (zero outside it), output rows
// [e.y_lo, e.y_hi) of the view (all when equal), stored planar into `out` with e.oh, e.ow,
// e.oy0, e.img_range and e.mean as Epi describes.
// `w` is the device copy of the PyTorch [3][64][3][3] weight, `bias` its [3] bias.
long launch_conv_last(const Opnd& x, const float* w, const float* bias, float* out, int hgt, int wid, const Epi& e,
                      cudaStream_t st);

}  // namespace hat
