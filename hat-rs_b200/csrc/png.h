// PNG file I/O around the forward pass (src/image.rs of the reference); see png.cpp.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace hat {

// A planar RGB image: `data` is [3][h][w] float in [0, 1].
struct PngImage {
    int w = 0, h = 0;
    std::vector<float> data;
};

// image::load_rgb_stream (src/image.rs:49-96): 8/16-bit grey, grey + alpha, RGB or RGBA.
PngImage png_decode(const uint8_t* data, size_t len);
// image::load_rgb (src/image.rs:43-47).
PngImage png_load(const std::string& path);
// Image::to_rgb8 (src/image.rs:29-39): clamp to [0, 1], x 255, round half up.
void to_rgb8(const float* planar, int w, int h, uint8_t* rgb);
// image::save_rgb_stream / save_rgb (src/image.rs:99-114): 8-bit RGB.
std::vector<uint8_t> png_encode_rgb8(int w, int h, const uint8_t* rgb);
void png_save_rgb8(const std::string& path, int w, int h, const uint8_t* rgb);

}  // namespace hat
