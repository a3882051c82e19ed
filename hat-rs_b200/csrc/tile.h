// The tile loop for images too large for one pass (src/tile.rs of hat-rs): window-
// aligned cores, each run as its own forward on the core plus a margin of context, the
// cores copied into the output without blending.
#pragma once

#include <cstdint>
#include <optional>

namespace hat {

class Engine;

struct Tiling {
    int tile = 0, margin = 0, scale = 0, tiles = 0;
    int largest_h = 0, largest_w = 0;  // the largest sub-image a forward ran on
};

// tile::forward (src/tile.rs:47-105): `in` planar [3][h][w], `out` planar
// [3][h*scale][w*scale], both on the host. `tile` and `margin` are rounded up to the
// window (the tile to at least one window); a tile's margin is clamped to the image.
Tiling tile_forward(Engine& e, int h, int w, const float* in, float* out, int tile, int margin);

// tile::auto_tile (src/tile.rs:147-184): the largest window-multiple core whose
// sub-image (core + 2 margin) fits `budget_bytes` at `per_pixel_floats` per pixel plus
// `constant_floats`, capped at the image; nullopt when not even one window fits.
std::optional<int> auto_tile(int h, int w, int win, uint64_t budget_bytes, uint64_t per_pixel_floats,
                             uint64_t constant_floats, int margin);

// gpu_auto_tile (src/main.rs:107-140): halving from the larger image side down to the
// window until the memory guard admits a pass of that size on the engine's device;
// nullopt when one window does not fit.
std::optional<int> gpu_auto_tile(const Engine& e, int h, int w);

}  // namespace hat
