// The tile loop (see tile.h).
#include "tile.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <tuple>
#include <vector>

#include "engine.h"

namespace hat {

static int round_up(int v, int to) { return to <= 0 ? v : (v + to - 1) / to * to; }

Tiling tile_forward(Engine& e, int h, int w, const float* in, float* out, int tile, int margin) {
    if (h <= 0 || w <= 0 || !in || !out) throw Error(1, "tile: empty image or null buffer");
    const int win = e.weights().window, s = e.weights().scale;
    Tiling t;
    t.tile = std::max(round_up(tile, win), win);
    t.margin = round_up(std::max(margin, 0), win);
    t.scale = s;
    const long oh = (long)h * s, ow = (long)w * s;
    // The tiles, run grouped by sub-image size so that each size is planned once (a
    // smaller sub-image reuses the device arena of a larger one).
    struct Job {
        int y0, x0, y1, x1, sy0, sx0, sy1, sx1;
    };
    std::vector<Job> jobs;
    for (int y0 = 0; y0 < h; y0 += t.tile)
        for (int x0 = 0; x0 < w; x0 += t.tile) {
            Job j;
            j.y0 = y0;
            j.x0 = x0;
            j.y1 = std::min(y0 + t.tile, h);
            j.x1 = std::min(x0 + t.tile, w);
            j.sy0 = std::max(y0 - t.margin, 0);
            j.sx0 = std::max(x0 - t.margin, 0);
            j.sy1 = std::min(j.y1 + t.margin, h);
            j.sx1 = std::min(j.x1 + t.margin, w);
            jobs.push_back(j);
        }
    std::stable_sort(jobs.begin(), jobs.end(), [](const Job& a, const Job& b) {
        return std::make_tuple(-(a.sy1 - a.sy0) * (a.sx1 - a.sx0), a.sy1 - a.sy0) <
               std::make_tuple(-(b.sy1 - b.sy0) * (b.sx1 - b.sx0), b.sy1 - b.sy0);
    });
    std::vector<float> sub, res;
    for (const Job& j : jobs) {
        const int sh = j.sy1 - j.sy0, sw = j.sx1 - j.sx0;
        t.largest_h = std::max(t.largest_h, sh);
        t.largest_w = std::max(t.largest_w, sw);
        // crop (src/tile.rs:113-125): the sub-image's three planes
        sub.resize((size_t)3 * sh * sw);
        for (int c = 0; c < 3; ++c)
            for (int y = 0; y < sh; ++y)
                memcpy(&sub[((size_t)c * sh + y) * sw], in + ((size_t)c * h + j.sy0 + y) * w + j.sx0,
                       sizeof(float) * sw);
        res.resize((size_t)3 * sh * s * sw * s);
        e.forward_host(1, sh, sw, sub.data(), res.data());
        // Copy the core, not the margin, to its place in the output.
        const int dy0 = (j.y0 - j.sy0) * s, dx0 = (j.x0 - j.sx0) * s;
        const int ch = (j.y1 - j.y0) * s, cw = (j.x1 - j.x0) * s;
        for (int c = 0; c < 3; ++c)
            for (int y = 0; y < ch; ++y)
                memcpy(out + ((size_t)c * oh + (size_t)j.y0 * s + y) * ow + (size_t)j.x0 * s,
                       &res[((size_t)c * sh * s + dy0 + y) * sw * s + dx0], sizeof(float) * cw);
        ++t.tiles;
    }
    return t;
}

std::optional<int> auto_tile(int h, int w, int win, uint64_t budget_bytes, uint64_t per_pixel_floats,
                             uint64_t constant_floats, int margin) {
    const uint64_t bytes_per_pixel = std::max<uint64_t>(per_pixel_floats, 1) * 4;
    const uint64_t constant = constant_floats * 4;
    // The sub-image a core runs on is the core plus the margin on both sides, so that
    // is what has to fit.
    const uint64_t halo = 2 * (uint64_t)margin;
    const uint64_t one_window = ((uint64_t)win + halo) * ((uint64_t)win + halo) * bytes_per_pixel + constant;
    if (budget_bytes < one_window) return std::nullopt;
    const uint64_t pixels = (budget_bytes - constant) / bytes_per_pixel;
    const uint64_t side = (uint64_t)std::sqrt((double)pixels);
    const uint64_t core = side > halo ? side - halo : 0;
    int t = (int)std::max<uint64_t>(core / win * win, (uint64_t)win);
    return std::min(t, std::max(h, w));
}

std::optional<int> gpu_auto_tile(const Engine& e, int h, int w) {
    const int win = e.weights().window;
    const int start = std::max(std::max(w, h), win);
    int t = start;
    while (true) {
        bool fits = true;
        try {
            e.check_memory(t, t);
        } catch (const Error& err) {
            if (err.code != 4) throw;
            fits = false;
        }
        if (fits) return t;
        if (t <= win) return std::nullopt;
        t = std::max(t / 2, win);
    }
}

}  // namespace hat
