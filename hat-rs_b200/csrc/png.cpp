// PNG decode and encode for the CLI's file path around the forward pass (the role of
// src/image.rs in the reference): decode 8- or 16-bit grey, grey + alpha, RGB or RGBA
// (interlaced or not) into planar float RGB in [0, 1]; encode 8-bit RGB. Host code with
// zlib for the deflate streams; the chunk layout, the CRCs, the five row filters and the
// Adam7 passes follow the PNG specification (ISO/IEC 15948).
#include "png.h"

#include <zlib.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iterator>

#include "common.cuh"

namespace hat {

namespace {

const uint8_t SIG[8] = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1a, '\n'};

uint32_t be32(const uint8_t* p) { return (uint32_t)p[0] << 24 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 8 | p[3]; }

void put32(std::vector<uint8_t>& v, uint32_t x) {
    v.push_back((uint8_t)(x >> 24));
    v.push_back((uint8_t)(x >> 16));
    v.push_back((uint8_t)(x >> 8));
    v.push_back((uint8_t)x);
}

// Paeth predictor (PNG specification, filter type 4).
inline int paeth(int a, int b, int c) {
    const int p = a + b - c, pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
    if (pa <= pb && pa <= pc) return a;
    return pb <= pc ? b : c;
}

// Undoes the row filters of one (sub-)image of `rows` rows of `rowbytes` bytes, each
// row preceded by its filter type byte; `bpp` is the filter's byte distance.
void unfilter(const uint8_t* in, uint8_t* out, size_t rows, size_t rowbytes, size_t bpp) {
    const uint8_t* prev = nullptr;
    for (size_t y = 0; y < rows; ++y) {
        const uint8_t ft = in[y * (rowbytes + 1)];
        const uint8_t* src = in + y * (rowbytes + 1) + 1;
        uint8_t* dst = out + y * rowbytes;
        for (size_t i = 0; i < rowbytes; ++i) {
            const int a = i >= bpp ? dst[i - bpp] : 0;
            const int b = prev ? prev[i] : 0;
            const int c = prev && i >= bpp ? prev[i - bpp] : 0;
            int v = src[i];
            switch (ft) {
                case 0: break;
                case 1: v += a; break;
                case 2: v += b; break;
                case 3: v += (a + b) >> 1; break;
                case 4: v += paeth(a, b, c); break;
                default: throw Error(2, "png: unknown row filter type " + std::to_string(ft));
            }
            dst[i] = (uint8_t)v;
        }
        prev = dst;
    }
}

std::vector<uint8_t> inflate_all(const std::vector<uint8_t>& z, size_t expect) {
    std::vector<uint8_t> out(expect);
    z_stream s;
    memset(&s, 0, sizeof s);
    if (inflateInit(&s) != Z_OK) throw Error(2, "png: zlib inflateInit failed");
    s.next_in = const_cast<Bytef*>(z.data());
    s.avail_in = (uInt)z.size();
    s.next_out = out.data();
    s.avail_out = (uInt)out.size();
    const int r = inflate(&s, Z_FINISH);
    const size_t got = out.size() - s.avail_out;
    inflateEnd(&s);
    if (r != Z_STREAM_END && !(r == Z_BUF_ERROR && got == expect))
        throw Error(2, std::string("png: corrupt image data (zlib: ") + (s.msg ? s.msg : std::to_string(r)) + ")");
    if (got != expect) throw Error(2, "png: image data is shorter than the header says");
    return out;
}

// Adam7: pass p covers pixels (x0 + k*dx, y0 + j*dy).
const int A7[7][4] = {{0, 0, 8, 8}, {4, 0, 8, 8}, {0, 4, 4, 8}, {2, 0, 4, 4}, {0, 2, 2, 4}, {1, 0, 2, 2}, {0, 1, 1, 2}};

}  // namespace

PngImage png_decode(const uint8_t* data, size_t len) {
    if (len < 8 || memcmp(data, SIG, 8) != 0) throw Error(2, "png: not a PNG file (bad signature)");
    size_t pos = 8;
    uint32_t w = 0, h = 0;
    int depth = 0, ctype = -1, interlace = 0;
    bool have_ihdr = false, ended = false;
    std::vector<uint8_t> z;
    while (pos + 12 <= len && !ended) {
        const uint32_t n = be32(data + pos);
        if (n > len - pos - 12) throw Error(2, "png: truncated chunk");
        const uint8_t* type = data + pos + 4;
        const uint8_t* body = data + pos + 8;
        const uint32_t crc = be32(body + n);
        if ((uint32_t)crc32(crc32(0L, Z_NULL, 0), type, n + 4) != crc)
            throw Error(2, std::string("png: CRC mismatch in chunk ") + std::string((const char*)type, 4));
        if (!memcmp(type, "IHDR", 4)) {
            if (n != 13) throw Error(2, "png: bad IHDR");
            w = be32(body);
            h = be32(body + 4);
            depth = body[8];
            ctype = body[9];
            if (body[10] != 0 || body[11] != 0) throw Error(2, "png: unknown compression or filter method");
            interlace = body[12];
            if (interlace > 1) throw Error(2, "png: unknown interlace method");
            have_ihdr = true;
        } else if (!memcmp(type, "IDAT", 4)) {
            z.insert(z.end(), body, body + n);
        } else if (!memcmp(type, "IEND", 4)) {
            ended = true;
        } else if (!have_ihdr) {
            throw Error(2, "png: first chunk is not IHDR");
        }
        pos += 12 + n;
    }
    if (!have_ihdr) throw Error(2, "png: no IHDR chunk");
    if (w == 0 || h == 0 || w > (1u << 20) || h > (1u << 20)) throw Error(2, "png: bad image size");
    int channels = 0;
    switch (ctype) {
        case 0: channels = 1; break;
        case 4: channels = 2; break;
        case 2: channels = 3; break;
        case 6: channels = 4; break;
        case 3: throw Error(2, "unsupported png colour type Indexed");
        default: throw Error(2, "png: unknown colour type " + std::to_string(ctype));
    }
    if (depth != 8 && depth != 16) throw Error(2, "unsupported png bit depth " + std::to_string(depth));
    if (z.empty()) throw Error(2, "png: no image data");
    const size_t bps = depth / 8, bpp = channels * bps;
    // The filtered byte stream: one sub-image per Adam7 pass, or the whole image.
    std::vector<uint8_t> px((size_t)w * h * bpp);
    if (!interlace) {
        const size_t rowbytes = (size_t)w * bpp;
        const std::vector<uint8_t> raw = inflate_all(z, (size_t)h * (rowbytes + 1));
        unfilter(raw.data(), px.data(), h, rowbytes, bpp);
    } else {
        size_t total = 0;
        size_t pw[7], ph[7];
        for (int p = 0; p < 7; ++p) {
            pw[p] = w > (uint32_t)A7[p][0] ? (w - A7[p][0] + A7[p][2] - 1) / A7[p][2] : 0;
            ph[p] = h > (uint32_t)A7[p][1] ? (h - A7[p][1] + A7[p][3] - 1) / A7[p][3] : 0;
            if (pw[p] && ph[p]) total += ph[p] * (pw[p] * bpp + 1);
        }
        const std::vector<uint8_t> raw = inflate_all(z, total);
        size_t off = 0;
        std::vector<uint8_t> sub;
        for (int p = 0; p < 7; ++p) {
            if (!pw[p] || !ph[p]) continue;
            const size_t rowbytes = pw[p] * bpp;
            sub.assign(ph[p] * rowbytes, 0);
            unfilter(raw.data() + off, sub.data(), ph[p], rowbytes, bpp);
            off += ph[p] * (rowbytes + 1);
            for (size_t j = 0; j < ph[p]; ++j)
                for (size_t k = 0; k < pw[p]; ++k) {
                    const size_t x = A7[p][0] + k * A7[p][2], y = A7[p][1] + j * A7[p][3];
                    memcpy(&px[(y * w + x) * bpp], &sub[(j * pw[p] + k) * bpp], bpp);
                }
        }
    }
    // Planar RGB in [0, 1]: grey replicated, alpha dropped (src/image.rs:55-96).
    PngImage img;
    img.w = (int)w;
    img.h = (int)h;
    img.data.resize((size_t)3 * w * h);
    const size_t hw = (size_t)w * h;
    const float sc = depth == 16 ? 1.f / 65535.f : 1.f / 255.f;
    for (size_t i = 0; i < hw; ++i) {
        auto sample = [&](int c) -> float {
            const uint8_t* s = &px[i * bpp + c * bps];
            return (depth == 16 ? (float)((uint32_t)s[0] << 8 | s[1]) : (float)s[0]) * sc;
        };
        if (channels <= 2) {
            const float v = sample(0);
            img.data[i] = img.data[hw + i] = img.data[2 * hw + i] = v;
        } else {
            img.data[i] = sample(0);
            img.data[hw + i] = sample(1);
            img.data[2 * hw + i] = sample(2);
        }
    }
    return img;
}

PngImage png_load(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw Error(2, "open " + path + ": cannot read the file");
    std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    try {
        return png_decode(bytes.data(), bytes.size());
    } catch (const Error& e) {
        throw Error(e.code, path + ": " + e.what());
    }
}

void to_rgb8(const float* planar, int w, int h, uint8_t* rgb) {
    const size_t hw = (size_t)w * h;
    for (size_t i = 0; i < hw; ++i)
        for (int c = 0; c < 3; ++c) {
            float v = planar[c * hw + i];
            v = (v < 0.f ? 0.f : v > 1.f ? 1.f : v) * 255.f;
            const float r = std::floor(v + 0.5f);
            // min(r, 255) where a NaN operand yields the other one, as Rust's f32::min does:
            // a NaN pixel becomes 255
            rgb[i * 3 + c] = (uint8_t)(std::isnan(r) || r > 255.f ? 255.f : r);
        }
}

std::vector<uint8_t> png_encode_rgb8(int w, int h, const uint8_t* rgb) {
    if (w <= 0 || h <= 0) throw Error(1, "png: empty image");
    const size_t rowbytes = (size_t)w * 3;
    // Every row with the Sub filter (type 1): neighbouring pixels of natural images are
    // alike, so the differences deflate well.
    std::vector<uint8_t> raw((size_t)h * (rowbytes + 1));
    for (int y = 0; y < h; ++y) {
        uint8_t* d = &raw[(size_t)y * (rowbytes + 1)];
        const uint8_t* s = rgb + (size_t)y * rowbytes;
        d[0] = 1;
        for (size_t i = 0; i < rowbytes; ++i) d[1 + i] = (uint8_t)(s[i] - (i >= 3 ? s[i - 3] : 0));
    }
    uLongf zlen = compressBound((uLong)raw.size());
    std::vector<uint8_t> zd(zlen);
    if (compress2(zd.data(), &zlen, raw.data(), (uLong)raw.size(), 6) != Z_OK)
        throw Error(3, "png: zlib compress failed");
    zd.resize(zlen);
    std::vector<uint8_t> out(SIG, SIG + 8);
    auto chunk = [&](const char* type, const uint8_t* body, size_t n) {
        put32(out, (uint32_t)n);
        const size_t at = out.size();
        out.insert(out.end(), type, type + 4);
        out.insert(out.end(), body, body + n);
        put32(out, (uint32_t)crc32(crc32(0L, Z_NULL, 0), &out[at], (uInt)(n + 4)));
    };
    std::vector<uint8_t> ihdr;
    put32(ihdr, (uint32_t)w);
    put32(ihdr, (uint32_t)h);
    const uint8_t rest[5] = {8, 2, 0, 0, 0};  // 8-bit RGB, deflate, adaptive filters, no interlace
    ihdr.insert(ihdr.end(), rest, rest + 5);
    chunk("IHDR", ihdr.data(), ihdr.size());
    chunk("IDAT", zd.data(), zd.size());
    chunk("IEND", nullptr, 0);
    return out;
}

void png_save_rgb8(const std::string& path, int w, int h, const uint8_t* rgb) {
    const std::vector<uint8_t> bytes = png_encode_rgb8(w, h, rgb);
    FILE* f = fopen(path.c_str(), "wb");
    if (!f) throw Error(2, "create " + path + ": cannot write the file");
    const size_t n = fwrite(bytes.data(), 1, bytes.size(), f);
    const int rc = fclose(f);
    if (n != bytes.size() || rc != 0) throw Error(2, path + ": write failed");
}

}  // namespace hat
