// Safetensors reader and checkpoint validation. Host-only; no device access, so a
// checkpoint can be inspected on a machine without a GPU.
#include "weights.h"

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <sstream>

#include "common.cuh"

namespace hat {

namespace {

// Just enough JSON for a safetensors header: objects, arrays, strings, numbers.
struct Json {
    enum Kind { NUL, NUM, STR, ARR, OBJ } kind = NUL;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
};

struct Parser {
    const char* p;
    const char* end;
    [[noreturn]] void fail(const char* what) {
        throw Error(2, std::string("safetensors header: ") + what);
    }
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    std::string string() {
        if (p >= end || *p != '"') fail("expected a string");
        ++p;
        std::string s;
        while (p < end && *p != '"') {
            if (*p == '\\') {
                ++p;
                if (p >= end) fail("bad escape");
                char c = *p;
                if (c == 'n') s += '\n';
                else if (c == 't') s += '\t';
                else if (c == 'u') {
                    if (end - p < 5) fail("bad \\u escape");
                    unsigned v = (unsigned)strtoul(std::string(p + 1, p + 5).c_str(), nullptr, 16);
                    if (v < 0x80) s += (char)v; else s += '?';
                    p += 4;
                } else s += c;
                ++p;
            } else {
                s += *p++;
            }
        }
        if (p >= end) fail("unterminated string");
        ++p;
        return s;
    }
    Json value() {
        ws();
        if (p >= end) fail("unexpected end");
        Json j;
        if (*p == '{') {
            j.kind = Json::OBJ;
            ++p;
            ws();
            if (p < end && *p == '}') { ++p; return j; }
            for (;;) {
                ws();
                std::string k = string();
                ws();
                if (p >= end || *p != ':') fail("expected ':'");
                ++p;
                j.obj.emplace_back(k, value());
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == '}') { ++p; break; }
                fail("expected ',' or '}'");
            }
        } else if (*p == '[') {
            j.kind = Json::ARR;
            ++p;
            ws();
            if (p < end && *p == ']') { ++p; return j; }
            for (;;) {
                j.arr.push_back(value());
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == ']') { ++p; break; }
                fail("expected ',' or ']'");
            }
        } else if (*p == '"') {
            j.kind = Json::STR;
            j.str = string();
        } else {
            char* e = nullptr;
            j.num = strtod(p, &e);
            if (e == p) fail("bad number");
            j.kind = Json::NUM;
            p = e;
        }
        return j;
    }
};

}  // namespace

void SafeTensors::open(const std::string& path) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) throw Error(2, path + ": " + strerror(errno));
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (n < 8) { fclose(f); throw Error(2, path + ": too short to be a safetensors file"); }
    bytes.resize((size_t)n);
    size_t got = fread(bytes.data(), 1, (size_t)n, f);
    fclose(f);
    if (got != (size_t)n) throw Error(2, path + ": short read");
    uint64_t hlen = 0;
    memcpy(&hlen, bytes.data(), 8);
    if (hlen > (uint64_t)n - 8) throw Error(2, path + ": header length past the end of the file");
    Parser ps{(const char*)bytes.data() + 8, (const char*)bytes.data() + 8 + hlen};
    Json root = ps.value();
    if (root.kind != Json::OBJ) throw Error(2, path + ": header is not an object");
    data_off = 8 + hlen;
    uint64_t data_len = (uint64_t)n - data_off;
    for (auto& kv : root.obj) {
        if (kv.first == "__metadata__") {
            for (auto& m : kv.second.obj)
                if (m.second.kind == Json::STR) meta[m.first] = m.second.str;
            continue;
        }
        const Json& t = kv.second;
        TensorInfo ti;
        for (auto& f2 : t.obj) {
            if (f2.first == "dtype") ti.dtype = f2.second.str;
            else if (f2.first == "shape") for (auto& d : f2.second.arr) ti.shape.push_back((int64_t)d.num);
            else if (f2.first == "data_offsets" && f2.second.arr.size() == 2) {
                ti.begin = (uint64_t)f2.second.arr[0].num;
                ti.end = (uint64_t)f2.second.arr[1].num;
            }
        }
        int64_t esize = ti.dtype == "F32" ? 4 : ti.dtype == "I64" ? 8 : 0;
        if (esize && ti.end > data_len)
            throw Error(2, path + ": `" + kv.first + "` runs past the end of the file");
        if (esize && (int64_t)(ti.end - ti.begin) != ti.numel() * esize)
            throw Error(2, path + ": `" + kv.first + "` byte range does not match its shape");
        tensors[kv.first] = ti;
        order.push_back(kv.first);
    }
}

const float* SafeTensors::f32(const std::string& name) const {
    auto it = tensors.find(name);
    if (it == tensors.end()) throw Error(2, "no tensor `" + name + "`");
    if (it->second.dtype != "F32") throw Error(2, "`" + name + "` is " + it->second.dtype + ", not F32");
    return reinterpret_cast<const float*>(bytes.data() + data_off + it->second.begin);
}

std::vector<int64_t> SafeTensors::i64(const std::string& name) const {
    auto it = tensors.find(name);
    if (it == tensors.end()) throw Error(2, "no tensor `" + name + "`");
    if (it->second.dtype != "I64") throw Error(2, "`" + name + "` is not int64");
    std::vector<int64_t> v((size_t)it->second.numel());
    memcpy(v.data(), bytes.data() + data_off + it->second.begin, v.size() * 8);
    return v;
}

std::vector<int64_t> Weights::shape(const std::string& name) const {
    auto it = st.tensors.find(name);
    if (it == st.tensors.end()) throw Error(2, "no tensor `" + name + "`");
    return it->second.shape;
}

std::vector<std::pair<int, int>> Weights::up_blocks() const {
    if (scale == 3) return {{3, 9 * head_feat}};
    int s = scale, n = 0;
    while (s > 1 && s % 2 == 0) { s /= 2; ++n; }
    if (s != 1 || n == 0) return {};
    return std::vector<std::pair<int, int>>(n, {2, 4 * head_feat});
}

static std::string shape_str(const std::vector<int64_t>& s) {
    std::ostringstream o;
    o << "[";
    for (size_t i = 0; i < s.size(); ++i) o << (i ? ", " : "") << s[i];
    o << "]";
    return o.str();
}

void Weights::load(const std::string& path) {
    st.open(path);
    static const char* keys[] = {"variant", "scale", "window_size", "overlap_ratio", "embed_dim",
                                 "num_heads", "mlp_ratio", "depths", "compress_ratio",
                                 "squeeze_factor", "conv_scale", "img_range", "rgb_mean", "source"};
    for (const char* k : keys)
        if (!st.meta.count(k))
            throw Error(2, path + ": no `" + k + "` in __metadata__ - convert the checkpoint with "
                           "tools/convert.py, which records the architecture; a plain state_dict "
                           "cannot be checked");
    auto num = [&](const char* k) -> int {
        char* e = nullptr;
        long v = strtol(st.meta[k].c_str(), &e, 10);
        if (e == st.meta[k].c_str() || *e) throw Error(2, path + ": `" + k + "` = \"" + st.meta[k] + "\" is not an integer");
        return (int)v;
    };
    variant = st.meta["variant"];
    scale = num("scale");
    window = num("window_size");
    embed = num("embed_dim");
    heads = num("num_heads");
    mlp_ratio = num("mlp_ratio");
    if (heads <= 0 || embed % heads)
        throw Error(2, "embed_dim " + std::to_string(embed) + " is not divisible by num_heads " + std::to_string(heads));
    head_dim = embed / heads;
    float overlap = strtof(st.meta["overlap_ratio"].c_str(), nullptr);
    // int(window * overlap) + window: a truncation, as the reference writes it.
    owin = window + (int)((float)window * overlap);
    {
        std::stringstream ss(st.meta["depths"]);
        std::string item;
        depths.clear();
        while (std::getline(ss, item, ',')) depths.push_back(atoi(item.c_str()));
    }
    int cr = num("compress_ratio"), sf = num("squeeze_factor");
    if (cr <= 0 || sf <= 0) throw Error(2, "compress_ratio / squeeze_factor must be positive");
    compressed = embed / cr;
    squeezed = embed / sf;
    conv_scale = strtof(st.meta["conv_scale"].c_str(), nullptr);
    img_range = strtof(st.meta["img_range"].c_str(), nullptr);
    {
        std::stringstream ss(st.meta["rgb_mean"]);
        std::string item;
        int i = 0;
        while (std::getline(ss, item, ',')) {
            if (i < 3) mean[i] = strtof(item.c_str(), nullptr);
            ++i;
        }
        if (i != 3) throw Error(2, "rgb_mean has " + std::to_string(i) + " entries, expected 3");
    }
    if (!has("conv_before_upsample.0.weight")) throw Error(2, path + ": no `conv_before_upsample.0.weight`");
    head_feat = (int)shape("conv_before_upsample.0.weight")[0];

    // validate (src/weights.rs:133-265): every tensor the graph reads, with its shape.
    const int64_t c = embed, hd = heads;
    std::vector<std::pair<std::string, std::vector<int64_t>>> want = {
        {"conv_first.weight", {c, 3, 3, 3}}, {"conv_first.bias", {c}},
        {"conv_after_body.weight", {c, c, 3, 3}}, {"conv_after_body.bias", {c}},
        {"norm.weight", {c}}, {"norm.bias", {c}},
        {"patch_embed.norm.weight", {c}}, {"patch_embed.norm.bias", {c}},
        {"relative_position_index_SA", {(int64_t)window * window, (int64_t)window * window}},
        {"relative_position_index_OCA", {(int64_t)window * window, (int64_t)owin * owin}},
        {"conv_before_upsample.0.weight", {head_feat, c, 3, 3}},
        {"conv_before_upsample.0.bias", {head_feat}},
    };
    auto blocks = up_blocks();
    if (blocks.empty())
        throw Error(2, "scale " + std::to_string(scale) + " is not one the reference's own `Upsample` "
                       "builds: it accepts a power of two and 3");
    for (size_t o = 0; o < blocks.size(); ++o) {
        want.push_back({"upsample." + std::to_string(2 * o) + ".weight", {blocks[o].second, head_feat, 3, 3}});
        want.push_back({"upsample." + std::to_string(2 * o) + ".bias", {blocks[o].second}});
    }
    want.push_back({"conv_last.weight", {3, head_feat, 3, 3}});
    want.push_back({"conv_last.bias", {3}});
    const int64_t mr = mlp_ratio, cc = compressed, sq = squeezed;
    const int64_t tsa = (2 * window - 1) * (2 * window - 1), toca = (int64_t)(window + owin - 1) * (window + owin - 1);
    for (size_t l = 0; l < depths.size(); ++l) {
        std::string L = "layers." + std::to_string(l);
        want.push_back({L + ".conv.weight", {c, c, 3, 3}});
        want.push_back({L + ".conv.bias", {c}});
        for (int b = 0; b < depths[l]; ++b) {
            std::string p = L + ".residual_group.blocks." + std::to_string(b);
            want.push_back({p + ".norm1.weight", {c}});
            want.push_back({p + ".norm1.bias", {c}});
            want.push_back({p + ".norm2.weight", {c}});
            want.push_back({p + ".norm2.bias", {c}});
            want.push_back({p + ".attn.qkv.weight", {3 * c, c}});
            want.push_back({p + ".attn.qkv.bias", {3 * c}});
            want.push_back({p + ".attn.proj.weight", {c, c}});
            want.push_back({p + ".attn.proj.bias", {c}});
            want.push_back({p + ".attn.relative_position_bias_table", {tsa, hd}});
            want.push_back({p + ".mlp.fc1.weight", {mr * c, c}});
            want.push_back({p + ".mlp.fc1.bias", {mr * c}});
            want.push_back({p + ".mlp.fc2.weight", {c, mr * c}});
            want.push_back({p + ".mlp.fc2.bias", {c}});
            want.push_back({p + ".conv_block.cab.0.weight", {cc, c, 3, 3}});
            want.push_back({p + ".conv_block.cab.0.bias", {cc}});
            want.push_back({p + ".conv_block.cab.2.weight", {c, cc, 3, 3}});
            want.push_back({p + ".conv_block.cab.2.bias", {c}});
            want.push_back({p + ".conv_block.cab.3.attention.1.weight", {sq, c, 1, 1}});
            want.push_back({p + ".conv_block.cab.3.attention.1.bias", {sq}});
            want.push_back({p + ".conv_block.cab.3.attention.3.weight", {c, sq, 1, 1}});
            want.push_back({p + ".conv_block.cab.3.attention.3.bias", {c}});
        }
        std::string p = L + ".residual_group.overlap_attn";
        want.push_back({p + ".norm1.weight", {c}});
        want.push_back({p + ".norm1.bias", {c}});
        want.push_back({p + ".norm2.weight", {c}});
        want.push_back({p + ".norm2.bias", {c}});
        want.push_back({p + ".qkv.weight", {3 * c, c}});
        want.push_back({p + ".qkv.bias", {3 * c}});
        want.push_back({p + ".proj.weight", {c, c}});
        want.push_back({p + ".proj.bias", {c}});
        want.push_back({p + ".relative_position_bias_table", {toca, hd}});
        want.push_back({p + ".mlp.fc1.weight", {mr * c, c}});
        want.push_back({p + ".mlp.fc1.bias", {mr * c}});
        want.push_back({p + ".mlp.fc2.weight", {c, mr * c}});
        want.push_back({p + ".mlp.fc2.bias", {c}});
    }
    for (auto& w : want) {
        if (!has(w.first))
            throw Error(2, path + ": the checkpoint has no `" + w.first + "`; the metadata says " + variant +
                           " with embed " + std::to_string(embed) + ", which does not describe these tensors");
        auto got = shape(w.first);
        if (got != w.second)
            throw Error(2, path + ": `" + w.first + "` is " + shape_str(got) + ", expected " +
                           shape_str(w.second) + " for " + variant + " at embed " + std::to_string(embed));
    }
    if (window != 16 || owin != 24)
        throw Error(2, path + ": window " + std::to_string(window) + " / overlap window " + std::to_string(owin) +
                       ": the B200 kernels are built for the released 16 / 24");
    if (head_dim != 24 && head_dim != 30)
        throw Error(2, path + ": head dim " + std::to_string(head_dim) + ": the B200 kernels are built for 24 and 30");
    f32_bytes = 0;
    for (auto& kv : st.tensors)
        if (kv.second.dtype == "F32") f32_bytes += kv.second.end - kv.second.begin;
}

}  // namespace hat
