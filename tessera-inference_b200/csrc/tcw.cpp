// .tcw reader with shape validation for the v2 Large pixel student.
#include "tcw.h"

#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>

namespace tcb {

WeightMap load_tcw(const char *path) {
    if (!path) throw std::runtime_error("null weights path");
    std::unique_ptr<FILE, int (*)(FILE *)> f(std::fopen(path, "rb"), std::fclose);
    if (!f) throw std::runtime_error(std::string("cannot open ") + path);
    char magic[4];
    uint32_t n = 0;
    if (std::fread(magic, 1, 4, f.get()) != 4 || std::memcmp(magic, "TCW1", 4) || std::fread(&n, 4, 1, f.get()) != 1)
        throw std::runtime_error("bad weights file");
    if (n > 100000) throw std::runtime_error("bad weights file: implausible tensor count");
    WeightMap w;
    for (uint32_t i = 0; i < n; ++i) {
        uint32_t len = 0, nd = 0;
        if (std::fread(&len, 4, 1, f.get()) != 1 || len > 4096) throw std::runtime_error("truncated weights");
        std::string name(len, '\0');
        if (std::fread(name.data(), 1, len, f.get()) != len || std::fread(&nd, 4, 1, f.get()) != 1 || nd > 8)
            throw std::runtime_error("truncated weights");
        HostTensor t;
        t.shape.resize(nd);
        if (std::fread(t.shape.data(), 8, nd, f.get()) != nd) throw std::runtime_error("truncated weights");
        int64_t count = 1;
        for (auto s : t.shape) {
            if (s < 0 || s > (int64_t(1) << 32)) throw std::runtime_error("bad weights file: dimension of " + name);
            count *= s;
        }
        if (count > (int64_t(1) << 32)) throw std::runtime_error("bad weights file: tensor too large: " + name);
        t.data.resize(count);
        if (std::fread(t.data.data(), 4, count, f.get()) != size_t(count)) throw std::runtime_error("truncated weights");
        w.emplace(std::move(name), std::move(t));
    }
    return w;
}

static void expect(const WeightMap &w, const std::string &name, std::initializer_list<int64_t> shape) {
    auto it = w.find(name);
    if (it == w.end()) throw std::runtime_error("weights: missing tensor " + name);
    const std::vector<int64_t> want(shape);
    if (it->second.shape != want) {
        std::string got;
        for (auto s : it->second.shape) got += (got.empty() ? "" : ",") + std::to_string(s);
        throw std::runtime_error("weights: " + name + " has shape (" + got + ")");
    }
}

void validate_large(const WeightMap &w) {
    for (int b = 0; b < 2; ++b) {
        const std::string p = b == 0 ? "s2_backbone" : "s1_backbone";
        const int64_t C = b == 0 ? 10 : 2;
        expect(w, p + ".embedding.0.weight", {640, C});
        expect(w, p + ".embedding.0.bias", {640});
        expect(w, p + ".embedding.2.weight", {640, 640});
        expect(w, p + ".embedding.2.bias", {640});
        for (int l = 0; l < 4; ++l) {
            const std::string L = p + ".transformer_encoder.layers." + std::to_string(l);
            expect(w, L + ".self_attn.in_proj_weight", {1920, 640});
            expect(w, L + ".self_attn.in_proj_bias", {1920});
            expect(w, L + ".self_attn.out_proj.weight", {640, 640});
            expect(w, L + ".self_attn.out_proj.bias", {640});
            expect(w, L + ".linear1.weight", {2560, 640});
            expect(w, L + ".linear1.bias", {2560});
            expect(w, L + ".linear2.weight", {640, 2560});
            expect(w, L + ".linear2.bias", {640});
            for (const char *nm : {".norm1.weight", ".norm1.bias", ".norm2.weight", ".norm2.bias"}) expect(w, L + nm, {640});
        }
        expect(w, p + ".attn_pool.query.weight", {1, 640});
        expect(w, p + ".attn_pool.query.bias", {1});
    }
    expect(w, "dim_reducer.0.weight", {2560, 1280});
    expect(w, "dim_reducer.0.bias", {2560});
    expect(w, "dim_reducer.1.weight", {2560});
    expect(w, "dim_reducer.1.bias", {2560});
    expect(w, "dim_reducer.4.weight", {128, 2560});
    expect(w, "dim_reducer.4.bias", {128});
}

}  // namespace tcb
