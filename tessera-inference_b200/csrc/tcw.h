// .tcw weight file reader (format of tools/export_weights.py:31-39 in the
// reference: b"TCW1", u32 count, then per tensor u32 name_len, name, u32 ndim,
// i64 dims[ndim], f32 data).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace tcb {

struct HostTensor {
    std::vector<int64_t> shape;
    std::vector<float> data;
};

using WeightMap = std::map<std::string, HostTensor>;

// Reads every tensor of a .tcw file. Throws std::runtime_error on a missing,
// truncated or malformed file.
WeightMap load_tcw(const char *path);

// Checks that every tensor the Large pixel student needs is present with the
// expected shape. Throws std::runtime_error naming the first mismatch.
void validate_large(const WeightMap &w);

// Round-to-nearest-even f32 -> bf16 bits (tessera_cpu.cpp:43-48).
inline uint16_t f2bf(float f) {
    uint32_t u;
    __builtin_memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return uint16_t(u >> 16);
}
inline float bf2f(uint16_t b) {
    uint32_t u = uint32_t(b) << 16;
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
}

}  // namespace tcb
