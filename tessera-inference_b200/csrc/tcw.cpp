// .tcw reader with shape validation for the v2 Large pixel student. The file
// is mapped read-only and parsed with a bounds-checked cursor; every error
// names the tensor and the byte offset it concerns.
#include "tcw.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstring>
#include <stdexcept>

namespace tcb {

namespace {

// Read-only mapping of a whole file, unmapped on scope exit.
class MappedFile {
  public:
    explicit MappedFile(const char *path) {
        const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
        if (fd < 0) throw std::runtime_error(std::string("cannot open ") + path + ": " + std::strerror(errno));
        struct stat st;
        if (::fstat(fd, &st) != 0) {
            ::close(fd);
            throw std::runtime_error(std::string("cannot stat ") + path);
        }
        size_ = (size_t)st.st_size;
        if (size_ > 0) {
            void *m = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
            if (m == MAP_FAILED) {
                ::close(fd);
                throw std::runtime_error(std::string("cannot map ") + path);
            }
            base_ = static_cast<const uint8_t *>(m);
            ::madvise(const_cast<uint8_t *>(base_), size_, MADV_SEQUENTIAL);
        }
        ::close(fd);
    }
    ~MappedFile() {
        if (base_) ::munmap(const_cast<uint8_t *>(base_), size_);
    }
    MappedFile(const MappedFile &) = delete;
    MappedFile &operator=(const MappedFile &) = delete;
    const uint8_t *data() const { return base_; }
    size_t size() const { return size_; }

  private:
    const uint8_t *base_ = nullptr;
    size_t size_ = 0;
};

// Bounds-checked little-endian reader over the mapped bytes; every failure
// names the byte offset and what was being read.
class Cursor {
  public:
    Cursor(const uint8_t *p, size_t n) : p_(p), n_(n) {}
    size_t left() const { return n_ - at_; }
    const uint8_t *take(size_t bytes, const std::string &what) {
        if (bytes > left())
            throw std::runtime_error("weight file ends at byte " + std::to_string(n_) + " while reading " + what +
                                     " (" + std::to_string(bytes) + " bytes at offset " + std::to_string(at_) + ")");
        const uint8_t *q = p_ + at_;
        at_ += bytes;
        return q;
    }
    template <class T> T scalar(const std::string &what) {
        T v;
        std::memcpy(&v, take(sizeof(T), what), sizeof(T));
        return v;
    }

  private:
    const uint8_t *p_;
    size_t n_, at_ = 0;
};

constexpr uint32_t MAX_TENSORS = 100000, MAX_NAME = 4096, MAX_RANK = 8;
constexpr int64_t MAX_ELEMS = int64_t(1) << 32;

}  // namespace

WeightMap load_tcw(const char *path) {
    if (!path) throw std::runtime_error("null weights path");
    const MappedFile file(path);
    Cursor c(file.data(), file.size());
    if (file.size() < 8 || std::memcmp(c.take(4, "the magic"), "TCW1", 4) != 0)
        throw std::runtime_error(std::string(path) + " is not a .tcw weight file (no TCW1 magic)");
    const uint32_t count = c.scalar<uint32_t>("the tensor count");
    if (count > MAX_TENSORS) throw std::runtime_error("implausible tensor count " + std::to_string(count));
    WeightMap w;
    for (uint32_t i = 0; i < count; ++i) {
        const std::string which = "tensor " + std::to_string(i);
        const uint32_t name_len = c.scalar<uint32_t>(which + "'s name length");
        if (name_len > MAX_NAME) throw std::runtime_error(which + ": implausible name length");
        const uint8_t *name_bytes = c.take(name_len, which + "'s name");
        std::string name(reinterpret_cast<const char *>(name_bytes), name_len);
        const uint32_t rank = c.scalar<uint32_t>(name + "'s rank");
        if (rank > MAX_RANK) throw std::runtime_error(name + ": implausible rank " + std::to_string(rank));
        HostTensor t;
        t.shape.resize(rank);
        int64_t elems = 1;
        for (uint32_t d = 0; d < rank; ++d) {
            t.shape[d] = c.scalar<int64_t>(name + "'s dimensions");
            if (t.shape[d] < 0 || t.shape[d] > MAX_ELEMS) throw std::runtime_error(name + ": dimension out of range");
            elems *= t.shape[d];
            if (elems > MAX_ELEMS) throw std::runtime_error(name + ": tensor too large");
        }
        const uint8_t *values = c.take((size_t)elems * sizeof(float), name + "'s values");
        t.data.resize((size_t)elems);
        std::memcpy(t.data.data(), values, (size_t)elems * sizeof(float));
        if (!w.emplace(std::move(name), std::move(t)).second)
            throw std::runtime_error(which + ": a tensor of that name was already read");
    }
    if (c.left() != 0)
        throw std::runtime_error(std::to_string(c.left()) + " stray bytes after the last tensor of " + path);
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
