// NumPy .npy reader and writer (see npy.h for the format).
#include "npy.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>

namespace npy {

namespace {

constexpr char MAGIC[6] = {'\x93', 'N', 'U', 'M', 'P', 'Y'};
constexpr uint64_t ALIGN = 64;                  // the data starts at a multiple of this
constexpr uint32_t MAX_HEADER = 1u << 20;       // far above any real header
constexpr size_t IO_CHUNK = size_t(64) << 20;   // bytes per read/write system call

[[noreturn]] void fail(const std::string &what, const std::string &why) {
    throw std::runtime_error(what + ": " + why);
}

// A file descriptor that closes itself.
struct Fd {
    int fd = -1;
    ~Fd() {
        if (fd >= 0) ::close(fd);
    }
};

// Reads exactly n bytes at offset off (pread loop over short reads).
void pread_all(int fd, void *dst, uint64_t n, uint64_t off, const std::string &what) {
    auto *p = static_cast<uint8_t *>(dst);
    while (n > 0) {
        const size_t want = (size_t)std::min<uint64_t>(n, IO_CHUNK);
        const ssize_t got = ::pread(fd, p, want, (off_t)off);
        if (got < 0 && errno == EINTR) continue;
        if (got < 0) fail(what, std::string("read error: ") + std::strerror(errno));
        if (got == 0) fail(what, "file ends inside the array data");
        p += got;
        off += (uint64_t)got;
        n -= (uint64_t)got;
    }
}

void write_all(int fd, const void *src, uint64_t n, const std::string &what) {
    auto *p = static_cast<const uint8_t *>(src);
    while (n > 0) {
        const size_t want = (size_t)std::min<uint64_t>(n, IO_CHUNK);
        const ssize_t put = ::write(fd, p, want);
        if (put < 0 && errno == EINTR) continue;
        if (put <= 0) fail(what, std::string("cannot write: ") + std::strerror(errno));
        p += put;
        n -= (uint64_t)put;
    }
}

// Tokens of the header's Python literal: {'key': value, ...} with string,
// boolean and tuple-of-integer values.
class Lexer {
  public:
    Lexer(const std::string &s, const std::string &what) : s_(s), what_(what) {}
    void skip() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\t' || s_[i_] == '\n' || s_[i_] == '\r')) ++i_;
    }
    bool accept(char c) {
        skip();
        if (i_ < s_.size() && s_[i_] == c) {
            ++i_;
            return true;
        }
        return false;
    }
    void need(char c) {
        if (!accept(c)) fail(what_, std::string("header: expected '") + c + "' at offset " + std::to_string(i_));
    }
    std::string string_literal() {
        skip();
        if (i_ >= s_.size() || (s_[i_] != '\'' && s_[i_] != '"')) fail(what_, "header: expected a quoted string");
        const char q = s_[i_++];
        const size_t end = s_.find(q, i_);
        if (end == std::string::npos) fail(what_, "header: unterminated string");
        std::string v = s_.substr(i_, end - i_);
        i_ = end + 1;
        return v;
    }
    bool boolean_literal() {
        skip();
        if (s_.compare(i_, 4, "True") == 0) {
            i_ += 4;
            return true;
        }
        if (s_.compare(i_, 5, "False") == 0) {
            i_ += 5;
            return false;
        }
        fail(what_, "header: expected True or False");
    }
    int64_t integer_literal() {
        skip();
        int64_t v = 0;
        size_t n = 0;
        while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') {
            if (v > (INT64_MAX - 9) / 10) fail(what_, "header: dimension out of range");
            v = v * 10 + (s_[i_++] - '0');
            ++n;
        }
        if (n == 0) fail(what_, "header: expected a non-negative integer");
        if (i_ < s_.size() && (s_[i_] == 'L' || s_[i_] == 'l')) ++i_;  // Python 2 long suffix
        return v;
    }
    bool at_end() {
        skip();
        return i_ == s_.size();
    }

  private:
    const std::string &s_;
    const std::string &what_;
    size_t i_ = 0;
};

void parse_descr(Header &h, const std::string &what) {
    const std::string &d = h.descr;
    if (d.size() < 3 || std::strchr("<>|=", d[0]) == nullptr || !std::isalpha((unsigned char)d[1]))
        fail(what, "unsupported dtype '" + d + "' (a simple dtype such as '<u2' is required)");
    int size = 0;
    for (size_t k = 2; k < d.size(); ++k) {
        if (d[k] < '0' || d[k] > '9') fail(what, "unsupported dtype '" + d + "'");
        size = size * 10 + (d[k] - '0');
        if (size > 64) fail(what, "unsupported dtype '" + d + "'");
    }
    if (size <= 0) fail(what, "unsupported dtype '" + d + "'");
    h.byteorder = d[0];
    h.kind = d[1];
    h.itemsize = size;
}

bool host_little_endian() {
    const uint16_t one = 1;
    uint8_t b;
    std::memcpy(&b, &one, 1);
    return b == 1;
}

}  // namespace

int64_t Header::count() const {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    return n;
}

bool Header::is(char k, int size) const {
    if (kind != k || itemsize != size) return false;
    return size == 1 || byteorder == '<' || (byteorder == '=' && host_little_endian());
}

Header parse_header_dict(const std::string &text, const std::string &what) {
    Header h;
    Lexer lx(text, what);
    bool have_descr = false, have_order = false, have_shape = false;
    lx.need('{');
    while (!lx.accept('}')) {
        const std::string key = lx.string_literal();
        lx.need(':');
        if (key == "descr") {
            h.descr = lx.string_literal();
            have_descr = true;
        } else if (key == "fortran_order") {
            h.fortran_order = lx.boolean_literal();
            have_order = true;
        } else if (key == "shape") {
            lx.need('(');
            h.shape.clear();
            while (!lx.accept(')')) {
                h.shape.push_back(lx.integer_literal());
                if (!lx.accept(',')) {
                    lx.need(')');
                    break;
                }
            }
            have_shape = true;
        } else {
            fail(what, "header has an unknown key '" + key + "'");
        }
        if (!lx.accept(',')) {
            lx.need('}');
            break;
        }
    }
    if (!lx.at_end()) fail(what, "header has text after its dictionary");
    if (!have_descr || !have_order || !have_shape) fail(what, "header lacks descr, fortran_order or shape");
    parse_descr(h, what);
    for (int64_t s : h.shape)
        if (s > (int64_t(1) << 40)) fail(what, "header: dimension out of range");
    return h;
}

Header read(const std::string &path, const std::function<void *(const Header &)> &dest) {
    Fd f;
    f.fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (f.fd < 0) fail(path, std::string("cannot open: ") + std::strerror(errno));
    struct stat st;
    if (::fstat(f.fd, &st) != 0) fail(path, std::string("cannot stat: ") + std::strerror(errno));
    const uint64_t file_size = (uint64_t)st.st_size;

    uint8_t pre[12];
    if (file_size < 10) fail(path, "too short to be a NumPy array file");
    pread_all(f.fd, pre, std::min<uint64_t>(12, file_size), 0, path);
    if (std::memcmp(pre, MAGIC, sizeof(MAGIC)) != 0) fail(path, "missing the NumPy array magic bytes");
    const int major = pre[6];
    uint32_t hlen = 0;
    uint64_t hstart = 0;
    if (major == 1) {
        hlen = (uint32_t)pre[8] | ((uint32_t)pre[9] << 8);
        hstart = 10;
    } else if (major == 2 || major == 3) {
        if (file_size < 12) fail(path, "too short to be a NumPy array file");
        hlen = (uint32_t)pre[8] | ((uint32_t)pre[9] << 8) | ((uint32_t)pre[10] << 16) | ((uint32_t)pre[11] << 24);
        hstart = 12;
    } else {
        fail(path, "unsupported NumPy format version " + std::to_string(major));
    }
    if (hlen == 0 || hlen > MAX_HEADER || hstart + hlen > file_size) fail(path, "header length out of range");
    std::string text(hlen, '\0');
    pread_all(f.fd, &text[0], hlen, hstart, path);

    Header h = parse_header_dict(text, path);
    if (h.fortran_order) fail(path, "array is stored in Fortran order; C order is required");
    h.data_offset = hstart + hlen;
    const uint64_t need = h.nbytes();
    if (h.data_offset + need > file_size)
        fail(path, "file holds " + std::to_string(file_size - h.data_offset) + " data bytes, the header needs " +
                       std::to_string(need));
    void *buf = dest(h);
    if (need > 0) {
        if (!buf) fail(path, "no destination buffer");
#ifdef POSIX_FADV_SEQUENTIAL
        ::posix_fadvise(f.fd, (off_t)h.data_offset, (off_t)need, POSIX_FADV_SEQUENTIAL);
#endif
        pread_all(f.fd, buf, need, h.data_offset, path);
    }
    return h;
}

void write(const std::string &path, const std::string &descr, const std::vector<int64_t> &shape, const void *data,
           uint64_t bytes) {
    // dictionary text; a 1-tuple keeps its trailing comma
    std::string dict = "{'descr': '" + descr + "', 'fortran_order': False, 'shape': (";
    for (size_t k = 0; k < shape.size(); ++k) {
        if (k) dict += ", ";
        dict += std::to_string(shape[k]);
    }
    if (shape.size() == 1) dict += ",";
    dict += "), }";
    // version 1.0 has a 2-byte length field; a longer header needs 2.0
    const bool v1 = dict.size() + 1 + ALIGN < 65536;
    const uint64_t fixed = v1 ? 10 : 12;
    const uint64_t total = (fixed + dict.size() + 1 + ALIGN - 1) / ALIGN * ALIGN;
    const uint64_t hlen = total - fixed;
    std::string pre(MAGIC, sizeof(MAGIC));
    pre += char(v1 ? 1 : 2);
    pre += char(0);
    for (int b = 0; b < (v1 ? 2 : 4); ++b) pre += char((hlen >> (8 * b)) & 0xFF);
    pre += dict;
    pre.append(total - 1 - pre.size(), ' ');
    pre += '\n';

    const std::string tmp = path + ".partial";
    {
        Fd f;
        f.fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
        if (f.fd < 0) fail(tmp, std::string("cannot create: ") + std::strerror(errno));
        write_all(f.fd, pre.data(), pre.size(), tmp);
        write_all(f.fd, data, bytes, tmp);
        if (::close(f.fd) != 0) {
            f.fd = -1;
            fail(tmp, std::string("cannot close: ") + std::strerror(errno));
        }
        f.fd = -1;
    }
    if (std::rename(tmp.c_str(), path.c_str()) != 0) {
        const int e = errno;
        std::remove(tmp.c_str());
        fail(path, std::string("cannot publish: ") + std::strerror(e));
    }
}

}  // namespace npy
