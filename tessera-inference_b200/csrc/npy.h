// NumPy .npy array files for the tile driver: a reader that parses the
// header dictionary and streams the payload into a caller-supplied buffer
// (page-locked memory, so the host->device copy needs no staging), and a
// writer that publishes a file atomically.
//
// Format (numpy.lib.format, versions 1.0, 2.0 and 3.0): the bytes "\x93NUMPY",
// a major and a minor version byte, the header length as a little-endian
// uint16 (1.0) or uint32 (2.0, 3.0), then the header, a Python dict literal
// with the keys 'descr', 'fortran_order' and 'shape', padded with spaces and
// a final newline so the array data starts at a multiple of 64 bytes.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace npy {

struct Header {
    std::string descr;        // e.g. "<u2", "|u1"
    char byteorder = '|';     // '<', '>', '|' or '='
    char kind = 0;            // 'u', 'i', 'f', 'b', ...
    int itemsize = 0;         // bytes per element
    bool fortran_order = false;
    std::vector<int64_t> shape;
    uint64_t data_offset = 0; // file offset of the first element
    int64_t count() const;
    uint64_t nbytes() const { return (uint64_t)count() * (uint64_t)itemsize; }
    // True if the elements are little-endian (or single bytes) of this kind and size.
    bool is(char k, int size) const;
};

// Parses the dictionary text of a header; throws std::runtime_error naming
// `what` on anything that is not a well-formed C- or Fortran-order header.
Header parse_header_dict(const std::string &text, const std::string &what);

// Reads the array at `path`. `dest` is called once with the parsed header and
// returns where its nbytes() of data go (it may throw to reject the header);
// the payload is then read straight into that buffer. Returns the header.
Header read(const std::string &path, const std::function<void *(const Header &)> &dest);

// Writes a C-order array of `bytes` bytes with the given dtype string and
// shape. The file appears under `path` only once it is complete.
void write(const std::string &path, const std::string &descr, const std::vector<int64_t> &shape, const void *data,
           uint64_t bytes);

}  // namespace npy
