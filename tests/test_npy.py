"""The tile driver's .npy reader and writer (tessera-inference_b200/csrc/npy.cpp)
against numpy's own implementation of the format, on the CPU: a small harness
is compiled from the same source file the driver links.

* files numpy writes (format versions 1.0, 2.0 and 3.0, every dtype the tile
  layout uses, 0-d to 4-d shapes, empty arrays) are read back byte for byte;
* files the harness writes load in numpy with the same dtype, shape and bytes,
  and start their data at a multiple of 64 bytes;
* Fortran order, a wrong element type, a truncated payload, a bad magic and a
  malformed header are refused with a message naming the file.
"""
import subprocess

import numpy as np
import pytest

from conftest import PKG

HARNESS = r"""
#include "npy.h"
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>
// npy_check read IN OUT.bin      -> prints descr and shape, writes the payload
// npy_check write OUT.npy DESCR RAW.bin d0 d1 ...
int main(int argc, char **argv) {
    try {
        const std::string mode = argv[1];
        if (mode == "read") {
            std::vector<char> buf;
            npy::Header h = npy::read(argv[2], [&](const npy::Header &hh) -> void * {
                buf.resize(hh.nbytes() + 1);
                return buf.data();
            });
            std::printf("%s %c %d", h.descr.c_str(), h.kind, h.itemsize);
            for (auto s : h.shape) std::printf(" %lld", (long long)s);
            std::printf("\n");
            FILE *f = std::fopen(argv[3], "wb");
            std::fwrite(buf.data(), 1, h.nbytes(), f);
            std::fclose(f);
        } else {
            std::vector<int64_t> shape;
            for (int i = 5; i < argc; ++i) shape.push_back(std::atoll(argv[i]));
            FILE *f = std::fopen(argv[4], "rb");
            std::vector<char> raw;
            char tmp[65536];
            size_t n;
            while ((n = std::fread(tmp, 1, sizeof(tmp), f)) > 0) raw.insert(raw.end(), tmp, tmp + n);
            std::fclose(f);
            npy::write(argv[2], argv[3], shape, raw.data(), raw.size());
        }
    } catch (const std::exception &e) {
        std::fprintf(stderr, "%s\n", e.what());
        return 1;
    }
    return 0;
}
"""


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    d = tmp_path_factory.mktemp("npy")
    src = d / "npy_check.cpp"
    src.write_text(HARNESS)
    exe = d / "npy_check"
    subprocess.run(["g++", "-O1", "-std=c++17", f"-I{PKG / 'csrc'}", "-o", str(exe), str(src),
                    str(PKG / "csrc" / "npy.cpp")], check=True)
    return exe


def run_read(harness, path, tmp_path):
    out = tmp_path / "payload.bin"
    r = subprocess.run([str(harness), "read", str(path), str(out)], capture_output=True, text=True)
    return r, (out.read_bytes() if r.returncode == 0 else None)


ARRAYS = [
    np.arange(2 * 3 * 4 * 10, dtype=np.uint16).reshape(2, 3, 4, 10),
    (np.arange(60) % 2).astype(np.uint8).reshape(3, 4, 5),
    np.array([5, 300, 65535], np.uint16),
    np.arange(-20, 28, dtype=np.int16).reshape(2, 3, 4, 2),
    np.zeros((0, 7, 3, 2), np.int16),
    np.linspace(-1, 1, 12, dtype=np.float32).reshape(3, 4),
    np.arange(-6, 6, dtype=np.int8).reshape(1, 3, 4),
    np.array(7, np.int16),
]


@pytest.mark.parametrize("version", [(1, 0), (2, 0), (3, 0)])
@pytest.mark.parametrize("k", range(len(ARRAYS)))
def test_reads_numpy_files(harness, tmp_path, version, k):
    a = ARRAYS[k]
    p = tmp_path / "a.npy"
    with open(p, "wb") as f:
        np.lib.format.write_array(f, a, version=version)
    r, payload = run_read(harness, p, tmp_path)
    assert r.returncode == 0, r.stderr
    fields = r.stdout.split()
    assert fields[0] == a.dtype.str
    assert [int(x) for x in fields[3:]] == list(a.shape)
    assert payload == a.tobytes()


@pytest.mark.parametrize("k", range(len(ARRAYS)))
def test_writes_files_numpy_reads(harness, tmp_path, k):
    a = ARRAYS[k]
    raw = tmp_path / "raw.bin"
    raw.write_bytes(a.tobytes())
    out = tmp_path / "w.npy"
    subprocess.run([str(harness), "write", str(out), a.dtype.str, str(raw), *map(str, a.shape)], check=True)
    b = np.load(out)
    assert b.dtype == a.dtype and b.shape == a.shape
    assert b.tobytes() == a.tobytes()
    with open(out, "rb") as f:
        major, _ = np.lib.format.read_magic(f)
        if major == 1:
            np.lib.format.read_array_header_1_0(f)
        else:
            np.lib.format.read_array_header_2_0(f)
        assert f.tell() % 64 == 0
    assert not (tmp_path / "w.npy.partial").exists()


def test_refusals(harness, tmp_path):
    a = np.arange(24, dtype=np.uint16).reshape(2, 3, 4)
    p = tmp_path / "f.npy"
    np.save(p, np.asfortranarray(a))
    r, _ = run_read(harness, p, tmp_path)
    assert r.returncode == 1 and "Fortran order" in r.stderr and str(p) in r.stderr
    np.save(p, a)
    data = p.read_bytes()
    (tmp_path / "t.npy").write_bytes(data[:-5])
    r, _ = run_read(harness, tmp_path / "t.npy", tmp_path)
    assert r.returncode == 1 and "data bytes" in r.stderr
    (tmp_path / "m.npy").write_bytes(b"\x93NUMPX" + data[6:])
    r, _ = run_read(harness, tmp_path / "m.npy", tmp_path)
    assert r.returncode == 1 and "magic" in r.stderr
    bad = bytearray(data)
    i = bad.index(b"'shape'")
    bad[i:i + 7] = b"'shapf'"
    (tmp_path / "k.npy").write_bytes(bytes(bad))
    r, _ = run_read(harness, tmp_path / "k.npy", tmp_path)
    assert r.returncode == 1 and "unknown key" in r.stderr
    r, _ = run_read(harness, tmp_path / "missing.npy", tmp_path)
    assert r.returncode == 1 and "cannot open" in r.stderr


def test_big_endian_is_not_the_tile_dtype(harness, tmp_path):
    """A '>u2' file parses, but is not the little-endian '<u2' the tile needs:
    the driver's element-type check (npy::Header::is) rejects it."""
    p = tmp_path / "be.npy"
    np.save(p, np.arange(6, dtype=">u2"))
    r, payload = run_read(harness, p, tmp_path)
    assert r.returncode == 0 and r.stdout.split()[0] == ">u2"
