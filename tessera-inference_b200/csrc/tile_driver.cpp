// tessera_b200_encode: the reference driver's command line
// (src/tessera_encode.cpp:362-377: TILE_DIR OUT_DIR [WEIGHTS]) on the B200
// back end, for one tile or a comma-separated list of tiles, with the tile
// I/O pipelined against the GPU.
//
//   loader thread   reads tile k+1's seven .npy arrays straight into
//                   page-locked buffers (tc_host_alloc), while
//   main thread     encodes tile k on the GPU(s) with tc_encode_tile (binning,
//                   padding, standardisation, network and int8 quantisation on
//                   the device; host<->device copies from the pinned buffers),
//                   while
//   writer thread   writes tile k-1's <grid>.npy (int8, H x W x 128) and
//                   <grid>_scales.npy (f32, H x W), as the reference does
//                   (src/tessera_encode.cpp:362-364).
//
// Tile directory layout and dtypes follow load_tile (src/tessera_encode.cpp:
// 188-209, 237-243): s2/{bands,masks,doys}.npy and s1/sar_{ascending,
// descending}{,_doy}.npy, or all seven files in the directory itself.
// TC_DEVICES = "0,1,2" or a count N (devices 0..N-1) splits every tile by
// pixel rows across those GPUs (tc_create_multi); unset = the current device.
#include <sys/stat.h>

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "npy.h"
#include "tessera_b200.h"

namespace {

using clk = std::chrono::steady_clock;
double since(clk::time_point t) { return std::chrono::duration<double>(clk::now() - t).count(); }

// Page-locked buffer that grows on demand and is reused across tiles.
struct Pinned {
    void *p = nullptr;
    size_t cap = 0;
    void reserve(size_t n) {
        if (n <= cap) return;
        tc_host_free(p);
        p = tc_host_alloc((int64_t)std::max<size_t>(n, 1));
        if (!p) throw std::runtime_error("cannot allocate " + std::to_string(n) + " bytes of page-locked memory");
        cap = n;
    }
    ~Pinned() { tc_host_free(p); }
};

struct Array {
    std::string descr;
    std::vector<int64_t> shape;
    Pinned buf;
    int64_t count() const {
        int64_t n = 1;
        for (int64_t s : shape) n *= s;
        return n;
    }
};

// Reads one array of the tile into its page-locked buffer, checking the
// element type the reference driver requires (src/tessera_encode.cpp:237-243).
void load_array(const std::string &path, char kind, int size, Array &a) {
    npy::read(path, [&](const npy::Header &h) -> void * {
        if (!h.is(kind, size))
            throw std::runtime_error(path + ": element type " + h.descr + ", this input must be " +
                                     (size == 1 ? "|" : "<") + kind + std::to_string(size));
        a.descr = h.descr;
        a.shape = h.shape;
        a.buf.reserve((size_t)h.nbytes());
        return a.buf.p;
    });
}

bool exists(const std::string &p) {
    struct stat st;
    return stat(p.c_str(), &st) == 0;
}

void mkdirs(const std::string &dir) {
    for (size_t i = 1; i <= dir.size(); ++i)
        if (i == dir.size() || dir[i] == '/') mkdir(dir.substr(0, i).c_str(), 0755);
}

struct TileIn {
    std::string grid, err;
    int64_t T2 = 0, Ta = 0, Td = 0, H = 0, W = 0;
    Array bands, masks, doys, asc, asc_doy, desc, desc_doy;
    double load_s = 0;
};

struct TileOut {
    std::string grid, err;
    int64_t H = 0, W = 0;
    Pinned codes, scales;
    double load_s = 0, net_s = 0, write_s = 0;
};

void load_tile(const std::string &dir_in, TileIn &t) {
    const auto t0 = clk::now();
    std::string d = dir_in;
    while (d.size() > 1 && d.back() == '/') d.pop_back();
    t.grid = d.substr(d.rfind('/') + 1);
    const bool sub = exists(d + "/s2");
    const std::string s2 = sub ? d + "/s2/" : d + "/", s1 = sub ? d + "/s1/" : d + "/";
    load_array(s2 + "bands.npy", 'u', 2, t.bands);
    load_array(s2 + "masks.npy", 'u', 1, t.masks);
    load_array(s2 + "doys.npy", 'u', 2, t.doys);
    load_array(s1 + "sar_ascending.npy", 'i', 2, t.asc);
    load_array(s1 + "sar_ascending_doy.npy", 'i', 2, t.asc_doy);
    load_array(s1 + "sar_descending.npy", 'i', 2, t.desc);
    load_array(s1 + "sar_descending_doy.npy", 'i', 2, t.desc_doy);
    if (t.bands.shape.size() != 4 || t.bands.shape[3] != 10) throw std::runtime_error(t.grid + ": bands must be (T2,H,W,10)");
    t.T2 = t.bands.shape[0];
    t.H = t.bands.shape[1];
    t.W = t.bands.shape[2];
    t.Ta = t.asc.count() ? t.asc.shape[0] : 0;
    t.Td = t.desc.count() ? t.desc.shape[0] : 0;
    auto want = [&](const Array &a, std::vector<int64_t> s, const char *name) {
        if (a.shape != s) throw std::runtime_error(t.grid + ": " + name + " has an unexpected shape");
    };
    want(t.masks, {t.T2, t.H, t.W}, "masks");
    want(t.doys, {t.T2}, "doys");
    if (t.Ta) want(t.asc, {t.Ta, t.H, t.W, 2}, "sar_ascending");
    if (t.Td) want(t.desc, {t.Td, t.H, t.W, 2}, "sar_descending");
    if ((int64_t)t.asc_doy.count() != t.Ta || (int64_t)t.desc_doy.count() != t.Td)
        throw std::runtime_error(t.grid + ": S1 day-of-year arrays do not match their series");
    t.load_s = since(t0);
}

// Two-slot handoff between pipeline stages.
struct Slots {
    std::mutex mu;
    std::condition_variable cv;
    int ready[2] = {-1, -1};  // tile index held by the slot, or -1 if free
    void put(int slot, int k) {
        std::lock_guard<std::mutex> l(mu);
        ready[slot] = k;
        cv.notify_all();
    }
    void wait_for(int slot, int k) {
        std::unique_lock<std::mutex> l(mu);
        cv.wait(l, [&] { return ready[slot] == k; });
    }
};

std::vector<std::string> split(const std::string &s, char sep) {
    std::vector<std::string> out;
    std::stringstream ss(s);
    for (std::string tok; std::getline(ss, tok, sep);)
        if (!tok.empty()) out.push_back(tok);
    return out;
}

}  // namespace

int main(int argc, char **argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: %s TILE_DIR[,TILE_DIR...] OUT_DIR [WEIGHTS]\n", argv[0]);
        return 2;
    }
    const std::vector<std::string> tiles = split(argv[1], ',');
    const std::string out_dir = argv[2];
    std::string weights = argc > 3 ? argv[3] : "";
    if (weights.empty()) {  // as the reference: <binary dir>/../student_large.tcw
        const std::string self = argv[0];
        const size_t slash = self.rfind('/');
        weights = (slash == std::string::npos ? std::string(".") : self.substr(0, slash)) + "/../student_large.tcw";
    }
    if (tiles.empty()) {
        std::fprintf(stderr, "tessera_b200_encode: no tile directory given\n");
        return 2;
    }
    void *h = nullptr;
    int ndev = 1;
    if (const char *e = std::getenv("TC_DEVICES")) {
        std::vector<int> devs;
        const std::vector<std::string> parts = split(e, ',');
        if (parts.size() == 1 && parts[0].find_first_not_of("0123456789") == std::string::npos && std::atoi(e) > 1)
            for (int i = 0; i < std::atoi(e); ++i) devs.push_back(i);
        else
            for (const auto &p : parts) devs.push_back(std::atoi(p.c_str()));
        ndev = (int)devs.size();
        h = tc_create_multi(weights.c_str(), devs.data(), ndev);
    } else {
        h = tc_create(weights.c_str(), 0);
    }
    if (!h) return 1;
    mkdirs(out_dir);

    const int n = (int)tiles.size();
    TileIn in[2];
    TileOut out[2];
    Slots in_full, in_free, out_full, out_free;
    // every slot starts free: "free for tile k" means slot k % 2 may be (re)used for tile k
    for (int s = 0; s < 2; ++s) {
        in_free.ready[s] = s;
        out_free.ready[s] = s;
    }
    std::string fatal;
    std::mutex fatal_mu;
    auto fail = [&](const std::string &m) {
        std::lock_guard<std::mutex> l(fatal_mu);
        if (fatal.empty()) fatal = m;
    };

    const auto t_all = clk::now();
    std::thread loader([&] {
        for (int k = 0; k < n; ++k) {
            const int s = k & 1;
            in_free.wait_for(s, k);
            try {
                in[s].err.clear();
                load_tile(tiles[k], in[s]);
            } catch (const std::exception &e) {
                in[s].err = e.what();
            }
            in_full.put(s, k);
        }
    });
    std::thread writer([&] {
        for (int k = 0; k < n; ++k) {
            const int s = k & 1;
            out_full.wait_for(s, k);
            TileOut &o = out[s];
            if (o.err.empty()) {
                try {
                    const auto t0 = clk::now();
                    npy::write(out_dir + "/" + o.grid + ".npy", "|i1", {o.H, o.W, 128}, o.codes.p,
                               (uint64_t)(o.H * o.W * 128));
                    npy::write(out_dir + "/" + o.grid + "_scales.npy", "<f4", {o.H, o.W}, o.scales.p,
                               (uint64_t)(o.H * o.W) * 4);
                    o.write_s = since(t0);
                    std::printf("ENCODE grid=%s px=%ld devices=%d  load=%.2fs net=%.2fs write=%.2fs\n", o.grid.c_str(),
                                (long)(o.H * o.W), ndev, o.load_s, o.net_s, o.write_s);
                    std::fflush(stdout);
                } catch (const std::exception &e) {
                    fail(e.what());
                }
            } else {
                fail(o.err);
            }
            out_free.put(s, k + 2);
        }
    });

    int64_t total_px = 0;
    for (int k = 0; k < n; ++k) {
        const int s = k & 1;
        in_full.wait_for(s, k);
        out_free.wait_for(s, k);
        TileIn &t = in[s];
        TileOut &o = out[s];
        o.grid = t.grid;
        o.err = t.err;
        o.load_s = t.load_s;
        o.H = t.H;
        o.W = t.W;
        if (o.err.empty()) {
            try {
                o.codes.reserve((size_t)(t.H * t.W * 128));
                o.scales.reserve((size_t)(t.H * t.W) * 4);
                const auto t0 = clk::now();
                const int rc = tc_encode_tile(
                    h, static_cast<const uint16_t *>(t.bands.buf.p), static_cast<const uint8_t *>(t.masks.buf.p),
                    static_cast<const uint16_t *>(t.doys.buf.p), t.Ta ? static_cast<const int16_t *>(t.asc.buf.p) : nullptr,
                    t.Ta ? static_cast<const int16_t *>(t.asc_doy.buf.p) : nullptr,
                    t.Td ? static_cast<const int16_t *>(t.desc.buf.p) : nullptr,
                    t.Td ? static_cast<const int16_t *>(t.desc_doy.buf.p) : nullptr, t.T2, t.Ta, t.Td, t.H, t.W,
                    static_cast<int8_t *>(o.codes.p), static_cast<float *>(o.scales.p));
                o.net_s = since(t0);
                if (rc != 0) o.err = "tc_encode_tile failed on " + t.grid;
                else total_px += t.H * t.W;
            } catch (const std::exception &e) {
                o.err = e.what();
            }
        }
        in_free.put(s, k + 2);
        out_full.put(s, k);
    }
    loader.join();
    writer.join();
    const double wall = since(t_all);
    tc_profile_dump(h);
    tc_destroy(h);
    if (!fatal.empty()) {
        std::fprintf(stderr, "tessera_b200_encode: %s\n", fatal.c_str());
        return 1;
    }
    std::printf("TOTAL tiles=%d px=%ld wall=%.2fs px/s=%.0f tiles/h=%.1f\n", n, (long)total_px, wall,
                total_px / std::max(wall, 1e-9), 3600.0 * n / std::max(wall, 1e-9));
    return 0;
}
