// Host side of the B200 back end: weight upload, workspace, the chunked
// forward pass over token streams, multi-GPU row sharding and the C ABI.
//
// Token-major design. Every pixel of a tile contributes its binned S2 and S1
// series as consecutive rows ("tokens") of two token streams. The dense layers
// are GEMMs over those streams, independent of pixel boundaries, so their M is
// tens of thousands of rows whatever each pixel's bin is; attention and
// pooling walk the per-pixel segments. Per-pixel results depend only on the
// pixel's own series, exactly as in the reference back ends, which batch
// pixels by (bin2, bin1) key only to give their library calls a fixed shape
// (tessera_encode.cpp:258-277).
//
// The stream is processed in chunks of at most tok_cap tokens per modality
// (default 524,288) and px_cap pixels. A chunk's activations take about 14 KB
// per token, 7.4 GB at the default cap, so they live in HBM: on config 1 fewer,
// larger launches measured faster than chunks small enough for the L2.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include <omp.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "kernels.h"
#include "tcw.h"
#include "tessera_b200.h"
#include "tessera_b200_ops.h"

namespace tcb {

static void ck(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
#define CK(x) ck((x), #x)

// ------------------------------------------------------------------ weights
// All weights live in one device allocation; WOff holds byte offsets into it.
struct LinOff { size_t w = 0, b = 0; int N = 0, K = 0; };
struct BackboneOff {
    int C = 0;
    size_t w1t = 0, b1 = 0;
    LinOff emb2, qkv[NL], out[NL], ffn1[NL], ffn2[NL];
    size_t ln1g[NL], ln1b[NL], ln2g[NL], ln2b[NL];
    size_t poolq = 0;
    float poolb = 0.f;
};
struct ModelOff {
    BackboneOff bb[2];
    LinOff red1, red2;
    size_t rlng = 0, rlnb = 0, pe_table = 0, pe_div = 0;
};

struct Blob {
    std::vector<uint8_t> bytes;
    size_t reserve(size_t n) {
        const size_t o = bytes.size();
        bytes.resize((o + n + 255) & ~size_t(255), 0);
        return o;
    }
    size_t put_f32(const std::vector<float> &v) {
        const size_t o = reserve(v.size() * 4);
        std::memcpy(bytes.data() + o, v.data(), v.size() * 4);
        return o;
    }
    size_t put_bf16(const std::vector<float> &v) {
        const size_t o = reserve(v.size() * 2);
        uint16_t *d = reinterpret_cast<uint16_t *>(bytes.data() + o);
        const int64_t n = (int64_t)v.size();
#pragma omp parallel for schedule(static) if (n > (1 << 16))
        for (int64_t i = 0; i < n; ++i) d[i] = f2bf(v[i]);
        return o;
    }
};

static LinOff put_linear(Blob &b, WeightMap &W, const std::string &wn, const std::string &bn) {
    const HostTensor &w = W.at(wn);
    LinOff l;
    l.N = (int)w.shape[0];
    l.K = (int)w.shape[1];
    l.w = b.put_bf16(w.data);
    l.b = b.put_f32(W.at(bn).data);  // f32 bias, as the oneDNN path (tessera_cpu.cpp:208,218)
    return l;
}

static void build_backbone(Blob &b, WeightMap &W, BackboneOff &o, const std::string &p, int C) {
    o.C = C;
    {   // emb1 transposed to [C][640] as f32 of the bf16-rounded weights
        const HostTensor &w = W.at(p + ".embedding.0.weight");
        std::vector<float> t((size_t)C * D);
        for (int n = 0; n < D; ++n)
            for (int k = 0; k < C; ++k) t[(size_t)k * D + n] = bf2f(f2bf(w.data[(size_t)n * C + k]));
        o.w1t = b.put_f32(t);
        o.b1 = b.put_f32(W.at(p + ".embedding.0.bias").data);
    }
    o.emb2 = put_linear(b, W, p + ".embedding.2.weight", p + ".embedding.2.bias");
    for (int l = 0; l < NL; ++l) {
        const std::string L = p + ".transformer_encoder.layers." + std::to_string(l);
        o.qkv[l] = put_linear(b, W, L + ".self_attn.in_proj_weight", L + ".self_attn.in_proj_bias");
        o.out[l] = put_linear(b, W, L + ".self_attn.out_proj.weight", L + ".self_attn.out_proj.bias");
        o.ffn1[l] = put_linear(b, W, L + ".linear1.weight", L + ".linear1.bias");
        o.ffn2[l] = put_linear(b, W, L + ".linear2.weight", L + ".linear2.bias");
        o.ln1g[l] = b.put_f32(W.at(L + ".norm1.weight").data);
        o.ln1b[l] = b.put_f32(W.at(L + ".norm1.bias").data);
        o.ln2g[l] = b.put_f32(W.at(L + ".norm2.weight").data);
        o.ln2b[l] = b.put_f32(W.at(L + ".norm2.bias").data);
    }
    o.poolq = b.put_f32(W.at(p + ".attn_pool.query.weight").data);
    o.poolb = W.at(p + ".attn_pool.query.bias").data[0];
}

static void build_model(Blob &b, WeightMap &W, ModelOff &m) {
    b.bytes.reserve(size_t(96) << 20);  // 88 MB of bf16 matrices plus f32 vectors and tables: no regrowth copies
    build_backbone(b, W, m.bb[0], "s2_backbone", 10);
    build_backbone(b, W, m.bb[1], "s1_backbone", 2);
    m.red1 = put_linear(b, W, "dim_reducer.0.weight", "dim_reducer.0.bias");
    m.red2 = put_linear(b, W, "dim_reducer.4.weight", "dim_reducer.4.bias");
    m.rlng = b.put_f32(W.at("dim_reducer.1.weight").data);
    m.rlnb = b.put_f32(W.at("dim_reducer.1.bias").data);
    // Day-of-year sinusoid, the same f32 host-libm formula as tessera_cpu.cpp:503-509,
    // rounded to bf16; pe_div is the per-pair frequency for non-table days.
    std::vector<float> div(D / 2), table((size_t)367 * D);
    for (int i = 0; i < D / 2; ++i) div[i] = std::exp(float(2 * i) * -(std::log(10000.0f) / float(D)));
    for (int d = 0; d <= 366; ++d)
        for (int i = 0; i < D / 2; ++i) {
            const float a = float(d) * std::exp(float(2 * i) * -(std::log(10000.0f) / float(D)));
            table[(size_t)d * D + 2 * i] = std::sin(a);
            table[(size_t)d * D + 2 * i + 1] = std::cos(a);
        }
    m.pe_table = b.put_bf16(table);
    m.pe_div = b.put_f32(div);
}

struct Lin { const bf16 *w = nullptr; const float *b = nullptr; int N = 0, K = 0; };
struct BackboneDev {
    int C = 0;
    const float *w1t = nullptr, *b1 = nullptr;
    Lin emb2, qkv[NL], out[NL], ffn1[NL], ffn2[NL];
    const float *ln1g[NL], *ln1b[NL], *ln2g[NL], *ln2b[NL];
    const float *poolq = nullptr;
    float poolb = 0.f;
};
struct ModelDev {
    BackboneDev bb[2];
    Lin red1, red2;
    const float *rlng = nullptr, *rlnb = nullptr;
    const bf16 *pe_table = nullptr;
    const float *pe_div = nullptr;
};

static Lin lin_at(const uint8_t *base, const LinOff &o) {
    return Lin{reinterpret_cast<const bf16 *>(base + o.w), reinterpret_cast<const float *>(base + o.b), o.N, o.K};
}
static ModelDev model_at(const uint8_t *base, const ModelOff &m) {
    ModelDev d;
    auto F = [&](size_t off) { return reinterpret_cast<const float *>(base + off); };
    for (int b = 0; b < 2; ++b) {
        const BackboneOff &o = m.bb[b];
        BackboneDev &x = d.bb[b];
        x.C = o.C;
        x.w1t = F(o.w1t);
        x.b1 = F(o.b1);
        x.emb2 = lin_at(base, o.emb2);
        for (int l = 0; l < NL; ++l) {
            x.qkv[l] = lin_at(base, o.qkv[l]);
            x.out[l] = lin_at(base, o.out[l]);
            x.ffn1[l] = lin_at(base, o.ffn1[l]);
            x.ffn2[l] = lin_at(base, o.ffn2[l]);
            x.ln1g[l] = F(o.ln1g[l]); x.ln1b[l] = F(o.ln1b[l]);
            x.ln2g[l] = F(o.ln2g[l]); x.ln2b[l] = F(o.ln2b[l]);
        }
        x.poolq = F(o.poolq);
        x.poolb = o.poolb;
    }
    d.red1 = lin_at(base, m.red1);
    d.red2 = lin_at(base, m.red2);
    d.rlng = F(m.rlng);
    d.rlnb = F(m.rlnb);
    d.pe_table = reinterpret_cast<const bf16 *>(base + m.pe_table);
    d.pe_div = F(m.pe_div);
    return d;
}

// Algorithmic FLOP of one pixel (dense layers on its real tokens, dense attention, head).
static double pixel_flop(int64_t t2, int64_t t1) {
    if (t2 == 0 && t1 == 0) return 0.0;
    auto ftok = [](double C) { return 1280.0 * C + 819200.0 + 39321600.0; };
    return t2 * ftok(10) + t1 * ftok(2) + 10240.0 * (double(t2) * t2 + double(t1) * t1) + 7208960.0;
}

static int bin_size(int64_t n) {  // tessera_encode.cpp:146-151
    if (n <= 0) return 0;
    for (int b = 8; b <= 256; b += 8)
        if (n <= b) return b;
    return 256;
}

// ------------------------------------------------------------------ device state
template <class T> struct DevBuf {
    T *p = nullptr;
    size_t n = 0;
    void ensure(size_t want) {
        if (want <= n) return;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        CK(cudaMalloc(&p, std::max<size_t>(want, 1) * sizeof(T)));
        n = want;
    }
    void release() { if (p) cudaFree(p); p = nullptr; n = 0; }
};
template <class T> struct HostBuf {
    T *p = nullptr;
    size_t n = 0;
    void ensure(size_t want) {
        if (want <= n) return;
        if (p) cudaFreeHost(p);
        p = nullptr;
        n = 0;
        CK(cudaMallocHost(&p, std::max<size_t>(want, 1) * sizeof(T)));
        n = want;
    }
    void release() { if (p) cudaFreeHost(p); p = nullptr; n = 0; }
};

struct Dev {
    int device = 0;
    cudaStream_t own = nullptr, st = nullptr;
    uint8_t *wdev = nullptr;
    ModelDev m;
    int64_t tok_cap = 0, px_cap = 0;
    // chunk workspace
    DevBuf<float> rec, logits;
    DevBuf<bf16> y, x, x1, att, qkv, hbuf, fused, r1, r2;
    DevBuf<int> status;
    // tc_encode inputs / output
    DevBuf<float> in2, in1, outf;
    // tile path
    DevBuf<uint8_t> tile;  // band copy of the tile arrays
    DevBuf<int32_t> n2, n1, bins2, bins1;
    DevBuf<int64_t> off2, off1;
    DevBuf<int32_t> list2, list1;  // per chunk, its pixels by attention class
    DevBuf<uint8_t> empty;
    DevBuf<int8_t> codes;
    DevBuf<float> scales;
    HostBuf<int32_t> hcnt;
    HostBuf<uint8_t> hseg;
    // profiling
    bool prof = false;
    std::vector<cudaEvent_t> evpool;
    std::vector<int> evcat;
    size_t evn = 0;
    tc_stats stats{};

    ~Dev() {
        if (device >= 0) cudaSetDevice(device);
        if (own) cudaStreamSynchronize(own);
        for (auto e : evpool) cudaEventDestroy(e);
        rec.release(); logits.release(); y.release(); x.release(); x1.release(); att.release(); qkv.release(); hbuf.release();
        fused.release(); r1.release(); r2.release(); status.release(); in2.release(); in1.release(); outf.release();
        tile.release(); n2.release(); n1.release(); bins2.release(); bins1.release(); off2.release(); off1.release();
        list2.release(); list1.release();
        empty.release(); codes.release(); scales.release(); hcnt.release(); hseg.release();
        if (wdev) cudaFree(wdev);
        if (own) cudaStreamDestroy(own);
    }

    void mark(int cat) {
        if (!prof) return;
        if (evn == evpool.size()) {
            cudaEvent_t e;
            CK(cudaEventCreate(&e));
            evpool.push_back(e);
            evcat.push_back(0);
        }
        evcat[evn] = cat;
        CK(cudaEventRecord(evpool[evn++], st));
    }
    // After a stream sync: attribute each gap between consecutive marks to the op that started it.
    // GEMM marks carry 100 + layer kind.
    void harvest() {
        if (!prof || evn < 2) { evn = 0; return; }
        for (size_t i = 0; i + 1 < evn; ++i) {
            float ms = 0.f;
            CK(cudaEventElapsedTime(&ms, evpool[i], evpool[i + 1]));
            const int c = evcat[i];
            if (c >= 100) {
                stats.ms_cat[TC_CAT_GEMM] += ms;
                stats.gemm_ms_kind[c - 100] += ms;
            } else {
                stats.ms_cat[c] += ms;
            }
        }
        evn = 0;
    }
};

static int64_t env_int(const char *name, int64_t dflt) {
    const char *e = std::getenv(name);
    if (!e || !*e) return dflt;
    const long long v = std::atoll(e);
    return v > 0 ? v : dflt;
}

static void dev_init(Dev &d, int device, const Blob &blob, const ModelOff &off) {
    d.device = device;
    CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) throw std::runtime_error(std::string("device ") + prop.name + " is not sm_100 (B200)");
    CK(cudaStreamCreateWithFlags(&d.own, cudaStreamNonBlocking));
    d.st = d.own;
    CK(cudaMalloc(&d.wdev, blob.bytes.size()));
    CK(cudaMemcpy(d.wdev, blob.bytes.data(), blob.bytes.size(), cudaMemcpyHostToDevice));
    d.m = model_at(d.wdev, off);
    // 512K tokens (7.4 GB of activations): half the launches of 256K chunks and
    // a quarter of 128K ones (config 1: 93.3k against 92.3k and 91.2k px/s)
    d.tok_cap = env_int("TC_CHUNK_TOKENS", 524288);
    d.px_cap = env_int("TC_CHUNK_PIXELS", 32768);
    d.status.ensure(1);
    CK(cudaMemset(d.status.p, 0, sizeof(int)));
    const size_t T = (size_t)d.tok_cap, P = (size_t)d.px_cap;
    d.rec.ensure(T * 11);
    d.logits.ensure(T);
    d.y.ensure(T * D); d.x.ensure(T * D); d.x1.ensure(T * D); d.att.ensure(T * D);
    d.qkv.ensure(T * 3 * D); d.hbuf.ensure(T * FF);
    d.fused.ensure(P * 2 * D); d.r1.ensure(P * RED); d.r2.ensure(P * OUT);
}

// ------------------------------------------------------------------ forward pass
enum GemmKind { GK_EMB2 = 0, GK_QKV, GK_OUT, GK_FFN1, GK_FFN2, GK_HEAD };

static void gemm(Dev &d, int kind, const Lin &L, const bf16 *A, int64_t M, bf16 *out, bool relu,
                 const bf16 *res = nullptr, const float *pe_doy = nullptr, int pe_stride = 1,
                 const float *ln_g = nullptr, const float *ln_b = nullptr) {
    if (M <= 0) return;
    d.mark(100 + kind);
    GemmArgs p;
    p.M = (int)M;
    p.N = L.N;
    p.K = L.K;
    p.bias = L.b;
    p.relu = relu ? 1 : 0;
    p.res = res;
    p.ldr = L.N;
    p.pe_doy = pe_doy;
    p.pe_stride = pe_stride;
    p.pe_table = d.m.pe_table;
    p.pe_div = d.m.pe_div;
    p.out = out;
    p.ldo = L.N;
    p.status = d.status.p;
    p.ln_g = ln_g;
    p.ln_b = ln_b;
    launch_gemm(p, A, L.K, L.w, d.st);
    d.stats.gemm_flop += 2.0 * double(M) * L.N * L.K;
    d.stats.gemm_flop_kind[kind] += 2.0 * double(M) * L.N * L.K;
    d.stats.gemm_launches += 1;
    d.stats.launches += 1;
}

// TC_LN_FUSE=1 runs LN1 / LN2 in the epilogues of out-proj / FFN2 (4-CTA
// cluster exchanging row statistics) instead of as a separate kernel. Off by
// default: on config 1 the fused GEMMs lost more time (out-proj + FFN2
// 2.80 s -> 5.05 s per tile) than the LayerNorm kernel they replace (1.12 s).
static bool ln_fused() {
    static const bool on = [] {
        const char *e = std::getenv("TC_LN_FUSE");
        return e && *e == '1';
    }();
    return on;
}

// One backbone over a chunk's token stream: records (M, C+1) -> fused[:, col0:col0+640].
// plan: the chunk's pixels by attention class; null when every series has length Tmax.
static void backbone(Dev &d, int b, const float *rec, Segs segs, int64_t M, int Tmax, int64_t npix,
                     const AttnPlan *plan = nullptr) {
    const BackboneDev &B = d.m.bb[b];
    if (M > d.tok_cap) throw std::runtime_error("chunk larger than the token workspace");
    bool logits_ready = false;
    if (M > 0) {
        d.mark(TC_CAT_EMB1);
        launch_emb1(B.C, rec, M, B.w1t, B.b1, d.y.p, d.st);
        d.stats.launches += 1;
        gemm(d, GK_EMB2, B.emb2, d.y.p, M, d.x.p, false, nullptr, rec + B.C, B.C + 1);  // + DOY sinusoid
        for (int l = 0; l < NL; ++l) {
            gemm(d, GK_QKV, B.qkv[l], d.x.p, M, d.qkv.p, false);
            d.mark(TC_CAT_ATTN);
            d.stats.launches += plan ? launch_attention_plan(d.qkv.p, segs, *plan, M, d.att.p, d.status.p, d.st)
                                     : launch_attention(d.qkv.p, segs, npix, M, Tmax, d.att.p, d.status.p, d.st);
            if (ln_fused()) {  // LN1 / LN2 in the epilogues of out-proj / FFN2
                gemm(d, GK_OUT, B.out[l], d.att.p, M, d.x1.p, false, d.x.p, nullptr, 1, B.ln1g[l], B.ln1b[l]);
                gemm(d, GK_FFN1, B.ffn1[l], d.x1.p, M, d.hbuf.p, true);
                gemm(d, GK_FFN2, B.ffn2[l], d.hbuf.p, M, d.x.p, false, d.x1.p, nullptr, 1, B.ln2g[l], B.ln2b[l]);
            } else {
                gemm(d, GK_OUT, B.out[l], d.att.p, M, d.y.p, false, d.x.p);
                d.mark(TC_CAT_LN);
                launch_layernorm640(d.y.p, M, B.ln1g[l], B.ln1b[l], d.x1.p, d.st);
                gemm(d, GK_FFN1, B.ffn1[l], d.x1.p, M, d.hbuf.p, true);
                gemm(d, GK_FFN2, B.ffn2[l], d.hbuf.p, M, d.y.p, false, d.x1.p);
                d.mark(TC_CAT_LN);
                // the last LN2 also writes the pooling logits, so pooling reads x once
                const bool last = l == NL - 1;
                launch_layernorm640(d.y.p, M, B.ln2g[l], B.ln2b[l], d.x.p, d.st, last ? B.poolq : nullptr, B.poolb,
                                    last ? d.logits.p : nullptr);
                logits_ready = last;
                d.stats.launches += 2;
            }
        }
    }
    d.mark(TC_CAT_POOL);
    launch_pool(d.x.p, segs, npix, B.poolq, B.poolb, d.fused.p, b * D, d.st, logits_ready ? d.logits.p : nullptr);
    d.stats.launches += 1;
    d.stats.tokens += double(M);
}

static void head(Dev &d, int64_t npix, const uint8_t *empty, float *outf, int8_t *codes, float *scales) {
    gemm(d, GK_HEAD, d.m.red1, d.fused.p, npix, d.r1.p, false);
    d.mark(TC_CAT_HEAD);
    launch_ln_relu2560(d.r1.p, npix, d.m.rlng, d.m.rlnb, d.st);
    gemm(d, GK_HEAD, d.m.red2, d.r1.p, npix, d.r2.p, false);
    d.mark(TC_CAT_HEAD);
    launch_out128(d.r2.p, npix, empty, outf, codes, scales, d.st);
    d.stats.launches += 2;
}

static void check_status(Dev &d) {
    int s = 0;
    CK(cudaMemcpy(&s, d.status.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (s != 0) {
        CK(cudaMemset(d.status.p, 0, sizeof(int)));
        throw std::runtime_error("device status " + std::to_string(s) + " (a bounded wait in a kernel ran out)");
    }
}

// tc_encode: prepared records (G, T, C+1) f32 from the host, f32 embeddings back.
static void encode_records(Dev &d, const float *s2, int64_t G, int64_t T2, const float *s1, int64_t T1, float *out) {
    if (T2 < 1 || T1 < 1 || T2 > 256 || T1 > 256) throw std::runtime_error("T2 and T1 must be in [1, 256]");
    CK(cudaSetDevice(d.device));
    d.in2.ensure((size_t)G * T2 * 11);
    d.in1.ensure((size_t)G * T1 * 3);
    d.outf.ensure((size_t)G * OUT);
    d.mark(TC_CAT_H2D);
    CK(cudaMemcpyAsync(d.in2.p, s2, (size_t)G * T2 * 11 * 4, cudaMemcpyHostToDevice, d.st));
    CK(cudaMemcpyAsync(d.in1.p, s1, (size_t)G * T1 * 3 * 4, cudaMemcpyHostToDevice, d.st));
    const int64_t per = std::max<int64_t>(1, std::min<int64_t>(d.px_cap, d.tok_cap / std::max(T2, T1)));
    for (int64_t i0 = 0; i0 < G; i0 += per) {
        const int64_t n = std::min(per, G - i0);
        backbone(d, 0, d.in2.p + i0 * T2 * 11, Segs{nullptr, 0, T2}, n * T2, (int)T2, n);
        backbone(d, 1, d.in1.p + i0 * T1 * 3, Segs{nullptr, 0, T1}, n * T1, (int)T1, n);
        head(d, n, nullptr, d.outf.p + i0 * OUT, nullptr, nullptr);
    }
    d.mark(TC_CAT_D2H);
    CK(cudaMemcpyAsync(out, d.outf.p, (size_t)G * OUT * 4, cudaMemcpyDeviceToHost, d.st));
    d.mark(TC_CAT_D2H);
    CK(cudaStreamSynchronize(d.st));
    CK(cudaGetLastError());
    d.harvest();
    check_status(d);
    d.stats.calls += 1;
    d.stats.pixels += double(G);
    d.stats.alg_flop += double(G) * pixel_flop(T2, T1);
}

// Encode pixels [p0, p0 + np) of device-resident tile arrays t into codes/scales
// (device, np pixels). The caller synchronises.
static void encode_band(Dev &d, const TileDev &t, int64_t p0, int64_t np, int8_t *codes, float *scales) {
    if (np <= 0) return;
    d.n2.ensure(np); d.n1.ensure(np);
    d.hcnt.ensure(2 * np);
    d.mark(TC_CAT_PREP);
    launch_count(t, p0, np, d.n2.p, d.n1.p, d.st);
    d.stats.launches += 1;
    CK(cudaMemcpyAsync(d.hcnt.p, d.n2.p, np * 4, cudaMemcpyDeviceToHost, d.st));
    CK(cudaMemcpyAsync(d.hcnt.p + np, d.n1.p, np * 4, cudaMemcpyDeviceToHost, d.st));
    CK(cudaStreamSynchronize(d.st));
    // host: bins, per-pixel token counts, offsets, chunk plan
    const size_t seg_bytes = (size_t)np * (4 + 4 + 1) + (size_t)(np + 1) * 16 + (size_t)np * 8 + 96;
    d.hseg.ensure(seg_bytes);
    int32_t *b2 = reinterpret_cast<int32_t *>(d.hseg.p);
    int32_t *b1 = b2 + np;
    int64_t *o2 = reinterpret_cast<int64_t *>(((uintptr_t)(b1 + np) + 15) & ~uintptr_t(15));
    int64_t *o1 = o2 + np + 1;
    uint8_t *em = reinterpret_cast<uint8_t *>(o1 + np + 1);
    int32_t *l2 = reinterpret_cast<int32_t *>(((uintptr_t)(em + np) + 15) & ~uintptr_t(15));
    int32_t *l1 = l2 + np;
    const int32_t *c2 = d.hcnt.p, *c1 = d.hcnt.p + np;
    o2[0] = o1[0] = 0;
    double flop = 0.0;
    for (int64_t i = 0; i < np; ++i) {
        const int k2 = bin_size(c2[i]), k1 = bin_size(c1[i]);
        const bool none = k2 == 0 && k1 == 0;  // skipped by the reference (tessera_encode.cpp:274)
        b2[i] = none ? 0 : std::max(k2, 1);
        b1[i] = none ? 0 : std::max(k1, 1);
        em[i] = none ? 1 : 0;
        o2[i + 1] = o2[i] + b2[i];
        o1[i + 1] = o1[i] + b1[i];
        flop += pixel_flop(b2[i], b1[i]);
    }
    d.bins2.ensure(np); d.bins1.ensure(np); d.off2.ensure(np + 1); d.off1.ensure(np + 1); d.empty.ensure(np);
    CK(cudaMemcpyAsync(d.bins2.p, b2, np * 4, cudaMemcpyHostToDevice, d.st));
    CK(cudaMemcpyAsync(d.bins1.p, b1, np * 4, cudaMemcpyHostToDevice, d.st));
    CK(cudaMemcpyAsync(d.off2.p, o2, (np + 1) * 8, cudaMemcpyHostToDevice, d.st));
    CK(cudaMemcpyAsync(d.off1.p, o1, (np + 1) * 8, cudaMemcpyHostToDevice, d.st));
    CK(cudaMemcpyAsync(d.empty.p, em, np, cudaMemcpyHostToDevice, d.st));
    // chunks, and each chunk's pixels by attention class (list entries of the
    // chunk [i0, i1) sit at [i0, i1), relative to i0)
    struct ChunkPlan { int64_t i0, i1; int Tm2, Tm1; AttnPlan a2, a1; };
    std::vector<ChunkPlan> chunks;
    for (int64_t i0 = 0; i0 < np;) {
        int64_t i1 = i0;
        int Tm2 = 0, Tm1 = 0;
        while (i1 < np && i1 - i0 < d.px_cap && o2[i1 + 1] - o2[i0] <= d.tok_cap && o1[i1 + 1] - o1[i0] <= d.tok_cap) {
            Tm2 = std::max(Tm2, b2[i1]);
            Tm1 = std::max(Tm1, b1[i1]);
            ++i1;
        }
        if (i1 == i0) throw std::runtime_error("token workspace smaller than one pixel");
        ChunkPlan c{i0, i1, Tm2, Tm1, {}, {}};
        attention_plan(o2 + i0, i1 - i0, l2 + i0, c.a2);
        attention_plan(o1 + i0, i1 - i0, l1 + i0, c.a1);
        chunks.push_back(c);
        i0 = i1;
    }
    d.list2.ensure(np); d.list1.ensure(np);
    CK(cudaMemcpyAsync(d.list2.p, l2, np * 4, cudaMemcpyHostToDevice, d.st));
    CK(cudaMemcpyAsync(d.list1.p, l1, np * 4, cudaMemcpyHostToDevice, d.st));
    for (ChunkPlan &c : chunks) {
        const int64_t i0 = c.i0, i1 = c.i1, n = i1 - i0;
        c.a2.pix = d.list2.p + i0;
        c.a1.pix = d.list1.p + i0;
        const Segs s2{d.off2.p + i0, o2[i0], 0}, s1{d.off1.p + i0, o1[i0], 0};
        d.mark(TC_CAT_PREP);
        launch_gather(0, t, p0 + i0, n, nullptr, d.bins2.p + i0, s2, d.rec.p, d.st);
        backbone(d, 0, d.rec.p, s2, o2[i1] - o2[i0], c.Tm2, n, &c.a2);
        d.mark(TC_CAT_PREP);
        launch_gather(1, t, p0 + i0, n, nullptr, d.bins1.p + i0, s1, d.rec.p, d.st);
        backbone(d, 1, d.rec.p, s1, o1[i1] - o1[i0], c.Tm1, n, &c.a1);
        head(d, n, d.empty.p + i0, nullptr, codes + i0 * OUT, scales + i0);
        d.stats.launches += 2;
    }
    d.stats.pixels += double(np);
    d.stats.alg_flop += flop;
}

struct TileHost {
    const uint16_t *bands;
    const uint8_t *masks;
    const uint16_t *doys;
    const int16_t *asc, *asc_doy, *desc, *desc_doy;
    int64_t T2, Ta, Td, H, W;
};

// Host tile rows [r0, r1) -> device band copy -> encode -> host outputs.
static void encode_rows_host(Dev &d, const TileHost &h, int64_t r0, int64_t r1, int8_t *codes, float *scales) {
    CK(cudaSetDevice(d.device));
    const int64_t N = h.H * h.W, np = (r1 - r0) * h.W, pbeg = r0 * h.W;
    if (np <= 0) return;
    // band layout: bands | masks | doys | asc | asc_doy | desc | desc_doy, 256-byte aligned sections
    auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
    const size_t sb = al((size_t)h.T2 * np * 20), sm = al((size_t)h.T2 * np), sd = al((size_t)h.T2 * 2);
    const size_t sa = al((size_t)h.Ta * np * 4), sad = al((size_t)h.Ta * 2 + 2);
    const size_t sdd = al((size_t)h.Td * np * 4), sddd = al((size_t)h.Td * 2 + 2);
    const size_t total = sb + sm + sd + sa + sad + sdd + sddd;
    const size_t outb = al((size_t)np * OUT);
    d.tile.ensure(total + outb + (size_t)np * 4);
    uint8_t *base = d.tile.p;
    TileDev t;
    t.bands = reinterpret_cast<const uint16_t *>(base);
    t.masks = base + sb;
    t.doys = reinterpret_cast<const uint16_t *>(base + sb + sm);
    t.asc = reinterpret_cast<const int16_t *>(base + sb + sm + sd);
    t.asc_doy = reinterpret_cast<const int16_t *>(base + sb + sm + sd + sa);
    t.desc = reinterpret_cast<const int16_t *>(base + sb + sm + sd + sa + sad);
    t.desc_doy = reinterpret_cast<const int16_t *>(base + sb + sm + sd + sa + sad + sdd);
    t.T2 = h.T2; t.Ta = h.Ta; t.Td = h.Td; t.N = np;
    int8_t *dcodes = reinterpret_cast<int8_t *>(base + total);
    float *dscales = reinterpret_cast<float *>(base + total + outb);
    d.mark(TC_CAT_H2D);
    auto copy2d = [&](const void *src, const void *dst, size_t esz, int64_t T) {
        if (T <= 0) return;
        CK(cudaMemcpy2DAsync(const_cast<void *>(dst), (size_t)np * esz, static_cast<const uint8_t *>(src) + pbeg * esz,
                             (size_t)N * esz, (size_t)np * esz, (size_t)T, cudaMemcpyHostToDevice, d.st));
    };
    copy2d(h.bands, t.bands, 20, h.T2);
    copy2d(h.masks, t.masks, 1, h.T2);
    if (h.T2) CK(cudaMemcpyAsync(const_cast<uint16_t *>(t.doys), h.doys, h.T2 * 2, cudaMemcpyHostToDevice, d.st));
    copy2d(h.asc, t.asc, 4, h.Ta);
    if (h.Ta) CK(cudaMemcpyAsync(const_cast<int16_t *>(t.asc_doy), h.asc_doy, h.Ta * 2, cudaMemcpyHostToDevice, d.st));
    copy2d(h.desc, t.desc, 4, h.Td);
    if (h.Td) CK(cudaMemcpyAsync(const_cast<int16_t *>(t.desc_doy), h.desc_doy, h.Td * 2, cudaMemcpyHostToDevice, d.st));
    encode_band(d, t, 0, np, dcodes, dscales);
    d.mark(TC_CAT_D2H);
    CK(cudaMemcpyAsync(codes + pbeg * OUT, dcodes, (size_t)np * OUT, cudaMemcpyDeviceToHost, d.st));
    CK(cudaMemcpyAsync(scales + pbeg, dscales, (size_t)np * 4, cudaMemcpyDeviceToHost, d.st));
    d.mark(TC_CAT_D2H);
    CK(cudaStreamSynchronize(d.st));
    CK(cudaGetLastError());
    d.harvest();
    check_status(d);
    d.stats.calls += 1;
}

// ------------------------------------------------------------------ planner
static void host_counts(const uint8_t *masks, const int16_t *asc, const int16_t *desc, int64_t T2, int64_t Ta,
                        int64_t Td, int64_t N, std::vector<int32_t> &b2, std::vector<int32_t> &b1) {
    b2.assign(N, 0);
    b1.assign(N, 0);
    const uint32_t *a = reinterpret_cast<const uint32_t *>(asc);
    const uint32_t *dd = reinterpret_cast<const uint32_t *>(desc);
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < N; ++p) {
        int c2 = 0, c1 = 0;
        for (int64_t s = 0; s < T2; ++s) c2 += masks[s * N + p] != 0;
        for (int64_t s = 0; s < Ta; ++s) c1 += a[s * N + p] != 0u;
        for (int64_t s = 0; s < Td; ++s) c1 += dd[s * N + p] != 0u;
        b2[p] = c2;
        b1[p] = c1;
    }
}

static std::vector<int64_t> plan_rows(const uint8_t *masks, const int16_t *asc, const int16_t *desc, int64_t T2,
                                      int64_t Ta, int64_t Td, int64_t H, int64_t W, int nparts) {
    std::vector<int64_t> bounds(nparts + 1, H);
    bounds[0] = 0;
    if (nparts == 1) return bounds;
    std::vector<int32_t> c2, c1;
    host_counts(masks, asc, desc, T2, Ta, Td, H * W, c2, c1);
    std::vector<double> row(H, 0.0);
    for (int64_t r = 0; r < H; ++r) {
        double s = 0;
        for (int64_t c = 0; c < W; ++c) {
            const int k2 = bin_size(c2[r * W + c]), k1 = bin_size(c1[r * W + c]);
            if (k2 || k1) s += pixel_flop(std::max(k2, 1), std::max(k1, 1));
        }
        row[r] = s;
    }
    double total = 0;
    for (double v : row) total += v;
    double acc = 0;
    int k = 1;
    for (int64_t r = 0; r < H && k < nparts; ++r) {
        acc += row[r];
        while (k < nparts && acc >= total * k / nparts) bounds[k++] = r + 1;
    }
    for (; k < nparts; ++k) bounds[k] = H;
    for (int i = 1; i <= nparts; ++i) bounds[i] = std::max(bounds[i], bounds[i - 1]);
    return bounds;
}

// ------------------------------------------------------------------ handle
struct Handle {
    Blob blob;
    ModelOff off;
    std::vector<std::unique_ptr<Dev>> devs;
};

// devices: CUDA ordinals; -1 = the calling thread's current device. The weight
// file is read and validated before any CUDA call.
static Handle *create(const char *path, const std::vector<int> &devices) {
    auto h = std::make_unique<Handle>();
    WeightMap W = load_tcw(path);
    validate_large(W);
    build_model(h->blob, W, h->off);
    for (int dv : devices) {
        if (dv < 0) CK(cudaGetDevice(&dv));
        auto d = std::make_unique<Dev>();
        dev_init(*d, dv, h->blob, h->off);
        h->devs.push_back(std::move(d));
    }
    return h.release();
}

static void tile_rows(Handle &h, const TileHost &t, int64_t row0, int64_t row1, int8_t *codes, float *scales) {
    if (t.T2 < 0 || t.Ta < 0 || t.Td < 0 || t.H < 0 || t.W < 0) throw std::runtime_error("negative tile dimension");
    if (row0 < 0 || row1 > t.H || row0 > row1) throw std::runtime_error("bad row range");
    if (!codes || !scales) throw std::runtime_error("null output");
    if ((t.T2 && (!t.bands || !t.masks || !t.doys)) || (t.Ta && (!t.asc || !t.asc_doy)) || (t.Td && (!t.desc || !t.desc_doy)))
        throw std::runtime_error("null input array");
    if (t.T2 > MAX_STEPS || t.Ta + t.Td > MAX_STEPS) throw std::runtime_error("series longer than supported");
    const int nd = (int)h.devs.size();
    if (nd == 1) { encode_rows_host(*h.devs[0], t, row0, row1, codes, scales); return; }
    // rows of [row0, row1) split by FLOP across the devices
    std::vector<int64_t> b(nd + 1);
    {
        const int64_t R = row1 - row0, off = row0 * t.W;
        const int64_t N = t.H * t.W;
        // plan on the selected rows only: count with a pixel offset into each slice
        std::vector<int32_t> c2(R * t.W), c1(R * t.W);
        const uint32_t *a = reinterpret_cast<const uint32_t *>(t.asc);
        const uint32_t *dd = reinterpret_cast<const uint32_t *>(t.desc);
#pragma omp parallel for schedule(static)
        for (int64_t p = 0; p < R * t.W; ++p) {
            int x2 = 0, x1 = 0;
            for (int64_t s = 0; s < t.T2; ++s) x2 += t.masks[s * N + off + p] != 0;
            for (int64_t s = 0; s < t.Ta; ++s) x1 += a[s * N + off + p] != 0u;
            for (int64_t s = 0; s < t.Td; ++s) x1 += dd[s * N + off + p] != 0u;
            c2[p] = x2;
            c1[p] = x1;
        }
        std::vector<double> row(R, 0.0);
        double total = 0;
        for (int64_t r = 0; r < R; ++r) {
            for (int64_t c = 0; c < t.W; ++c) {
                const int k2 = bin_size(c2[r * t.W + c]), k1 = bin_size(c1[r * t.W + c]);
                if (k2 || k1) row[r] += pixel_flop(std::max(k2, 1), std::max(k1, 1));
            }
            total += row[r];
        }
        b[0] = row0;
        double acc = 0;
        int k = 1;
        for (int64_t r = 0; r < R && k < nd; ++r) {
            acc += row[r];
            while (k < nd && acc >= total * k / nd) b[k++] = row0 + r + 1;
        }
        for (; k <= nd; ++k) b[k] = row1;
    }
    std::vector<std::string> errs(nd);
    std::vector<std::thread> th;
    for (int i = 0; i < nd; ++i)
        th.emplace_back([&, i] {
            try {
                encode_rows_host(*h.devs[i], t, b[i], b[i + 1], codes, scales);
            } catch (const std::exception &e) {
                errs[i] = e.what();
            }
        });
    for (auto &x : th) x.join();
    for (int i = 0; i < nd; ++i)
        if (!errs[i].empty()) throw std::runtime_error("device " + std::to_string(h.devs[i]->device) + ": " + errs[i]);
}

}  // namespace tcb

using namespace tcb;

// ------------------------------------------------------------------ C ABI
extern "C" {

void *tc_create(const char *weights_path, int /*block_pixels*/) {
    try {
        return create(weights_path, {-1});
    } catch (const std::exception &e) {
        std::fprintf(stderr, "tc_create: %s\n", e.what());
        return nullptr;
    }
}

void *tc_create_multi(const char *weights_path, const int *devices, int ndev) {
    try {
        if (ndev < 1) throw std::runtime_error("ndev must be >= 1");
        std::vector<int> dv(ndev);
        for (int i = 0; i < ndev; ++i) dv[i] = devices ? devices[i] : i;
        return create(weights_path, dv);
    } catch (const std::exception &e) {
        std::fprintf(stderr, "tc_create: %s\n", e.what());
        return nullptr;
    }
}

int tc_encode(void *handle, const float *s2, int64_t G, int64_t T2, const float *s1, int64_t T1, float *out) {
    try {
        if (!handle) throw std::runtime_error("null handle");
        if (G <= 0) return 0;
        if (!s2 || !s1 || !out) throw std::runtime_error("null buffer");
        Handle &h = *static_cast<Handle *>(handle);
        encode_records(*h.devs[0], s2, G, T2, s1, T1, out);
        return 0;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "tc_encode: %s\n", e.what());
        return -1;
    }
}

int tc_encode_tile_rows(void *handle, const uint16_t *bands, const uint8_t *masks, const uint16_t *doys,
                        const int16_t *asc, const int16_t *asc_doy, const int16_t *desc, const int16_t *desc_doy,
                        int64_t T2, int64_t Ta, int64_t Td, int64_t H, int64_t W, int64_t row0, int64_t row1,
                        int8_t *codes, float *scales) {
    try {
        if (!handle) throw std::runtime_error("null handle");
        Handle &h = *static_cast<Handle *>(handle);
        TileHost t{bands, masks, doys, asc, asc_doy, desc, desc_doy, T2, Ta, Td, H, W};
        tile_rows(h, t, row0, row1, codes, scales);
        return 0;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "tc_encode_tile: %s\n", e.what());
        return -1;
    }
}

int tc_encode_tile(void *handle, const uint16_t *bands, const uint8_t *masks, const uint16_t *doys, const int16_t *asc,
                   const int16_t *asc_doy, const int16_t *desc, const int16_t *desc_doy, int64_t T2, int64_t Ta,
                   int64_t Td, int64_t H, int64_t W, int8_t *codes, float *scales) {
    return tc_encode_tile_rows(handle, bands, masks, doys, asc, asc_doy, desc, desc_doy, T2, Ta, Td, H, W, 0, H, codes,
                               scales);
}

int tc_encode_tile_device(void *handle, const uint16_t *bands, const uint8_t *masks, const uint16_t *doys,
                          const int16_t *asc, const int16_t *asc_doy, const int16_t *desc, const int16_t *desc_doy,
                          int64_t T2, int64_t Ta, int64_t Td, int64_t H, int64_t W, int64_t row0, int64_t row1,
                          int8_t *codes, float *scales) {
    try {
        if (!handle) throw std::runtime_error("null handle");
        Handle &h = *static_cast<Handle *>(handle);
        if (h.devs.size() != 1) throw std::runtime_error("device-resident encode needs a single-device handle");
        if (row0 < 0 || row1 > H || row0 > row1 || T2 < 0 || Ta < 0 || Td < 0) throw std::runtime_error("bad arguments");
        if (T2 > MAX_STEPS || Ta + Td > MAX_STEPS) throw std::runtime_error("series longer than supported");
        Dev &d = *h.devs[0];
        CK(cudaSetDevice(d.device));
        TileDev t;
        t.bands = bands; t.masks = masks; t.doys = doys; t.asc = asc; t.asc_doy = asc_doy;
        t.desc = desc; t.desc_doy = desc_doy; t.T2 = T2; t.Ta = Ta; t.Td = Td; t.N = H * W;
        const int64_t p0 = row0 * W;
        encode_band(d, t, p0, (row1 - row0) * W, codes + p0 * OUT, scales + p0);
        d.mark(TC_CAT_D2H);
        CK(cudaStreamSynchronize(d.st));
        CK(cudaGetLastError());
        d.harvest();
        check_status(d);
        d.stats.calls += 1;
        return 0;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "tc_encode_tile: %s\n", e.what());
        return -1;
    }
}

int tc_plan_rows(const uint8_t *masks, const int16_t *asc, const int16_t *desc, int64_t T2, int64_t Ta, int64_t Td,
                 int64_t H, int64_t W, int nparts, int64_t *row_bounds) {
    try {
        if (nparts < 1 || !row_bounds || H < 0 || W < 0) throw std::runtime_error("bad arguments");
        if ((T2 && !masks) || (Ta && !asc) || (Td && !desc)) throw std::runtime_error("null input array");
        auto b = plan_rows(masks, asc, desc, T2, Ta, Td, H, W, nparts);
        for (int i = 0; i <= nparts; ++i) row_bounds[i] = b[i];
        return 0;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "tc_plan_rows: %s\n", e.what());
        return -1;
    }
}

void *tc_host_alloc(int64_t bytes) {
    if (bytes <= 0) return nullptr;
    void *p = nullptr;
    cudaError_t e = cudaHostAlloc(&p, (size_t)bytes, cudaHostAllocPortable);
    if (e != cudaSuccess) {
        std::fprintf(stderr, "tc_host_alloc: %s\n", cudaGetErrorString(e));
        return nullptr;
    }
    return p;
}

void tc_host_free(void *p) {
    if (p) cudaFreeHost(p);
}

int tc_set_stream(void *handle, void *stream) {
    if (!handle) return -1;
    Handle &h = *static_cast<Handle *>(handle);
    if (h.devs.size() != 1) return -1;
    Dev &d = *h.devs[0];
    d.st = stream ? static_cast<cudaStream_t>(stream) : d.own;
    return 0;
}

int tc_set_profiling(void *handle, int enable) {
    if (!handle) return -1;
    for (auto &d : static_cast<Handle *>(handle)->devs) d->prof = enable != 0;
    return 0;
}

int tc_get_stats(void *handle, tc_stats *out) {
    if (!handle || !out) return -1;
    std::memset(out, 0, sizeof(*out));
    for (auto &d : static_cast<Handle *>(handle)->devs) {
        const tc_stats &s = d->stats;
        out->calls = std::max(out->calls, s.calls);
        out->pixels += s.pixels;
        out->tokens += s.tokens;
        out->alg_flop += s.alg_flop;
        out->gemm_flop += s.gemm_flop;
        out->gemm_launches += s.gemm_launches;
        out->launches += s.launches;
        for (int k = 0; k < TC_CAT_N; ++k) out->ms_cat[k] += s.ms_cat[k];
        for (int k = 0; k < 6; ++k) {
            out->gemm_ms_kind[k] += s.gemm_ms_kind[k];
            out->gemm_flop_kind[k] += s.gemm_flop_kind[k];
        }
    }
    return 0;
}

void tc_reset_stats(void *handle) {
    if (!handle) return;
    for (auto &d : static_cast<Handle *>(handle)->devs) d->stats = tc_stats{};
}

void tc_profile_dump(void *handle) {
    if (!handle) return;
    Handle &h = *static_cast<Handle *>(handle);
    static const char *names[TC_CAT_N] = {"host->device copy", "input prep", "embedding (K=10/2)", "tcgen05 GEMMs",
                                          "attention", "LayerNorm", "attention pooling", "head LN + quant",
                                          "device->host copy"};
    tc_stats s;
    tc_get_stats(handle, &s);
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, h.devs[0]->device);
    std::printf("TCPROF b200 devices=%zu (%s) calls=%.0f px=%.0f tokens=%.0f launches=%.0f gemm_launches=%.0f\n",
                h.devs.size(), prop.name, s.calls, s.pixels, s.tokens, s.launches, s.gemm_launches);
    double tot = 0;
    for (int k = 0; k < TC_CAT_N; ++k) tot += s.ms_cat[k];
    if (tot > 0) {
        for (int k = 0; k < TC_CAT_N; ++k)
            std::printf("TCPROF %-20s %9.2f ms %5.1f%%\n", names[k], s.ms_cat[k], 100.0 * s.ms_cat[k] / tot);
        if (s.ms_cat[TC_CAT_GEMM] > 0)
            std::printf("TCPROF GEMM throughput %.1f TFLOP/s over %.3g FLOP\n",
                        s.gemm_flop / (s.ms_cat[TC_CAT_GEMM] * 1e-3) / 1e12, s.gemm_flop);
        static const char *kinds[6] = {"emb2+DOY", "QKV", "out-proj+res", "FFN1+ReLU", "FFN2+res", "head"};
        for (int k = 0; k < 6; ++k)
            if (s.gemm_ms_kind[k] > 0)
                std::printf("TCPROF   GEMM %-13s %9.2f ms %7.1f TFLOP/s\n", kinds[k], s.gemm_ms_kind[k],
                            s.gemm_flop_kind[k] / (s.gemm_ms_kind[k] * 1e-3) / 1e12);
    } else {
        std::printf("TCPROF per-category timing disabled (tc_set_profiling)\n");
    }
    std::fflush(stdout);
}

void tc_destroy(void *handle) {
    if (!handle) return;
    delete static_cast<Handle *>(handle);
}

// ------------------------------------------------------------------ per-op entry points
#define OP_TRY(name, body)                                                                         \
    try {                                                                                          \
        body;                                                                                      \
        CK(cudaGetLastError());                                                                    \
        return 0;                                                                                  \
    } catch (const std::exception &e) {                                                           \
        std::fprintf(stderr, "%s: %s\n", name, e.what());                                          \
        return -1;                                                                                 \
    }

int tcb_op_gemm(const void *A, int lda, const void *W, const float *bias, int relu, const void *res, int ldr,
                const float *pe_doy, int pe_stride, const void *pe_table, const float *pe_div, void *out, int ldo, int M,
                int N, int K, int bn, int variant, int *status, void *stream) {
    OP_TRY("tcb_op_gemm", {
        GemmArgs p;
        p.M = M; p.N = N; p.K = K; p.bias = bias; p.relu = relu;
        p.res = static_cast<const bf16 *>(res); p.ldr = ldr;
        p.pe_doy = pe_doy; p.pe_stride = pe_stride;
        p.pe_table = static_cast<const bf16 *>(pe_table); p.pe_div = pe_div;
        p.out = static_cast<bf16 *>(out); p.ldo = ldo; p.status = status;
        launch_gemm(p, static_cast<const bf16 *>(A), lda, static_cast<const bf16 *>(W),
                    static_cast<cudaStream_t>(stream), bn, 0, variant);
    })
}

int tcb_op_gemm_ln(const void *A, int lda, const void *W, const float *bias, const void *res, int ldr,
                   const float *ln_g, const float *ln_b, void *out, int ldo, int M, int K, int *status, void *stream) {
    OP_TRY("tcb_op_gemm_ln", {
        GemmArgs p;
        p.M = M; p.N = 640; p.K = K; p.bias = bias;
        p.res = static_cast<const bf16 *>(res); p.ldr = ldr;
        p.out = static_cast<bf16 *>(out); p.ldo = ldo; p.status = status;
        p.ln_g = ln_g; p.ln_b = ln_b;
        launch_gemm(p, static_cast<const bf16 *>(A), lda, static_cast<const bf16 *>(W),
                    static_cast<cudaStream_t>(stream));
    })
}

int tcb_op_count(const uint8_t *masks, const int16_t *asc, const int16_t *desc, int64_t T2, int64_t Ta, int64_t Td,
                 int64_t N, int64_t p0, int64_t np, int32_t *n2, int32_t *n1, void *stream) {
    OP_TRY("tcb_op_count", {
        TileDev t;
        t.masks = masks; t.asc = asc; t.desc = desc; t.T2 = T2; t.Ta = Ta; t.Td = Td; t.N = N;
        launch_count(t, p0, np, n2, n1, static_cast<cudaStream_t>(stream));
    })
}

int tcb_op_gather(int modality, const uint16_t *bands, const uint8_t *masks, const uint16_t *doys, const int16_t *asc,
                  const int16_t *asc_doy, const int16_t *desc, const int16_t *desc_doy, int64_t T2, int64_t Ta,
                  int64_t Td, int64_t N, int64_t p0, int64_t np, const int32_t *bins, const int64_t *off, float *rec,
                  void *stream) {
    OP_TRY("tcb_op_gather", {
        TileDev t;
        t.bands = bands; t.masks = masks; t.doys = doys; t.asc = asc; t.asc_doy = asc_doy;
        t.desc = desc; t.desc_doy = desc_doy; t.T2 = T2; t.Ta = Ta; t.Td = Td; t.N = N;
        launch_gather(modality, t, p0, np, nullptr, bins, Segs{off, 0, 0}, rec, static_cast<cudaStream_t>(stream));
    })
}

int tcb_op_emb1(int C, const float *rec, int64_t M, const float *w1t, const float *b1, void *y, void *stream) {
    OP_TRY("tcb_op_emb1", launch_emb1(C, rec, M, w1t, b1, static_cast<bf16 *>(y), static_cast<cudaStream_t>(stream)))
}

namespace {
struct DevFree {
    void operator()(int32_t *p) const { cudaFree(p); }
};
using DevList = std::unique_ptr<int32_t, DevFree>;
}  // namespace

int tcb_op_attention(const void *qkv, const int64_t *off, int64_t uniform_T, int64_t npix, int Tmax, void *att,
                     void *stream) {
    OP_TRY("tcb_op_attention", {
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (!off || npix <= 0) {
            launch_attention(static_cast<const bf16 *>(qkv), Segs{nullptr, 0, uniform_T}, npix, npix * uniform_T,
                             Tmax, static_cast<bf16 *>(att), nullptr, st);
        } else {
            // the offsets are read back to list the pixels by attention class, as
            // the tile path does; the qkv rows the segments reach are off[npix]
            std::vector<int64_t> ho((size_t)npix + 1);
            std::vector<int32_t> list((size_t)npix);
            CK(cudaMemcpyAsync(ho.data(), off, (npix + 1) * sizeof(int64_t), cudaMemcpyDeviceToHost, st));
            CK(cudaStreamSynchronize(st));
            for (int64_t i = 0; i < npix; ++i)
                if (ho[i + 1] - ho[i] > Tmax) throw std::runtime_error("a segment is longer than Tmax");
            AttnPlan plan;
            attention_plan(ho.data(), npix, list.data(), plan);
            int32_t *dl = nullptr;
            CK(cudaMalloc(&dl, std::max<size_t>(list.size(), 1) * sizeof(int32_t)));
            const DevList guard(dl);
            CK(cudaMemcpyAsync(dl, list.data(), list.size() * sizeof(int32_t), cudaMemcpyHostToDevice, st));
            plan.pix = dl;
            launch_attention_plan(static_cast<const bf16 *>(qkv), Segs{off, 0, 0}, plan, ho[npix],
                                  static_cast<bf16 *>(att), nullptr, st);
            CK(cudaStreamSynchronize(st));
        }
    })
}

int tcb_op_layernorm640(const void *x, int64_t M, const float *g, const float *b, void *y, void *stream) {
    OP_TRY("tcb_op_layernorm640", launch_layernorm640(static_cast<const bf16 *>(x), M, g, b, static_cast<bf16 *>(y),
                                                      static_cast<cudaStream_t>(stream)))
}

int tcb_op_pool(const void *x, const int64_t *off, int64_t uniform_T, int64_t npix, const float *q, float qb,
                void *fused, int col0, void *stream) {
    OP_TRY("tcb_op_pool", launch_pool(static_cast<const bf16 *>(x), Segs{off, 0, uniform_T}, npix, q, qb,
                                      static_cast<bf16 *>(fused), col0, static_cast<cudaStream_t>(stream)))
}

int tcb_op_ln_relu2560(void *r, int64_t P, const float *g, const float *b, void *stream) {
    OP_TRY("tcb_op_ln_relu2560", launch_ln_relu2560(static_cast<bf16 *>(r), P, g, b, static_cast<cudaStream_t>(stream)))
}

int tcb_op_out128(const void *r2, int64_t P, const uint8_t *empty, float *out, int8_t *codes, float *scales,
                  void *stream) {
    OP_TRY("tcb_op_out128", launch_out128(static_cast<const bf16 *>(r2), P, empty, out, codes, scales,
                                          static_cast<cudaStream_t>(stream)))
}

int tcb_attention_plan(const int64_t *off, int64_t npix, int32_t *list, int64_t *n, int32_t *tmax) {
    // host arithmetic only: no CUDA call, so it runs without a GPU
    try {
        if (!off || !list || !n || !tmax || npix < 0) throw std::runtime_error("bad arguments");
        for (int64_t i = 0; i < npix; ++i)
            if (off[i + 1] < off[i]) throw std::runtime_error("decreasing offsets");
        AttnPlan plan;
        attention_plan(off, npix, list, plan);
        for (int c = 0; c < 3; ++c) {
            n[c] = plan.n[c];
            tmax[c] = plan.tmax[c];
        }
        return 0;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "tcb_attention_plan: %s\n", e.what());
        return -1;
    }
}

int tcb_op_wait_probe(int64_t limit_us, int *status, void *stream) {
    OP_TRY("tcb_op_wait_probe", launch_wait_probe((uint64_t)std::max<int64_t>(limit_us, 0) * 1000, status,
                                                  static_cast<cudaStream_t>(stream)))
}

}  // extern "C"
