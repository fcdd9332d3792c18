// Warp-level kernels of the pixel-student forward pass: input preparation
// (valid counts, pad pattern, gather + z-score), the K=10/2 embedding layer,
// per-pixel self-attention, LayerNorm, attention pooling and the head's
// LayerNorms with the int8 quantisation.
//
// Rounding follows the reference CPU back end (tessera_cpu.cpp) and driver
// (tessera_encode.cpp): inputs z-scored in f32 with IEEE division, bf16 RNE at
// every layer boundary, f32 statistics and softmax.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gemm_sm100.h"
#include "kernels.h"

namespace tcb {

// ------------------------------------------------------------------ constants
// Standardisation constants of tessera_v2_student (tessera_encode.cpp:60-67).
__constant__ float c_s2_mean[10] = {1633.0042f, 1341.1090f, 1539.5536f, 3054.8269f, 3117.4658f,
                                    2004.1648f, 2694.7275f, 2945.1504f, 2266.6079f, 1657.3094f};
__constant__ float c_s2_std[10] = {1999.4603f, 2014.7549f, 1929.2201f, 1754.2493f, 1649.9807f,
                                   1936.8988f, 1748.6041f, 1708.6991f, 1207.5250f, 1108.6046f};
__constant__ float c_s1a_mean[2] = {5909.3921f, 3405.0322f};
__constant__ float c_s1a_std[2] = {1507.1750f, 1531.2615f};
__constant__ float c_s1d_mean[2] = {5816.1382f, 3277.7576f};
__constant__ float c_s1d_std[2] = {1554.6475f, 1546.4733f};
constexpr float Z_EPS = 1e-9f;

__device__ __forceinline__ int64_t seg_at(const Segs &s, int64_t i) {
    return s.off ? s.off[i] - s.base : i * s.uniform_T;
}
// The chunk segment that segment k of an attention launch stands for.
__device__ __forceinline__ int64_t seg_pix(const Segs &s, int64_t k) { return s.pix ? (int64_t)s.pix[k] : k; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

static void check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// ------------------------------------------------------------------ prep
// Valid counts: S2 mask != 0; S1 either band != 0 (tessera_encode.cpp:249-255).
__global__ void k_count(TileDev t, int64_t p0, int64_t np, int32_t *n2, int32_t *n1) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= np) return;
    const int64_t p = p0 + i, N = t.N;
    int c2 = 0, c1 = 0;
    for (int64_t s = 0; s < t.T2; ++s) c2 += t.masks[s * N + p] != 0;
    const uint32_t *a = reinterpret_cast<const uint32_t *>(t.asc);
    const uint32_t *d = reinterpret_cast<const uint32_t *>(t.desc);
    for (int64_t s = 0; s < t.Ta; ++s) c1 += a[s * N + p] != 0u;
    for (int64_t s = 0; s < t.Td; ++s) c1 += d[s * N + p] != 0u;
    n2[i] = c2;
    n1[i] = c1;
}

// _pad_pattern(n, B)[k] for n > 0 (tessera_encode.cpp:154-180): numpy
// linspace floor when n >= B, middle of each array_split group when the
// shortfall is at most n, otherwise modulo fill.
__device__ __forceinline__ int64_t pad_index(int64_t n, int64_t B, int64_t k) {
    if (n >= B) {
        if (B == 1) return 0;
        if (k == B - 1) return n - 1;
        const double delta = double(n - 1), div = double(B - 1), step = delta / div;
        const double y = step == 0 ? (double(k) / div) * delta : double(k) * step;
        return (int64_t)floor(y);
    }
    if (k < n) return k;
    const int64_t g = k - n, remain = B - n;
    if (remain <= n) {
        const int64_t q = n / remain, r = n % remain;
        const int64_t start = g * q + (g < r ? g : r);
        const int64_t len = q + (g < r ? 1 : 0);
        return start + len / 2;
    }
    return g % n;
}

// One warp per pixel: ordered valid-step list by ballot, then B padded steps.
template <int MOD>
__global__ void __launch_bounds__(128) k_gather(TileDev t, int64_t p0, int64_t np, const int32_t *bins, Segs segs,
                                                float *rec) {
    constexpr int C = MOD == 0 ? 10 : 2;
    __shared__ uint16_t lists[4][MAX_STEPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t i = (int64_t)blockIdx.x * 4 + warp;
    if (i >= np) return;
    const int64_t B = bins[i];
    if (B <= 0) return;
    const int64_t p = p0 + i, N = t.N;
    const int64_t Tsteps = MOD == 0 ? t.T2 : t.Ta + t.Td;
    uint16_t *list = lists[warp];
    const uint32_t *a32 = reinterpret_cast<const uint32_t *>(t.asc);
    const uint32_t *d32 = reinterpret_cast<const uint32_t *>(t.desc);
    int nv = 0;
    for (int64_t base = 0; base < Tsteps; base += 32) {
        const int64_t s = base + lane;
        bool v = false;
        if (s < Tsteps) {
            if (MOD == 0) v = t.masks[s * N + p] != 0;
            else v = (s < t.Ta ? a32[s * N + p] : d32[(s - t.Ta) * N + p]) != 0u;
        }
        const uint32_t m = __ballot_sync(0xffffffffu, v);
        if (v) list[nv + __popc(m & ((1u << lane) - 1u))] = (uint16_t)s;
        nv += __popc(m);
    }
    __syncwarp();
    float *out = rec + seg_at(segs, i) * (C + 1);
    for (int64_t k = lane; k < B; k += 32) {
        float *row = out + k * (C + 1);
        if (nv == 0) {  // empty modality: one all-zero row (tessera_encode.cpp:275,279-280)
#pragma unroll
            for (int c = 0; c <= C; ++c) row[c] = 0.f;
            continue;
        }
        const int64_t s = list[pad_index(nv, B, k)];
        if (MOD == 0) {
            const uint16_t *src = t.bands + (s * N + p) * 10;
#pragma unroll
            for (int c = 0; c < 10; ++c) row[c] = (float(src[c]) - c_s2_mean[c]) / (c_s2_std[c] + Z_EPS);
            row[10] = float(t.doys[s]);
        } else if (s < t.Ta) {
            const int16_t *v = t.asc + (s * N + p) * 2;
#pragma unroll
            for (int c = 0; c < 2; ++c) row[c] = (float(v[c]) - c_s1a_mean[c]) / (c_s1a_std[c] + Z_EPS);
            row[2] = float(t.asc_doy[s]);
        } else {
            const int16_t *v = t.desc + ((s - t.Ta) * N + p) * 2;
#pragma unroll
            for (int c = 0; c < 2; ++c) row[c] = (float(v[c]) - c_s1d_mean[c]) / (c_s1d_std[c] + Z_EPS);
            row[2] = float(t.desc_doy[s - t.Ta]);
        }
    }
}

// ------------------------------------------------------------------ emb1
// Warp per token pair; lane computes columns lane*4 + 128*j (j < 5) of two
// tokens, so each float4 of weights read from shared memory serves both.
// Every output is fmaf over k = 0..C-1 in order, then + bias, then ReLU.
template <int C>
__global__ void __launch_bounds__(256) k_emb1(const float *__restrict__ rec, int64_t M, const float *__restrict__ w1t,
                                              const float *__restrict__ b1, bf16 *__restrict__ y) {
    __shared__ __align__(16) float ws[C * D];
    __shared__ __align__(16) float bs[D];
    for (int i = threadIdx.x; i < C * D; i += blockDim.x) ws[i] = w1t[i];
    for (int i = threadIdx.x; i < D; i += blockDim.x) bs[i] = b1[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = ((int64_t)blockIdx.x * (blockDim.x >> 5) + warp) * 2; r < M; r += nwarps * 2) {
        const bool two = r + 1 < M;
        float a[2][C];
#pragma unroll
        for (int k = 0; k < C; ++k) {
            a[0][k] = bf16_round(__ldg(rec + r * (C + 1) + k));
            a[1][k] = two ? bf16_round(__ldg(rec + (r + 1) * (C + 1) + k)) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            const int n = j * 128 + lane * 4;
            float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < C; ++k) {
                const float4 wk = *reinterpret_cast<const float4 *>(ws + k * D + n);
                s0[0] = fmaf(a[0][k], wk.x, s0[0]); s0[1] = fmaf(a[0][k], wk.y, s0[1]);
                s0[2] = fmaf(a[0][k], wk.z, s0[2]); s0[3] = fmaf(a[0][k], wk.w, s0[3]);
                s1[0] = fmaf(a[1][k], wk.x, s1[0]); s1[1] = fmaf(a[1][k], wk.y, s1[1]);
                s1[2] = fmaf(a[1][k], wk.z, s1[2]); s1[3] = fmaf(a[1][k], wk.w, s1[3]);
            }
            const float4 bb = *reinterpret_cast<const float4 *>(bs + n);
            *reinterpret_cast<uint2 *>(y + r * D + n) =
                make_uint2(pack_bf16x2(fmaxf(s0[0] + bb.x, 0.f), fmaxf(s0[1] + bb.y, 0.f)),
                           pack_bf16x2(fmaxf(s0[2] + bb.z, 0.f), fmaxf(s0[3] + bb.w, 0.f)));
            if (two)
                *reinterpret_cast<uint2 *>(y + (r + 1) * D + n) =
                    make_uint2(pack_bf16x2(fmaxf(s1[0] + bb.x, 0.f), fmaxf(s1[1] + bb.y, 0.f)),
                               pack_bf16x2(fmaxf(s1[2] + bb.z, 0.f), fmaxf(s1[3] + bb.w, 0.f)));
        }
    }
}

// ------------------------------------------------------------------ attention
constexpr int ATT_LD = HD + 8;  // smem row pitch of K/V tiles (336 B): conflict-free ldmatrix

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void *gptr) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// One CTA per (pixel, head); NTMAX = key tiles of 8 the kernel is built for
// (Tpad <= 8 * NTMAX). K and V of the head are staged in shared memory with
// cp.async; each warp owns 16 query rows at a time:
//   S = bf16(scale * Q K^T) over all keys, four independent key tiles in flight,
//   softmax in f32 over the T valid keys (only tile padding is masked), P = bf16,
//   O = bf16(P V) in two 80-column halves to bound register use
// (tessera_cpu.cpp:333-343: matmul + linear post-op, softmax_accurate, matmul).
template <int NTMAX>
__global__ void __launch_bounds__(NTMAX == 24 ? 512 : 256, NTMAX <= 16 ? 2 : 1)
    k_attention(const bf16 *__restrict__ qkv, Segs segs, bf16 *__restrict__ att, float scale) {
    extern __shared__ __align__(16) uint8_t att_smem[];
    const int64_t i = seg_pix(segs, blockIdx.x);
    const int h = blockIdx.y;
    const int64_t t0 = seg_at(segs, i);
    const int T = (int)(seg_at(segs, i + 1) - t0);
    if (T <= 0) return;
    const int Tpad = (T + 15) & ~15;
    bf16 *Ks = reinterpret_cast<bf16 *>(att_smem);
    bf16 *Vs = Ks + Tpad * ATT_LD;
    const uint32_t ks_base = smem_u32(Ks), vs_base = smem_u32(Vs);
    for (int idx = threadIdx.x; idx < Tpad * (HD / 8); idx += blockDim.x) {
        const int r = idx / (HD / 8), c = idx % (HD / 8);
        const uint32_t off = (uint32_t)((r * ATT_LD + c * 8) * 2);
        if (r < T) {
            const bf16 *row = qkv + (t0 + r) * (3 * D) + h * HD + c * 8;
            cp_async16(ks_base + off, row + D);
            cp_async16(vs_base + off, row + 2 * D);
        } else {
            *reinterpret_cast<uint4 *>(Ks + r * ATT_LD + c * 8) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4 *>(Vs + r * ATT_LD + c * 8) = make_uint4(0, 0, 0, 0);
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
    const int nwarps = blockDim.x >> 5;
    const int nrb = Tpad / 16, nnt = Tpad / 8;
    // Q fragments straight from global; the first row block's loads are in
    // flight together with the K/V staging.
    uint32_t qa[HD / 16][4];
    auto load_q = [&](int rb) {
        const int r0 = rb * 16 + g, r1 = r0 + 8;
        const uint32_t *q0 = r0 < T ? reinterpret_cast<const uint32_t *>(qkv + (t0 + r0) * (3 * D) + h * HD) : nullptr;
        const uint32_t *q1 = r1 < T ? reinterpret_cast<const uint32_t *>(qkv + (t0 + r1) * (3 * D) + h * HD) : nullptr;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            qa[ks][0] = q0 ? __ldg(q0 + ks * 8 + tq) : 0u;
            qa[ks][1] = q1 ? __ldg(q1 + ks * 8 + tq) : 0u;
            qa[ks][2] = q0 ? __ldg(q0 + ks * 8 + 4 + tq) : 0u;
            qa[ks][3] = q1 ? __ldg(q1 + ks * 8 + 4 + tq) : 0u;
        }
    };
    if (warp < nrb) load_q(warp);
    cp_async_wait_all();
    __syncthreads();
    for (int rb = warp; rb < nrb; rb += nwarps) {
        const int r0 = rb * 16 + g, r1 = r0 + 8;
        if (rb != warp) load_q(rb);
        // S tiles, packed bf16: sp[nt][0] row r0 cols (nt*8 + 2tq, +1), sp[nt][1] row r1.
        uint32_t sp[NTMAX][2];
#pragma unroll
        for (int nt0 = 0; nt0 < NTMAX; nt0 += 4) {
            if (nt0 < nnt) {
                float c[4][4];
#pragma unroll
                for (int j = 0; j < 4; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
#pragma unroll
                for (int ks = 0; ks < HD / 16; ks += 2) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (nt0 + j < nnt) {
                            const uint32_t addr =
                                ks_base + (uint32_t)((((nt0 + j) * 8 + (lane & 7)) * ATT_LD + (lane >> 3) * 8 + ks * 16) * 2);
                            uint32_t b0, b1, b2, b3;
                            ldsm_x4(addr, b0, b1, b2, b3);
                            mma_bf16_16816(c[j], qa[ks], b0, b1);
                            mma_bf16_16816(c[j], qa[ks + 1], b2, b3);
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (nt0 + j < NTMAX) {
                        const int col = (nt0 + j) * 8 + 2 * tq;
                        const float ninf = -INFINITY;
                        const float s0 = col < T ? c[j][0] * scale : ninf, s1 = col + 1 < T ? c[j][1] * scale : ninf;
                        const float s2 = col < T ? c[j][2] * scale : ninf, s3 = col + 1 < T ? c[j][3] * scale : ninf;
                        sp[nt0 + j][0] = pack_bf16x2(s0, s1);
                        sp[nt0 + j][1] = pack_bf16x2(s2, s3);
                    }
                }
            }
        }
        // softmax over keys: rows r0 (sp[.][0]) and r1 (sp[.][1]); a row lives in one lane quad
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < NTMAX; ++nt)
            if (nt < nnt) {
                mx0 = fmaxf(mx0, fmaxf(bf16lo(sp[nt][0]), bf16hi(sp[nt][0])));
                mx1 = fmaxf(mx1, fmaxf(bf16lo(sp[nt][1]), bf16hi(sp[nt][1])));
            }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        float z0 = 0.f, z1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < NTMAX; ++nt)
            if (nt < nnt) {
                z0 += __expf(bf16lo(sp[nt][0]) - mx0) + __expf(bf16hi(sp[nt][0]) - mx0);
                z1 += __expf(bf16lo(sp[nt][1]) - mx1) + __expf(bf16hi(sp[nt][1]) - mx1);
            }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
            z0 += __shfl_xor_sync(0xffffffffu, z0, o);
            z1 += __shfl_xor_sync(0xffffffffu, z1, o);
        }
        const float inv0 = 1.f / z0, inv1 = 1.f / z1;
#pragma unroll
        for (int nt = 0; nt < NTMAX; ++nt)
            if (nt < nnt) {
                sp[nt][0] = pack_bf16x2(__expf(bf16lo(sp[nt][0]) - mx0) * inv0, __expf(bf16hi(sp[nt][0]) - mx0) * inv0);
                sp[nt][1] = pack_bf16x2(__expf(bf16lo(sp[nt][1]) - mx1) * inv1, __expf(bf16hi(sp[nt][1]) - mx1) * inv1);
            }
        // O = P V, in two halves of 80 columns
        uint32_t *dst0 = r0 < T ? reinterpret_cast<uint32_t *>(att + (t0 + r0) * D + h * HD) : nullptr;
        uint32_t *dst1 = r1 < T ? reinterpret_cast<uint32_t *>(att + (t0 + r1) * D + h * HD) : nullptr;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            float o[HD / 16][4];
#pragma unroll
            for (int dn = 0; dn < HD / 16; ++dn) o[dn][0] = o[dn][1] = o[dn][2] = o[dn][3] = 0.f;
#pragma unroll
            for (int kt = 0; kt < NTMAX / 2; ++kt) {
                if (kt < nrb) {
                    const uint32_t a[4] = {sp[2 * kt][0], sp[2 * kt][1], sp[2 * kt + 1][0], sp[2 * kt + 1][1]};
                    const int vrow = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                    const uint32_t addr = vs_base + (uint32_t)((vrow * ATT_LD + half * (HD / 2) + (lane >> 4) * 8) * 2);
#pragma unroll
                    for (int dn2 = 0; dn2 < HD / 32; ++dn2) {
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4_t(addr + dn2 * 32, b0, b1, b2, b3);
                        mma_bf16_16816(o[2 * dn2], a, b0, b1);
                        mma_bf16_16816(o[2 * dn2 + 1], a, b2, b3);
                    }
                }
            }
            if (dst0) {
#pragma unroll
                for (int dn = 0; dn < HD / 16; ++dn) dst0[half * (HD / 4) + dn * 4 + tq] = pack_bf16x2(o[dn][0], o[dn][1]);
            }
            if (dst1) {
#pragma unroll
                for (int dn = 0; dn < HD / 16; ++dn) dst1[half * (HD / 4) + dn * 4 + tq] = pack_bf16x2(o[dn][2], o[dn][3]);
            }
        }
    }
}

// ------------------------------------------------------------------ attention on tcgen05
// Persistent, one CTA per SM, over (pixel, head) items with T <= 128 keys.
//   warp 0       TMA, boxes of 32 rows x 64 columns with 128-byte swizzle,
//                three 64-column slabs per matrix covering the head's 160
//                columns. Lane 0: the item's Q and K rows into the one Q/K
//                stage, released once S has read it; lane 1: its V rows into
//                one of two V stages, each released once O has read it.
//   warp 1       TMEM allocation and MMA issue (one thread):
//                  S = Q K^T   A = Q, B = K (both K-major in shared memory), M = 128, N = Tpad
//                  O = P V     A = P from TMEM, B = V (MN-major), M = 128, N = 160
//                S of the next item is issued before O of this one, so it runs
//                while this item's softmax does; the Q/K rows of the item after
//                that load meanwhile.
//   warps 2-17   softmax: four warps per TMEM lane quadrant, one query row per
//                lane and 32 of the 128 key columns per warp. s = bf16(scale *
//                S) and the row max, e = exp(s - max) and the row sum, then
//                P = bf16(e / sum) over the T real keys back into TMEM. The
//                four partial maxima and sums of a row meet in shared memory
//                (one named barrier per quadrant).
//   warps 18-21  O rows -> bf16 -> att: 32 columns at a time through a 2 KB
//                staging buffer per warp, so that each store instruction
//                writes 8 rows x 64 contiguous bytes.
// Tensor memory (512 columns): two S/P buffers [96, 224) and [224, 352) (P
// overwrites the first Tpad/2 columns of its S), O [352, 512).
// Rows of K/V past T (up to the next multiple of 32) belong to the next pixel
// or are zero-filled past the chunk; S columns >= T are masked and P is 0
// there, so they never reach O. Rows of S, P and O >= T come from rows of Q
// that are not this item's and are never stored.
// Every mbarrier wait is bounded.
constexpr int AT_SLAB = 128 * 128;          // 128 rows x 64 bf16 = 16 KB
constexpr int AT_MAT = 3 * AT_SLAB;         // one matrix: three slabs
constexpr int AT_QK = 2 * AT_MAT;           // the Q/K stage
constexpr int AT_SOFT_WARPS = 16, AT_IO_WARP0 = 2 + AT_SOFT_WARPS;
constexpr int AT_THREADS = 32 * (AT_IO_WARP0 + 4);
constexpr int AT_RED_BYTES = 2 * 4 * 128 * 4;  // partial max and sum: [slice][row] floats
constexpr int AT_OSTAGE = 2048;                // per O warp: 32 rows x 64 bytes
constexpr int AT_RED_OFF = AT_QK + 2 * AT_MAT, AT_OST_OFF = AT_RED_OFF + AT_RED_BYTES,
              AT_BAR_OFF = AT_OST_OFF + 4 * AT_OSTAGE;
constexpr int AT_SMEM = 1024 + AT_BAR_OFF + 256;
constexpr uint32_t AT_SCOL0 = 96, AT_SCOL1 = 224, AT_OCOL = 352;

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__global__ void __launch_bounds__(AT_THREADS, 1)
    k_attention_tc(const __grid_constant__ CUtensorMap tm, Segs segs, int64_t nitems, bf16 *__restrict__ att,
                   float scale, int *status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *red_max = reinterpret_cast<float *>(smem + AT_RED_OFF), *red_sum = red_max + 4 * 128;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + AT_BAR_OFF);
    uint64_t *qk_full = bars, *qk_empty = bars + 1, *v_full = bars + 2, *v_empty = bars + 4;
    uint64_t *s_full = bars + 6, *p_full = bars + 8, *o_full = bars + 10, *o_free = bars + 11;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 12);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(qk_full, 1);
        mbar_init(qk_empty, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], AT_SOFT_WARPS);
        }
        mbar_init(o_full, 1);
        mbar_init(o_free, 4);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tensormap(&tm);
    }
    if (warp == 1) { tmem_alloc(tmem_holder, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = *tmem_holder;
    // Every role walks the items with 1 <= T <= 128 in the same order. A longer
    // series (a caller's Tmax below the real one) is skipped by all roles and
    // reported as a bad segment.
    auto item_at = [&](int64_t it, int64_t &t0, int &T, int &h) {
        const int64_t p = seg_pix(segs, it >> 2);
        h = (int)(it & 3);
        t0 = seg_at(segs, p);
        const int64_t len = seg_at(segs, p + 1) - t0;
        T = len > 128 ? 0 : (int)len;
        if (len > 128 && warp == 0 && lane == 0 && status) atomicCAS(status, 0, ERR_BAD_SEGMENT);
    };
    auto next_item = [&](int64_t it, int64_t &t0, int &T, int &h) -> int64_t {
        for (; it < nitems; it += gridDim.x) {
            item_at(it, t0, T, h);
            if (T > 0) break;
        }
        return it;
    };
    // The offsets of a candidate item, loaded before a barrier wait so that
    // their round trip overlaps the wait.
    struct Pf { int64_t a = 0, b = 0; };
    auto pf_load = [&](int64_t it) {
        Pf f;
        if (segs.off && it < nitems) {
            const int64_t p = seg_pix(segs, it >> 2);
            f.a = segs.off[p];
            f.b = segs.off[p + 1];
        }
        return f;
    };
    // next_item(it, ...) for a candidate whose offsets pf_load(it) fetched
    auto next_item_pf = [&](int64_t it, const Pf &f, int64_t &t0, int &T, int &h) -> int64_t {
        if (it >= nitems || !segs.off) return next_item(it, t0, T, h);
        h = (int)(it & 3);
        t0 = f.a - segs.base;
        const int64_t len = f.b - f.a;
        T = len > 128 ? 0 : (int)len;
        return T > 0 ? it : next_item(it + gridDim.x, t0, T, h);
    };

    if (warp == 0) {
        if (lane < 2) {  // lane 0 loads Q and K, lane 1 loads V
            int j = 0;
            int64_t t0;
            int T, h;
            for (int64_t it = next_item(blockIdx.x, t0, T, h); it < nitems; it = next_item(it + gridDim.x, t0, T, h)) {
                const int nb = (T + 31) >> 5;
                if (lane == 0) {
                    if (!mbar_wait(qk_empty, (j & 1) ^ 1, abort_flag, status, ERR_WAIT_SMEM_EMPTY)) break;
                    mbar_arrive_expect_tx(qk_full, (uint32_t)(nb * 2 * 3 * 32 * 128));
                    for (int rb = 0; rb < nb; ++rb)
                        for (int sl = 0; sl < 3; ++sl) {
                            tma_load_2d(smem + sl * AT_SLAB + rb * 4096, &tm, h * HD + sl * 64, (int)t0 + rb * 32, qk_full);
                            tma_load_2d(smem + AT_MAT + sl * AT_SLAB + rb * 4096, &tm, D + h * HD + sl * 64,
                                        (int)t0 + rb * 32, qk_full);
                        }
                } else {
                    const int s = j & 1;
                    if (!mbar_wait(&v_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, status, ERR_WAIT_SMEM_EMPTY)) break;
                    mbar_arrive_expect_tx(&v_full[s], (uint32_t)(nb * 3 * 32 * 128));
                    uint8_t *dst = smem + AT_QK + s * AT_MAT;
                    for (int rb = 0; rb < nb; ++rb)
                        for (int sl = 0; sl < 3; ++sl)
                            tma_load_2d(dst + sl * AT_SLAB + rb * 4096, &tm, 2 * D + h * HD + sl * 64, (int)t0 + rb * 32,
                                        &v_full[s]);
                }
                ++j;
            }
            // every stage released: no MMA still reads shared memory at exit
            if (lane == 0) {
                mbar_wait(qk_empty, (j & 1) ^ 1, abort_flag, status, ERR_WAIT_SMEM_EMPTY);
            } else {
                for (int q = 0; q < 2; ++q, ++j)
                    if (!mbar_wait(&v_empty[j & 1], ((j >> 1) & 1) ^ 1, abort_flag, status, ERR_WAIT_SMEM_EMPTY)) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_o = umma_idesc_bf16_bmn(128, HD);
            int j = 0, prev_tpad = 0;
            bool ok = true;
            auto issue_pv = [&](int jj, int tpad) -> bool {
                const int b = jj & 1;
                if (!mbar_wait(&v_full[b], (jj >> 1) & 1, abort_flag, status, ERR_WAIT_TMA_FULL)) return false;
                if (!mbar_wait(&p_full[b], (jj >> 1) & 1, abort_flag, status, ERR_WAIT_TMEM_FULL)) return false;
                if (!mbar_wait(o_free, (jj & 1) ^ 1, abort_flag, status, ERR_WAIT_TMEM_EMPTY)) return false;
                tc_fence_after();
                const uint32_t pcol = b ? AT_SCOL1 : AT_SCOL0;
                const uint32_t sv = smem_u32(smem + AT_QK + b * AT_MAT);
                for (int k = 0; k < tpad / 16; ++k)
                    umma_bf16_tmem_a(tb + AT_OCOL, tb + pcol + (uint32_t)(k * 8),
                                     umma_desc_sw128_mn(sv + (uint32_t)(k * 16 * 128), AT_SLAB), idesc_o, k > 0);
                umma_commit(o_full);
                umma_commit(&v_empty[b]);
                return true;
            };
            const uint32_t sq = smem_u32(smem), sk = smem_u32(smem + AT_MAT);
            int64_t t0;
            int T, h;
            for (int64_t it = next_item(blockIdx.x, t0, T, h); it < nitems; it = next_item(it + gridDim.x, t0, T, h)) {
                const int b = j & 1, tpad = (T + 15) & ~15;
                // S(j)
                if (!mbar_wait(qk_full, j & 1, abort_flag, status, ERR_WAIT_TMA_FULL)) { ok = false; break; }
                // S(j) overwrites the S/P buffer of item j - 2: its O must be complete
                if (!mbar_wait(&v_empty[b], ((j >> 1) & 1) ^ 1, abort_flag, status, ERR_WAIT_TMEM_EMPTY)) { ok = false; break; }
                tc_fence_after();
                const uint32_t scol = b ? AT_SCOL1 : AT_SCOL0;
                const uint32_t idesc_s = umma_idesc_bf16(128, tpad);
#pragma unroll
                for (int k = 0; k < HD / 16; ++k) {
                    const uint32_t slab = (uint32_t)((k >> 2) * AT_SLAB);
                    umma_bf16(tb + scol, umma_desc_sw128(sq + slab) + (uint64_t)(2 * (k & 3)),
                              umma_desc_sw128(sk + slab) + (uint64_t)(2 * (k & 3)), idesc_s, k > 0);
                }
                umma_commit(&s_full[b]);
                umma_commit(qk_empty);
                // O(j - 1)
                if (j > 0 && !issue_pv(j - 1, prev_tpad)) { ok = false; break; }
                prev_tpad = tpad;
                ++j;
            }
            if (ok && j > 0) issue_pv(j - 1, prev_tpad);
        }
    } else if (warp < AT_IO_WARP0) {
        // softmax: quadrant = warp % 4 (the TMEM lanes this warp may access), 32-column slice
        const int quad = warp & 3, slice = (warp - 2) >> 2, r = quad * 32 + lane, c0 = slice * 32;
        const uint32_t lanebits = (uint32_t)(quad * 32) << 16;
        int j = 0;
        int64_t t0;
        int T, h;
        int64_t it = next_item(blockIdx.x, t0, T, h);
        while (it < nitems) {
            const int b = j & 1, tpad = (T + 15) & ~15;
            const uint32_t scol = (b ? AT_SCOL1 : AT_SCOL0) + (uint32_t)c0;
            const Pf pfn = pf_load(it + gridDim.x);
            if (!mbar_wait(&s_full[b], (j >> 1) & 1, abort_flag, status, ERR_WAIT_TMEM_FULL)) break;
            tc_fence_after();
            uint32_t v[2][16];  // 32 columns of the S row, then s, then e, as f32 bits
            if (c0 < tpad) tmem_ld16(tb + lanebits + scol, v[0]);
            if (c0 + 16 < tpad) tmem_ld16(tb + lanebits + scol + 16, v[1]);
            tmem_ld_wait();
            // 16-column halves past Tpad are skipped (the branch is uniform per warp)
            float mx = -INFINITY;
#pragma unroll
            for (int q = 0; q < 2; ++q)
                if (c0 + q * 16 < tpad) {
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int col = c0 + q * 16 + k;
                        const float x = col < T ? bf16_round(__uint_as_float(v[q][k]) * scale) : -INFINITY;
                        v[q][k] = __float_as_uint(x);
                        mx = fmaxf(mx, x);
                    }
                }
            red_max[slice * 128 + r] = mx;
            named_bar_sync(1 + quad, 128);
            mx = fmaxf(fmaxf(red_max[r], red_max[128 + r]), fmaxf(red_max[256 + r], red_max[384 + r]));
            float z = 0.f;
#pragma unroll
            for (int q = 0; q < 2; ++q)
                if (c0 + q * 16 < tpad) {
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const float ex = __expf(__uint_as_float(v[q][k]) - mx);  // 0 for masked columns
                        v[q][k] = __float_as_uint(ex);
                        z += ex;
                    }
                }
            red_sum[slice * 128 + r] = z;
            named_bar_sync(1 + quad, 128);
            z = ((red_sum[r] + red_sum[128 + r]) + red_sum[256 + r]) + red_sum[384 + r];
            const float inv = 1.f / z;
#pragma unroll
            for (int q = 0; q < 2; ++q)
                if (c0 + q * 16 < tpad) {
                    uint32_t w[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        w[k] = pack_bf16x2(__uint_as_float(v[q][2 * k]) * inv, __uint_as_float(v[q][2 * k + 1]) * inv);
                    tmem_st8(tb + lanebits + (b ? AT_SCOL1 : AT_SCOL0) + (uint32_t)(c0 / 2 + q * 8), w);
                }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
            it = next_item_pf(it + gridDim.x, pfn, t0, T, h);
            ++j;
        }
    } else {
        // O warps: each drains its TMEM lane quadrant (32 query rows) of O(j)
        const int quad = warp & 3;
        const uint32_t lanebits = (uint32_t)(quad * 32) << 16;
        uint8_t *stage = smem + AT_OST_OFF + (warp - AT_IO_WARP0) * AT_OSTAGE;
        uint4 *my_row = reinterpret_cast<uint4 *>(stage + lane * 64);
        const int sw = (lane >> 1) & 3;
        int j = 0;
        int64_t t0;
        int T, h;
        int64_t it = next_item(blockIdx.x, t0, T, h);
        while (it < nitems) {
            const Pf pfn = pf_load(it + gridDim.x);
            if (!mbar_wait(o_full, j & 1, abort_flag, status, ERR_WAIT_TMEM_FULL)) break;
            tc_fence_after();
            const int nrows = T - quad * 32;  // real rows of this quadrant (uniform per warp)
            if (nrows > 0) {
                bf16 *dst = att + (t0 + quad * 32) * D + h * HD;
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                    uint32_t v[16], w[16];
                    tmem_ld16(tb + lanebits + AT_OCOL + (uint32_t)(c * 32), v);
                    tmem_ld16(tb + lanebits + AT_OCOL + (uint32_t)(c * 32 + 16), w);
                    tmem_ld_wait();
                    uint32_t o[16];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        o[k] = pack_bf16x2(__uint_as_float(v[2 * k]), __uint_as_float(v[2 * k + 1]));
                        o[8 + k] = pack_bf16x2(__uint_as_float(w[2 * k]), __uint_as_float(w[2 * k + 1]));
                    }
                    // row-per-lane into the staging rows (16-byte chunks XOR-swizzled
                    // so the writes and the row-wise reads are conflict-free), then
                    // 8 rows x 64 bytes per store instruction
#pragma unroll
                    for (int k = 0; k < 4; ++k) my_row[k ^ sw] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int rr = i * 8 + (lane >> 2), k = lane & 3;
                        const uint4 val = reinterpret_cast<const uint4 *>(stage + rr * 64)[k ^ ((rr >> 1) & 3)];
                        if (rr < nrows) *reinterpret_cast<uint4 *>(dst + (int64_t)rr * D + c * 32 + k * 8) = val;
                    }
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);
            it = next_item_pf(it + gridDim.x, pfn, t0, T, h);
            ++j;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tb, 512);
}

// ------------------------------------------------------------------ attention, 128 < T <= 256 (tcgen05)
// Persistent, one CTA per SM, over (pixel, head, query half) items: half 0 is
// the query rows [0, 128), half 1 the rows [128, T); both attend over all T
// keys. The two halves of a head are adjacent items, so the second read of its
// K and V rows comes from L2.
//   warp 0       TMA, boxes of 32 rows x 32 columns with 64-byte swizzle,
//                five 32-column slabs per matrix covering the head's 160
//                columns exactly. Lane 0: the item's query rows into the Q
//                stage and its T key rows into the K stage, both released once
//                S has read them; lane 1: its T value rows into the V stage,
//                released once O has read it.
//   warp 1       TMEM allocation and MMA issue (one thread):
//                  S = Q K^T   A = Q, B = K (both K-major), M = 128, N = Tpad <= 256, 10 k-steps
//                  O = P V     A = P from TMEM, B = V (MN-major), M = 128, N = 160, Tpad / 16 k-steps
//                S of the next item waits until O of this one has read P, which
//                shares S's columns.
//   warps 2-17   softmax: four warps per TMEM lane quadrant, one query row per
//                lane and 64 of the 256 key columns per warp: s = bf16(scale *
//                S) and the row max, e = exp(s - max) and the row sum, then
//                P = bf16(e / sum) over the T real keys back into TMEM; the
//                four partial maxima and sums of a row meet in shared memory.
//   warps 18-21  O rows -> bf16 -> att, 32 columns at a time through a 2 KB
//                staging buffer per warp (8 rows x 64 contiguous bytes per store).
// Tensor memory (512 columns): S / P [0, 256) (P overwrites the first Tpad/2
// columns of S), O [256, 416).
// K/V rows past T (up to the next multiple of 32) belong to the next pixel or
// are zero-filled past the chunk; S columns >= T are masked and P is 0 there.
// Query rows past the half's last row are never stored.
// Every mbarrier wait is bounded.
constexpr int A2_QSLAB = 128 * 64;                 // 128 rows x 32 bf16 = 8 KB
constexpr int A2_KSLAB = 256 * 64;                 // 256 rows x 32 bf16 = 16 KB
constexpr int A2_Q_OFF = 0, A2_K_OFF = 5 * A2_QSLAB, A2_V_OFF = A2_K_OFF + 5 * A2_KSLAB;
constexpr int A2_RED_OFF = A2_V_OFF + 5 * A2_KSLAB;  // partial max and sum: [slice][row] floats
constexpr int A2_OST_OFF = A2_RED_OFF + AT_RED_BYTES;
constexpr int A2_BAR_OFF = A2_OST_OFF + 4 * AT_OSTAGE;
constexpr int A2_SMEM = 1024 + A2_BAR_OFF + 256;
constexpr uint32_t A2_SCOL = 0, A2_OCOL = 256;
static_assert(A2_SMEM <= 227 * 1024, "k_attention_tc256 shared memory");

__global__ void __launch_bounds__(AT_THREADS, 1)
    k_attention_tc256(const __grid_constant__ CUtensorMap tm, Segs segs, int64_t nitems, bf16 *__restrict__ att,
                      float scale, int *status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *red_max = reinterpret_cast<float *>(smem + A2_RED_OFF), *red_sum = red_max + 4 * 128;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + A2_BAR_OFF);
    uint64_t *qk_full = bars, *qk_empty = bars + 1, *v_full = bars + 2, *v_empty = bars + 3;
    uint64_t *s_full = bars + 4, *p_full = bars + 5, *o_full = bars + 6, *o_free = bars + 7, *pv_done = bars + 8;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 9);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(qk_full, 1);
        mbar_init(qk_empty, 1);
        mbar_init(v_full, 1);
        mbar_init(v_empty, 1);
        mbar_init(s_full, 1);
        mbar_init(p_full, AT_SOFT_WARPS);
        mbar_init(o_full, 1);
        mbar_init(o_free, 4);
        mbar_init(pv_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tensormap(&tm);
    }
    if (warp == 1) { tmem_alloc(tmem_holder, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = *tmem_holder;
    // Item it: launch segment it >> 3, head (it >> 1) & 3, query half it & 1.
    // Every role walks the items with 128 < T <= 256 in the same order; any
    // other length is skipped by all roles (a longer one is reported).
    auto item_at = [&](int64_t it, int64_t &t0, int &T, int &h, int &half) {
        const int64_t p = seg_pix(segs, it >> 3);
        h = (int)((it >> 1) & 3);
        half = (int)(it & 1);
        t0 = seg_at(segs, p);
        const int64_t len = seg_at(segs, p + 1) - t0;
        T = (len > 128 && len <= 256) ? (int)len : 0;
        if (len > 256 && warp == 0 && lane == 0 && status) atomicCAS(status, 0, ERR_BAD_SEGMENT);
    };
    auto next_item = [&](int64_t it, int64_t &t0, int &T, int &h, int &half) -> int64_t {
        for (; it < nitems; it += gridDim.x) {
            item_at(it, t0, T, h, half);
            if (T > 0) break;
        }
        return it;
    };

    if (warp == 0) {
        if (lane < 2) {  // lane 0 loads Q and K, lane 1 loads V
            int j = 0;
            int64_t t0;
            int T, h, half;
            for (int64_t it = next_item(blockIdx.x, t0, T, h, half); it < nitems;
                 it = next_item(it + gridDim.x, t0, T, h, half)) {
                const int nbk = (T + 31) >> 5;
                if (lane == 0) {
                    const int Tq = half ? T - 128 : 128, nbq = (Tq + 31) >> 5;
                    const int q0 = (int)t0 + half * 128;
                    if (!mbar_wait(qk_empty, (j & 1) ^ 1, abort_flag, status, ERR_WAIT_SMEM_EMPTY)) break;
                    mbar_arrive_expect_tx(qk_full, (uint32_t)((nbq + nbk) * 5 * 32 * 64));
                    for (int rb = 0; rb < nbq; ++rb)
                        for (int sl = 0; sl < 5; ++sl)
                            tma_load_2d(smem + A2_Q_OFF + sl * A2_QSLAB + rb * 2048, &tm, h * HD + sl * 32, q0 + rb * 32,
                                        qk_full);
                    for (int rb = 0; rb < nbk; ++rb)
                        for (int sl = 0; sl < 5; ++sl)
                            tma_load_2d(smem + A2_K_OFF + sl * A2_KSLAB + rb * 2048, &tm, D + h * HD + sl * 32,
                                        (int)t0 + rb * 32, qk_full);
                } else {
                    if (!mbar_wait(v_empty, (j & 1) ^ 1, abort_flag, status, ERR_WAIT_SMEM_EMPTY)) break;
                    mbar_arrive_expect_tx(v_full, (uint32_t)(nbk * 5 * 32 * 64));
                    for (int rb = 0; rb < nbk; ++rb)
                        for (int sl = 0; sl < 5; ++sl)
                            tma_load_2d(smem + A2_V_OFF + sl * A2_KSLAB + rb * 2048, &tm, 2 * D + h * HD + sl * 32,
                                        (int)t0 + rb * 32, v_full);
                }
                ++j;
            }
            // every stage released: no MMA still reads shared memory at exit
            mbar_wait(lane == 0 ? qk_empty : v_empty, (j & 1) ^ 1, abort_flag, status, ERR_WAIT_SMEM_EMPTY);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_o = umma_idesc_bf16_bmn(128, HD);
            const uint32_t sq = smem_u32(smem + A2_Q_OFF), sk = smem_u32(smem + A2_K_OFF),
                           sv = smem_u32(smem + A2_V_OFF);
            int j = 0;
            int64_t t0;
            int T, h, half;
            for (int64_t it = next_item(blockIdx.x, t0, T, h, half); it < nitems;
                 it = next_item(it + gridDim.x, t0, T, h, half)) {
                const int tpad = (T + 15) & ~15;
                // S(j): its columns hold P(j - 1) until O(j - 1) has read it
                if (!mbar_wait(qk_full, j & 1, abort_flag, status, ERR_WAIT_TMA_FULL)) break;
                if (j > 0 && !mbar_wait(pv_done, (j - 1) & 1, abort_flag, status, ERR_WAIT_TMEM_EMPTY)) break;
                tc_fence_after();
                const uint32_t idesc_s = umma_idesc_bf16(128, tpad);
#pragma unroll
                for (int k = 0; k < HD / 16; ++k) {
                    const uint32_t sl = (uint32_t)(k >> 1);
                    umma_bf16(tb + A2_SCOL, umma_desc_sw64(sq + sl * A2_QSLAB) + (uint64_t)(2 * (k & 1)),
                              umma_desc_sw64(sk + sl * A2_KSLAB) + (uint64_t)(2 * (k & 1)), idesc_s, k > 0);
                }
                umma_commit(s_full);
                umma_commit(qk_empty);
                // O(j) = P(j) V(j)
                if (!mbar_wait(v_full, j & 1, abort_flag, status, ERR_WAIT_TMA_FULL)) break;
                if (!mbar_wait(p_full, j & 1, abort_flag, status, ERR_WAIT_TMEM_FULL)) break;
                if (!mbar_wait(o_free, (j & 1) ^ 1, abort_flag, status, ERR_WAIT_TMEM_EMPTY)) break;
                tc_fence_after();
                for (int k = 0; k < tpad / 16; ++k)
                    umma_bf16_tmem_a(tb + A2_OCOL, tb + A2_SCOL + (uint32_t)(k * 8),
                                     umma_desc_sw64_mn(sv + (uint32_t)(k * 16 * 64), A2_KSLAB), idesc_o, k > 0);
                umma_commit(o_full);
                umma_commit(v_empty);
                umma_commit(pv_done);
                ++j;
            }
            // the last item's arrivals have landed before the CTA's shared memory is released
            if (j > 0) mbar_wait(pv_done, (j - 1) & 1, abort_flag, status, ERR_WAIT_TMEM_EMPTY);
        }
    } else if (warp < AT_IO_WARP0) {
        // softmax: quadrant = warp % 4 (the TMEM lanes this warp may access), 64-column slice
        const int quad = warp & 3, slice = (warp - 2) >> 2, r = quad * 32 + lane, c0 = slice * 64;
        const uint32_t lanebits = (uint32_t)(quad * 32) << 16;
        int j = 0;
        int64_t t0;
        int T, h, half;
        for (int64_t it = next_item(blockIdx.x, t0, T, h, half); it < nitems;
             it = next_item(it + gridDim.x, t0, T, h, half)) {
            const int tpad = (T + 15) & ~15;
            if (!mbar_wait(s_full, j & 1, abort_flag, status, ERR_WAIT_TMEM_FULL)) break;
            tc_fence_after();
            uint32_t v[4][16];  // 64 columns of the S row, then s, then e, as f32 bits
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (c0 + q * 16 < tpad) tmem_ld16(tb + lanebits + A2_SCOL + (uint32_t)(c0 + q * 16), v[q]);
            tmem_ld_wait();
            float mx = -INFINITY;
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (c0 + q * 16 < tpad) {
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int col = c0 + q * 16 + k;
                        const float x = col < T ? bf16_round(__uint_as_float(v[q][k]) * scale) : -INFINITY;
                        v[q][k] = __float_as_uint(x);
                        mx = fmaxf(mx, x);
                    }
                }
            red_max[slice * 128 + r] = mx;
            named_bar_sync(1 + quad, 128);
            mx = fmaxf(fmaxf(red_max[r], red_max[128 + r]), fmaxf(red_max[256 + r], red_max[384 + r]));
            float z = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (c0 + q * 16 < tpad) {
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const float ex = __expf(__uint_as_float(v[q][k]) - mx);  // 0 for masked columns
                        v[q][k] = __float_as_uint(ex);
                        z += ex;
                    }
                }
            red_sum[slice * 128 + r] = z;
            named_bar_sync(1 + quad, 128);
            z = ((red_sum[r] + red_sum[128 + r]) + red_sum[256 + r]) + red_sum[384 + r];
            const float inv = 1.f / z;
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (c0 + q * 16 < tpad) {
                    uint32_t w[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        w[k] = pack_bf16x2(__uint_as_float(v[q][2 * k]) * inv, __uint_as_float(v[q][2 * k + 1]) * inv);
                    tmem_st8(tb + lanebits + A2_SCOL + (uint32_t)(c0 / 2 + q * 8), w);
                }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
            ++j;
        }
    } else {
        // O warps: each drains its TMEM lane quadrant (32 query rows) of O(j)
        const int quad = warp & 3;
        const uint32_t lanebits = (uint32_t)(quad * 32) << 16;
        uint8_t *stage = smem + A2_OST_OFF + (warp - AT_IO_WARP0) * AT_OSTAGE;
        uint4 *my_row = reinterpret_cast<uint4 *>(stage + lane * 64);
        const int sw = (lane >> 1) & 3;
        int j = 0;
        int64_t t0;
        int T, h, half;
        for (int64_t it = next_item(blockIdx.x, t0, T, h, half); it < nitems;
             it = next_item(it + gridDim.x, t0, T, h, half)) {
            if (!mbar_wait(o_full, j & 1, abort_flag, status, ERR_WAIT_TMEM_FULL)) break;
            tc_fence_after();
            const int Tq = half ? T - 128 : 128;
            const int nrows = Tq - quad * 32;  // real rows of this quadrant (uniform per warp)
            if (nrows > 0) {
                bf16 *dst = att + (t0 + half * 128 + quad * 32) * D + h * HD;
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                    uint32_t v[16], w[16];
                    tmem_ld16(tb + lanebits + A2_OCOL + (uint32_t)(c * 32), v);
                    tmem_ld16(tb + lanebits + A2_OCOL + (uint32_t)(c * 32 + 16), w);
                    tmem_ld_wait();
                    uint32_t o[16];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        o[k] = pack_bf16x2(__uint_as_float(v[2 * k]), __uint_as_float(v[2 * k + 1]));
                        o[8 + k] = pack_bf16x2(__uint_as_float(w[2 * k]), __uint_as_float(w[2 * k + 1]));
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k) my_row[k ^ sw] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int rr = i * 8 + (lane >> 2), k = lane & 3;
                        const uint4 val = reinterpret_cast<const uint4 *>(stage + rr * 64)[k ^ ((rr >> 1) & 3)];
                        if (rr < nrows) *reinterpret_cast<uint4 *>(dst + (int64_t)rr * D + c * 32 + k * 8) = val;
                    }
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);
            ++j;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tb, 512);
}

// ------------------------------------------------------------------ LayerNorm
// Warp per row of 640, two-pass f32 statistics.

// With pool_q set (the last layer's LN2), each row's attention-pooling logit
// s = sum_k y[k] q[k] + qb of the bf16 output row is also written to
// logits[row], summed in exactly the order k_pool sums it (per lane over its
// five 4-column groups, then the warp), so the pooling kernel reads x once.
template <bool LOGITS>
__global__ void __launch_bounds__(256) k_layernorm640(const bf16 *__restrict__ x, int64_t M, const float *__restrict__ g,
                                                      const float *__restrict__ b, bf16 *__restrict__ y,
                                                      const float *__restrict__ pool_q, float pool_qb,
                                                      float *__restrict__ logits) {
    // Grid-stride over rows, one warp per row: lane l holds columns
    // 128j + 4l .. 128j + 4l + 3 (j = 0..4) packed as bf16, so each 8-byte
    // load instruction of the warp reads 256 contiguous bytes. The next row is
    // loaded before the current one is reduced, which keeps two rows (2.5 KB)
    // of loads in flight per warp at a low register count. gamma/beta are read
    // once per block into shared memory.
    __shared__ __align__(16) float gs[D], bs[D], qs[LOGITS ? D : 4];
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        gs[i] = g ? g[i] : 1.f;
        bs[i] = b ? b[i] : 0.f;
        if constexpr (LOGITS) qs[i] = pool_q[i];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t stride = (int64_t)gridDim.x * (blockDim.x >> 5);
    auto load = [&](int64_t r, uint2 (&q)[5]) {
        const bf16 *xr = x + r * D + lane * 4;
#pragma unroll
        for (int j = 0; j < 5; ++j) q[j] = *reinterpret_cast<const uint2 *>(xr + j * 128);
    };
    int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    uint2 q[5], qn[5];
    if (r < M) load(r, q);
    for (; r < M; r += stride) {
        if (r + stride < M) load(r + stride, qn);
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            s += bf16lo(q[j].x); s += bf16hi(q[j].x);
            s += bf16lo(q[j].y); s += bf16hi(q[j].y);
        }
        const float mean = warp_sum(s) / (float)D;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            const float d0 = bf16lo(q[j].x) - mean, d1 = bf16hi(q[j].x) - mean;
            const float d2 = bf16lo(q[j].y) - mean, d3 = bf16hi(q[j].y) - mean;
            ss += d0 * d0; ss += d1 * d1; ss += d2 * d2; ss += d3 * d3;
        }
        const float rstd = 1.f / sqrtf(warp_sum(ss) / (float)D + LN_EPS);
        bf16 *yr = y + r * D + lane * 4;
        float dq = 0.f;
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            const int c = j * 128 + lane * 4;
            const float4 gg = *reinterpret_cast<const float4 *>(gs + c), bb = *reinterpret_cast<const float4 *>(bs + c);
            const uint32_t o0 = pack_bf16x2((bf16lo(q[j].x) - mean) * rstd * gg.x + bb.x,
                                            (bf16hi(q[j].x) - mean) * rstd * gg.y + bb.y);
            const uint32_t o1 = pack_bf16x2((bf16lo(q[j].y) - mean) * rstd * gg.z + bb.z,
                                            (bf16hi(q[j].y) - mean) * rstd * gg.w + bb.w);
            *reinterpret_cast<uint2 *>(yr + j * 128) = make_uint2(o0, o1);
            if constexpr (LOGITS)
                dq += bf16lo(o0) * qs[c] + bf16hi(o0) * qs[c + 1] + bf16lo(o1) * qs[c + 2] + bf16hi(o1) * qs[c + 3];
        }
        if constexpr (LOGITS) {
            dq = warp_sum(dq);
            if (lane == 0) logits[r] = dq + pool_qb;
        }
#pragma unroll
        for (int j = 0; j < 5; ++j) q[j] = qn[j];
    }
}

// ------------------------------------------------------------------ pooling
// One CTA (160 threads) per pixel: warp-per-step logits, softmax in warp 0,
// then each thread accumulates 4 columns over the steps. When the last
// LayerNorm already wrote the logits (logits != null), x is read once.
__global__ void __launch_bounds__(160) k_pool(const bf16 *__restrict__ x, Segs segs, const float *__restrict__ q,
                                              float qb, bf16 *__restrict__ fused, int col0,
                                              const float *__restrict__ logits) {
    __shared__ float w[256];
    const int64_t i = blockIdx.x;
    const int64_t t0 = seg_at(segs, i);
    const int T = (int)(seg_at(segs, i + 1) - t0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    bf16 *fo = fused + i * (2 * D) + col0;
    if (T <= 0) {  // pixel with no observation at all: zero row (never reaches the output)
        *reinterpret_cast<uint2 *>(fo + threadIdx.x * 4) = make_uint2(0u, 0u);
        return;
    }
    const bf16 *xp = x + t0 * D;
    if (logits) {
        for (int t = threadIdx.x; t < T; t += blockDim.x) w[t] = logits[t0 + t];
    } else for (int t = warp; t < T; t += 5) {
        float d = 0.f;
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            const int c = j * 128 + lane * 4;
            const uint2 v = *reinterpret_cast<const uint2 *>(xp + (int64_t)t * D + c);
            d += bf16lo(v.x) * q[c] + bf16hi(v.x) * q[c + 1] + bf16lo(v.y) * q[c + 2] + bf16hi(v.y) * q[c + 3];
        }
        d = warp_sum(d);
        if (lane == 0) w[t] = d + qb;
    }
    __syncthreads();
    if (warp == 0) {
        float mx = -INFINITY;
        for (int t = lane; t < T; t += 32) mx = fmaxf(mx, w[t]);
        mx = warp_max(mx);
        float z = 0.f;
        for (int t = lane; t < T; t += 32) { const float e = expf(w[t] - mx); w[t] = e; z += e; }
        z = warp_sum(z);
        __syncwarp();
        for (int t = lane; t < T; t += 32) w[t] = w[t] / z;  // the weights, each divided once
    }
    __syncthreads();
    // p = sum_t w_t x_t in t order; four steps' loads are issued ahead of their FMAs
    const int c = threadIdx.x * 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    auto add = [&](float wt, uint2 v) {
        acc[0] += wt * bf16lo(v.x); acc[1] += wt * bf16hi(v.x); acc[2] += wt * bf16lo(v.y); acc[3] += wt * bf16hi(v.y);
    };
    int t = 0;
    for (; t + 4 <= T; t += 4) {
        uint2 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const uint2 *>(xp + (int64_t)(t + u) * D + c);
#pragma unroll
        for (int u = 0; u < 4; ++u) add(w[t + u], v[u]);
    }
    for (; t < T; ++t) add(w[t], *reinterpret_cast<const uint2 *>(xp + (int64_t)t * D + c));
    *reinterpret_cast<uint2 *>(fo + c) = make_uint2(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]));
}

// ------------------------------------------------------------------ head
// Warp per row of 2560: LN with affine, rounded to bf16, then ReLU on the bf16 value.
__global__ void __launch_bounds__(256) k_ln_relu2560(bf16 *__restrict__ r, int64_t P, const float *__restrict__ g,
                                                     const float *__restrict__ b) {
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= P) return;
    bf16 *xr = r + row * RED;
    float v[80];
#pragma unroll
    for (int j = 0; j < 20; ++j) {
        const uint2 q = *reinterpret_cast<const uint2 *>(xr + j * 128 + lane * 4);
        v[4 * j] = bf16lo(q.x); v[4 * j + 1] = bf16hi(q.x); v[4 * j + 2] = bf16lo(q.y); v[4 * j + 3] = bf16hi(q.y);
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 80; ++j) s += v[j];
    const float mean = warp_sum(s) / (float)RED;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < 80; ++j) { const float d = v[j] - mean; q += d * d; }
    const float rstd = 1.f / sqrtf(warp_sum(q) / (float)RED + LN_EPS);
#pragma unroll
    for (int j = 0; j < 20; ++j) {
        const int c = j * 128 + lane * 4;
        uint32_t w2[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const float o0 = (v[4 * j + 2 * k] - mean) * rstd * g[c + 2 * k] + b[c + 2 * k];
            const float o1 = (v[4 * j + 2 * k + 1] - mean) * rstd * g[c + 2 * k + 1] + b[c + 2 * k + 1];
            uint32_t u = pack_bf16x2(o0, o1);
            if (u & 0x8000u) u &= 0xFFFF0000u;      // relu on the bf16 sign bit (tessera_cpu.cpp:570-571)
            if (u & 0x80000000u) u &= 0x0000FFFFu;
            w2[k] = u;
        }
        *reinterpret_cast<uint2 *>(xr + c) = make_uint2(w2[0], w2[1]);
    }
}

// Warp per pixel: LN(128, no affine) -> bf16 -> f32 output or int8 quantisation.
__global__ void __launch_bounds__(256) k_out128(const bf16 *__restrict__ r2, int64_t P, const uint8_t *__restrict__ empty,
                                                float *__restrict__ out, int8_t *__restrict__ codes,
                                                float *__restrict__ scales) {
    const int64_t p = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (p >= P) return;
    const uint2 q = *reinterpret_cast<const uint2 *>(r2 + p * OUT + lane * 4);
    float v[4] = {bf16lo(q.x), bf16hi(q.x), bf16lo(q.y), bf16hi(q.y)};
    const float mean = warp_sum(v[0] + v[1] + v[2] + v[3]) / (float)OUT;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) { const float d = v[k] - mean; s += d * d; }
    const float rstd = 1.f / sqrtf(warp_sum(s) / (float)OUT + LN_EPS);
    const bool is_empty = empty && empty[p];
    float e[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) e[k] = is_empty ? 0.f : bf16_round((v[k] - mean) * rstd);
    if (out) {
        *reinterpret_cast<float4 *>(out + p * OUT + lane * 4) = make_float4(e[0], e[1], e[2], e[3]);
        return;
    }
    float am = fmaxf(fmaxf(fabsf(e[0]), fabsf(e[1])), fmaxf(fabsf(e[2]), fabsf(e[3])));
    am = fmaxf(warp_max(am), 1e-12f);
    const float sc = am / 127.0f;
    uint32_t packed = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float c = rintf(e[k] / sc);
        c = fminf(127.f, fmaxf(-127.f, c));
        packed |= (uint32_t)(uint8_t)(int8_t)(int)c << (8 * k);
    }
    *reinterpret_cast<uint32_t *>(codes + p * OUT + lane * 4) = packed;
    if (lane == 0) scales[p] = sc;
}

// ------------------------------------------------------------------ wait probe
// Waits on an mbarrier that nothing ever arrives on, with a caller-given limit:
// the bounded-wait path every pipeline kernel relies on. It must end with
// status ERR_WAIT_PROBE and a usable context, never a trap or a hang.
__global__ void k_wait_probe(uint64_t limit_ns, int *status) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, status, ERR_WAIT_PROBE, limit_ns);
}

void launch_wait_probe(uint64_t limit_ns, int *status, cudaStream_t st) {
    k_wait_probe<<<1, 32, 0, st>>>(limit_ns, status);
    check_launch("k_wait_probe");
}

// ------------------------------------------------------------------ launchers
static unsigned blocks_for(int64_t n, int per_block) { return (unsigned)((n + per_block - 1) / per_block); }

void launch_count(const TileDev &t, int64_t p0, int64_t np, int32_t *n2, int32_t *n1, cudaStream_t st) {
    if (np <= 0) return;
    k_count<<<blocks_for(np, 256), 256, 0, st>>>(t, p0, np, n2, n1);
    check_launch("k_count");
}

void launch_gather(int modality, const TileDev &t, int64_t p0, int64_t np, const int32_t * /*nvalid*/,
                   const int32_t *bins, Segs segs, float *rec, cudaStream_t st) {
    if (np <= 0) return;
    const int64_t steps = modality == 0 ? t.T2 : t.Ta + t.Td;
    if (steps > MAX_STEPS) throw std::runtime_error("gather: series longer than " + std::to_string(MAX_STEPS));
    if (modality == 0) k_gather<0><<<blocks_for(np, 4), 128, 0, st>>>(t, p0, np, bins, segs, rec);
    else k_gather<1><<<blocks_for(np, 4), 128, 0, st>>>(t, p0, np, bins, segs, rec);
    check_launch("k_gather");
}

void launch_emb1(int C, const float *rec, int64_t M, const float *w1t, const float *b1, bf16 *y, cudaStream_t st) {
    if (M <= 0) return;
    const unsigned grid = (unsigned)std::min<int64_t>(blocks_for(M, 16), 148 * 8);
    if (C == 10) k_emb1<10><<<grid, 256, 0, st>>>(rec, M, w1t, b1, y);
    else if (C == 2) k_emb1<2><<<grid, 256, 0, st>>>(rec, M, w1t, b1, y);
    else throw std::runtime_error("emb1: unsupported band count");
    check_launch("k_emb1");
}

template <int NT> static void attention_nt(const bf16 *qkv, Segs segs, int64_t npix, int Tpad, bf16 *att,
                                          cudaStream_t st) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        cudaFuncSetAttribute(k_attention<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 8 * NT * ATT_LD * 2);
        attr[dev & 63] = true;
    }
    const size_t smem = (size_t)2 * Tpad * ATT_LD * sizeof(bf16);
    // Past 128 keys one CTA fills an SM's shared memory. Up to 192 keys it runs
    // 16 warps, one per 16-row query block (T = 160: 440 against 517 us per
    // 131k-token chunk with 8 warps); at 256 keys the 128-register cap of 16
    // warps spills, so 8 warps stay.
    const int warps = std::min(NT == 24 ? 16 : 8, Tpad / 16);
    const dim3 grid((unsigned)npix, NH);
    k_attention<NT><<<grid, 32 * warps, smem, st>>>(qkv, segs, att, 1.f / std::sqrt((float)HD));
}

// TC_ATTN_TC: 0 = always the mma.sync kernel; 1 (default) = the tcgen05 kernels
// for a series longer than AT_MMA_MAX_T (k_attention_tc up to 128 steps,
// k_attention_tc256 above); 2 = the tcgen05 kernels for every length.
static int attention_tcgen05() {
    static const int mode = [] {
        const char *e = std::getenv("TC_ATTN_TC");
        return e && (*e == '0' || *e == '2') ? *e - '0' : 1;
    }();
    return mode;
}

// Longest series left to the mma.sync kernel when both kernels are on. Timed
// on B200 over 131,072-token chunks of uniform T (us per chunk, mma.sync /
// tcgen05): T = 32: 156 / 243, T = 48: 169 / 195, T = 64: 183 / 165, T = 96:
// 244 / 144, T = 128: 272 / 131. Bins are multiples of 8, so 48 is the last
// length where mma.sync is faster.
constexpr int AT_MMA_MAX_T = 48;

static void attention_tc(const bf16 *qkv, Segs segs, int64_t npix, int64_t ntok, bf16 *att, int *status,
                         cudaStream_t st) {
    static int grid_per_dev[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!grid_per_dev[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
        if (e != cudaSuccess) throw std::runtime_error(std::string("attention smem attribute: ") + cudaGetErrorString(e));
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        grid_per_dev[dev & 63] = std::max(1, sms);
    }
    // qkv rows [0, ntok) x 1920 columns; boxes of 32 rows x 64 columns, 128-byte swizzle
    CUtensorMap tm;
    make_tmap_box(&tm, qkv, (uint64_t)ntok, (uint64_t)(3 * D), (uint64_t)(3 * D), 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    const int64_t items = npix * NH;
    const unsigned grid = (unsigned)std::min<int64_t>(items, grid_per_dev[dev & 63]);
    k_attention_tc<<<grid, AT_THREADS, AT_SMEM, st>>>(tm, segs, items, att, 1.f / std::sqrt((float)HD), status);
}

static void attention_tc256(const bf16 *qkv, Segs segs, int64_t npix, int64_t ntok, bf16 *att, int *status,
                            cudaStream_t st) {
    static int grid_per_dev[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!grid_per_dev[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_tc256, cudaFuncAttributeMaxDynamicSharedMemorySize, A2_SMEM);
        if (e != cudaSuccess) throw std::runtime_error(std::string("attention smem attribute: ") + cudaGetErrorString(e));
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        grid_per_dev[dev & 63] = std::max(1, sms);
    }
    // qkv rows [0, ntok) x 1920 columns; boxes of 32 rows x 32 columns, 64-byte swizzle
    CUtensorMap tm;
    make_tmap_box(&tm, qkv, (uint64_t)ntok, (uint64_t)(3 * D), (uint64_t)(3 * D), 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    const int64_t items = npix * NH * 2;
    const unsigned grid = (unsigned)std::min<int64_t>(items, grid_per_dev[dev & 63]);
    k_attention_tc256<<<grid, AT_THREADS, A2_SMEM, st>>>(tm, segs, items, att, 1.f / std::sqrt((float)HD), status);
}

int attention_class(int T) {
    if (T > 128) return 2;
    const int mode = attention_tcgen05();
    return mode == 2 || (mode == 1 && T > AT_MMA_MAX_T) ? 1 : 0;
}

void attention_plan(const int64_t *off, int64_t npix, int32_t *list, AttnPlan &plan) {
    plan = AttnPlan{};
    for (int64_t i = 0; i < npix; ++i) {
        const int64_t T = off[i + 1] - off[i];
        if (T <= 0) continue;
        const int c = attention_class((int)std::min<int64_t>(T, 1 << 30));
        ++plan.n[c];
        plan.tmax[c] = (int)std::max<int64_t>(plan.tmax[c], T);
    }
    int64_t pos[3] = {0, plan.n[0], plan.n[0] + plan.n[1]};
    for (int64_t i = 0; i < npix; ++i) {
        const int64_t T = off[i + 1] - off[i];
        if (T > 0) list[pos[attention_class((int)std::min<int64_t>(T, 1 << 30))]++] = (int32_t)i;
    }
}

// npix segments of one class (through segs.pix when set), the longest tmax.
static void attention_of_class(int cls, const bf16 *qkv, Segs segs, int64_t npix, int64_t ntok, int tmax, bf16 *att,
                               int *status, cudaStream_t st) {
    if (npix <= 0 || tmax <= 0) return;
    if (tmax > 256) throw std::runtime_error("attention: T > 256");
    const int Tpad = (tmax + 15) & ~15;
    if (cls == 1) {
        attention_tc(qkv, segs, npix, ntok, att, status, st);
    } else if (cls == 2 && attention_tcgen05() != 0) {
        attention_tc256(qkv, segs, npix, ntok, att, status, st);
    } else {
        if (Tpad <= 32) attention_nt<4>(qkv, segs, npix, Tpad, att, st);
        else if (Tpad <= 64) attention_nt<8>(qkv, segs, npix, Tpad, att, st);
        else if (Tpad <= 96) attention_nt<12>(qkv, segs, npix, Tpad, att, st);
        else if (Tpad <= 128) attention_nt<16>(qkv, segs, npix, Tpad, att, st);
        else if (Tpad <= 192) attention_nt<24>(qkv, segs, npix, Tpad, att, st);
        else attention_nt<32>(qkv, segs, npix, Tpad, att, st);
    }
}

int launch_attention_plan(const bf16 *qkv, Segs segs, const AttnPlan &plan, int64_t ntok, bf16 *att, int *status,
                          cudaStream_t st) {
    int64_t o = 0;
    int launched = 0;
    for (int c = 0; c < 3; ++c) {
        Segs s = segs;
        s.pix = plan.pix + o;
        if (plan.n[c] > 0 && plan.tmax[c] > 0) {
            attention_of_class(c, qkv, s, plan.n[c], ntok, plan.tmax[c], att, status, st);
            ++launched;
        }
        o += plan.n[c];
    }
    check_launch("k_attention");
    return launched;
}

int launch_attention(const bf16 *qkv, Segs segs, int64_t npix, int64_t ntok, int Tmax, bf16 *att, int *status,
                     cudaStream_t st) {
    if (npix <= 0 || Tmax <= 0) return 0;
    attention_of_class(attention_class(Tmax), qkv, segs, npix, ntok, Tmax, att, status, st);
    check_launch("k_attention");
    return 1;
}

void launch_layernorm640(const bf16 *x, int64_t M, const float *g, const float *b, bf16 *y, cudaStream_t st,
                         const float *pool_q, float pool_qb, float *logits) {
    if (M <= 0) return;
    // grid-stride: as many blocks as fit on the device at once
    static int resident[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!resident[dev & 63]) {
        int per_sm = 0, sms = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_layernorm640<false>, 256, 0);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        resident[dev & 63] = std::max(1, per_sm) * std::max(1, sms);
    }
    const unsigned grid = (unsigned)std::min<int64_t>(blocks_for(M, 8), resident[dev & 63]);
    if (pool_q) k_layernorm640<true><<<grid, 256, 0, st>>>(x, M, g, b, y, pool_q, pool_qb, logits);
    else k_layernorm640<false><<<grid, 256, 0, st>>>(x, M, g, b, y, nullptr, 0.f, nullptr);
    check_launch("k_layernorm640");
}

void launch_pool(const bf16 *x, Segs segs, int64_t npix, const float *q, float qb, bf16 *fused, int col0,
                 cudaStream_t st, const float *logits) {
    if (npix <= 0) return;
    k_pool<<<(unsigned)npix, 160, 0, st>>>(x, segs, q, qb, fused, col0, logits);
    check_launch("k_pool");
}

void launch_ln_relu2560(bf16 *r, int64_t P, const float *g, const float *b, cudaStream_t st) {
    if (P <= 0) return;
    k_ln_relu2560<<<blocks_for(P, 8), 256, 0, st>>>(r, P, g, b);
    check_launch("k_ln_relu2560");
}

void launch_out128(const bf16 *r2, int64_t P, const uint8_t *empty, float *out, int8_t *codes, float *scales,
                   cudaStream_t st) {
    if (P <= 0) return;
    k_out128<<<blocks_for(P, 8), 256, 0, st>>>(r2, P, empty, out, codes, scales);
    check_launch("k_out128");
}

}  // namespace tcb
