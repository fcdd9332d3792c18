// Dense layers of the pixel student on the sm_100a tensor cores.
//
//   out[M, N] (bf16) = round_bf16( [relu]( A[M, K] . W[N, K]^T + bias[N] ) [+ residual[M, N]] )
//
// A is a token-major activation matrix, W a torch-layout (out x in) weight
// matrix; both are bf16 and K-contiguous. This is the rounding contract of the
// reference's oneDNN matmul with bias + [relu] + [binary add] post-ops
// (tessera_cpu.cpp:215-243): f32 accumulation, f32 bias, residual added in f32,
// one round-to-nearest-even to bf16 at the end.
//
// Kernel shape: persistent, one CTA per SM, warp-specialised.
//   warp 0      TMA producer: A and W tiles (128-byte swizzle) into a ring of
//               shared-memory stages, completion tracked by mbarriers.
//   warp 1      TMEM allocator and MMA issuer: one elected thread issues
//               tcgen05.mma (M=128, N=BN, K=16; the last column tile may be
//               narrower) into a double-buffered f32 accumulator in tensor
//               memory and commits stage/tile barriers.
//   warps 2-9   epilogue: tcgen05.ld of the accumulator (two warps per TMEM
//               lane quadrant, splitting the columns; one output row per
//               lane), bias, ReLU, residual, bf16 rounding, then a swizzled
//               shared-memory staging buffer and row-contiguous global stores.
// The double-buffered accumulator lets the epilogue of tile i overlap the
// main loop of tile i+1.
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm_sm100.h"

namespace tcb {

constexpr int BM = 128;           // UMMA M (cta_group::1)
constexpr int BK = 64;            // one 128-byte swizzle atom of bf16 along K
constexpr int UMMA_K = 16;        // K per tcgen05.mma for 16-bit inputs
constexpr int GEMM_THREADS = 320; // 10 warps: producer, MMA, 8 epilogue
constexpr int EPI_WARPS = 8;      // two per TMEM lane quadrant, splitting the tile's columns
constexpr int STAGING_BYTES = EPI_WARPS * 32 * 64;  // per epilogue warp: 32 rows x 32 bf16
constexpr int SMEM_BUDGET = 225 * 1024;
constexpr int RES_BOX = 128;      // residual L2-prefetch box: 128 columns x BM rows
// The bias vector, copied to shared memory once per CTA by the epilogue warps
// (N <= BIAS_MAX; wider layers read it from global memory). Read per column
// group from global memory, the bias loads sat on the epilogue's critical
// path and made it, not the MMA, the limit of the K = 640 layers.
constexpr int BIAS_MAX = 2560;
constexpr int BIAS_BYTES = BIAS_MAX * 4;
constexpr int BARRIER_BYTES = 256;

template <int BN> struct GemmCfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES_RAW = (SMEM_BUDGET - 2048 - STAGING_BYTES - BIAS_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    // align slack, stages, staging, barriers, bias
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + STAGING_BYTES + BARRIER_BYTES + BIAS_BYTES;
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 must be a multiple of 16 in [16,256]");
    static_assert(B_BYTES % 1024 == 0, "B stage must keep 1024-byte alignment for the 128B swizzle");
    static_assert(STAGES >= 2, "need at least two pipeline stages");
};

__device__ __forceinline__ float pe_value(float doy, int n, const bf16 *__restrict__ table,
                                          const float *__restrict__ div, bool tab, int di) {
    if (tab) return __bfloat162float(table[di * D + n]);
    const float a = doy * div[n >> 1];
    return bf16_round((n & 1) ? cosf(a) : sinf(a));
}

// bias, [relu], residual or DOY sinusoid and bf16 rounding of 16 accumulator
// columns of one output row, packed into two 16-byte words.
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// The epilogue warps' copy of the bias into shared memory (bias_sa: its
// shared address), then a barrier among those 8 warps only. Returns the
// address, or 0 when the bias is read from global memory.
__device__ __forceinline__ uint32_t stage_bias(const GemmArgs &p, uint8_t *bias_smem) {
    if (!p.bias || p.N > BIAS_MAX) return 0u;
    float *sb = reinterpret_cast<float *>(bias_smem);
    for (int i = threadIdx.x - 64; i < p.N; i += EPI_WARPS * 32) sb[i] = __ldg(p.bias + i);
    asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
    return smem_u32(sb);
}

__device__ __forceinline__ void epilogue_cols16(const GemmArgs &p, const uint32_t (&r)[16], const uint4 (&res)[2],
                                                bool has_res, float pe_doy, bool pe_tab, int pe_di, int n,
                                                uint4 (&o)[2], bool pe_irregular, uint32_t bias_sa) {
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
    if (bias_sa) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 b = lds_f4(bias_sa + (uint32_t)(n + 4 * j) * 4u);
            v[4 * j] += b.x; v[4 * j + 1] += b.y; v[4 * j + 2] += b.z; v[4 * j + 3] += b.w;
        }
    } else if (p.bias) {
        const float4 *b4 = reinterpret_cast<const float4 *>(p.bias + n);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 b = __ldg(b4 + j);
            v[4 * j] += b.x; v[4 * j + 1] += b.y; v[4 * j + 2] += b.z; v[4 * j + 3] += b.w;
        }
    }
    if (p.relu) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = fmaxf(v[j], 0.f);
    }
    if (has_res) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t w[4] = {res[h].x, res[h].y, res[h].z, res[h].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[8 * h + 2 * j] += bf16lo(w[j]);
                v[8 * h + 2 * j + 1] += bf16hi(w[j]);
            }
        }
    } else if (pe_irregular) {  // a day of year outside the table: sinusoid computed per element
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += pe_value(pe_doy, n + j, p.pe_table, p.pe_div, pe_tab, pe_di);
    }
    o[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                      pack_bf16x2(v[6], v[7]));
    o[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                      pack_bf16x2(v[14], v[15]));
}

// Lane `src`'s pointer, for every lane of the warp.
__device__ __forceinline__ const bf16 *shfl_ptr(const bf16 *ptr, int src) {
    const unsigned long long v = reinterpret_cast<unsigned long long>(ptr);
    return reinterpret_cast<const bf16 *>(__shfl_sync(0xFFFFFFFFu, v, src));
}

// The residual of a 32-column group (two = true) or a 16-column one, in the
// coalesced pattern: 32 columns are rows i * 8 + lane / 4 (i < 4, pointers
// r0..r3), 16 bytes at lane % 4; 16 columns are rows i * 16 + lane / 2 (i < 2),
// 16 bytes at lane % 2. A null row pointer gives zeros.
__device__ __forceinline__ void res_load_group(const bf16 *res_row, const bf16 *r0, const bf16 *r1,
                                               const bf16 *r2, const bf16 *r3, int n0, int c, bool two, int lane,
                                               uint4 &g0, uint4 &g1, uint4 &g2, uint4 &g3) {
    const uint4 zero = make_uint4(0, 0, 0, 0);
    if (two) {
        const int k = lane & 3;
        g0 = r0 ? reinterpret_cast<const uint4 *>(r0 + n0 + c)[k] : zero;
        g1 = r1 ? reinterpret_cast<const uint4 *>(r1 + n0 + c)[k] : zero;
        g2 = r2 ? reinterpret_cast<const uint4 *>(r2 + n0 + c)[k] : zero;
        g3 = r3 ? reinterpret_cast<const uint4 *>(r3 + n0 + c)[k] : zero;
    } else {
        const int k = lane & 1;
        const bf16 *h0 = shfl_ptr(res_row, lane >> 1), *h1 = shfl_ptr(res_row, 16 + (lane >> 1));
        g0 = h0 ? reinterpret_cast<const uint4 *>(h0 + n0 + c)[k] : zero;
        g1 = h1 ? reinterpret_cast<const uint4 *>(h1 + n0 + c)[k] : zero;
    }
}
// Write a group loaded by res_load_group into the staging rows (same swizzle
// as the output staging: chunk k of row rr at position k ^ ((rr >> 1) & 3)).
__device__ __forceinline__ void res_stage_group(uint8_t *stage, bool two, int lane, const uint4 &g0, const uint4 &g1,
                                                const uint4 &g2, const uint4 &g3) {
    if (two) {
        const int k = lane & 3, r = lane >> 2;
        reinterpret_cast<uint4 *>(stage + r * 64)[k ^ ((r >> 1) & 3)] = g0;
        reinterpret_cast<uint4 *>(stage + (r + 8) * 64)[k ^ (((r + 8) >> 1) & 3)] = g1;
        reinterpret_cast<uint4 *>(stage + (r + 16) * 64)[k ^ (((r + 16) >> 1) & 3)] = g2;
        reinterpret_cast<uint4 *>(stage + (r + 24) * 64)[k ^ (((r + 24) >> 1) & 3)] = g3;
    } else {
        const int k = lane & 1, r = lane >> 1;
        reinterpret_cast<uint4 *>(stage + r * 64)[k ^ ((r >> 1) & 3)] = g0;
        reinterpret_cast<uint4 *>(stage + (r + 16) * 64)[k ^ (((r + 16) >> 1) & 3)] = g1;
    }
}

// One epilogue warp: output rows row_base .. row_base + 31 (its TMEM lane
// quadrant, one row per lane) and accumulator columns [c0, c1) of a tile whose
// first output column is n0. Per group of 32 columns: TMEM -> registers ->
// epilogue math -> a 2 KB staging buffer (32 rows x 64 B, 16-byte chunks XOR-
// swizzled by (row >> 1) & 3, which is the TMA 64-byte swizzle) -> one bulk
// tensor store of the 32 x 32 block (tmO), issued by lane 0. Issued by the
// warp as 8-row x 64-byte global stores instead, the output cost about a
// fifth of the FFN1 launch's time; the bulk store takes it off the warps.
// A 16-column group (a tile width that is not a multiple of 32) is stored by
// the warp, 16 rows x 32 bytes per instruction.
// The residual (or, for an integer day of year, the DOY-table row, which is
// an ordinary residual row) takes the same way in reverse: loaded 8 rows x 64
// contiguous bytes per instruction (the row pointers passed between lanes by
// shuffle), written into the staging buffer and read back one row per lane.
// Its loads run one group ahead, the first group's before the wait for the
// accumulator.
// Returns false if the wait for the accumulator gave up.
__device__ __forceinline__ bool epilogue_tile(const GemmArgs &p, uint32_t tbase, int row_base, int n0, int c0, int c1,
                                              uint8_t *stage, int lane, uint64_t *tfull_bar, uint32_t parity,
                                              volatile int *abort_flag, uint32_t bias_sa, const CUtensorMap *tmO) {
    const int row = row_base + lane;
    const bool live = row < p.M;
    const bf16 *res_row = nullptr;
    bool pe_irregular = false;
    float pe_doy = 0.f;
    if (live) {
        if (p.res) {
            res_row = p.res + (size_t)row * p.ldr;
        } else if (p.pe_doy) {
            pe_doy = p.pe_doy[(size_t)row * p.pe_stride];
            if (pe_doy >= 0.f && pe_doy <= 366.f && floorf(pe_doy) == pe_doy) res_row = p.pe_table + (int)pe_doy * D;
            else pe_irregular = true;
        }
    }
    const bool any_res = p.res != nullptr || p.pe_doy != nullptr;  // uniform
    // residual rows of the coalesced pattern: row i * 8 + lane / 4, 16 bytes at lane % 4
    const bf16 *rp0 = nullptr, *rp1 = nullptr, *rp2 = nullptr, *rp3 = nullptr;
    if (any_res) {
        rp0 = shfl_ptr(res_row, (lane >> 2));
        rp1 = shfl_ptr(res_row, 8 + (lane >> 2));
        rp2 = shfl_ptr(res_row, 16 + (lane >> 2));
        rp3 = shfl_ptr(res_row, 24 + (lane >> 2));
    }
    uint4 *my_row = reinterpret_cast<uint4 *>(stage + lane * 64);
    const int sw = (lane >> 1) & 3;
    uint4 g0 = make_uint4(0, 0, 0, 0), g1 = g0, g2 = g0, g3 = g0;
    if (any_res) res_load_group(res_row, rp0, rp1, rp2, rp3, n0, c0, c0 + 32 <= c1, lane, g0, g1, g2, g3);
    if (!mbar_wait(tfull_bar, parity, abort_flag, p.status, ERR_WAIT_TMEM_FULL)) return false;
    tc_fence_after();
#pragma unroll 1
    for (int c = c0; c < c1; c += 32) {
        const bool two = c + 32 <= c1;
        uint4 q[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        if (any_res) {
            // the staging buffer is free once the previous group's bulk store has read it
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
            // the group's residual, from the coalesced layout to one row per lane
            res_stage_group(stage, two, lane, g0, g1, g2, g3);
            __syncwarp();
            q[0] = my_row[0 ^ sw];
            q[1] = my_row[1 ^ sw];
            if (two) {
                q[2] = my_row[2 ^ sw];
                q[3] = my_row[3 ^ sw];
            }
            __syncwarp();
            if (c + 32 < c1)
                res_load_group(res_row, rp0, rp1, rp2, rp3, n0, c + 32, c + 64 <= c1, lane, g0, g1, g2, g3);
        }
        const uint4 q0[2] = {q[0], q[1]}, q1[2] = {q[2], q[3]};
        uint32_t r0[16], r1[16];
        tmem_ld16(tbase + (uint32_t)c, r0);
        if (two) tmem_ld16(tbase + (uint32_t)(c + 16), r1);
        tmem_ld_wait();
        uint4 o[2], o1[2];
        epilogue_cols16(p, r0, q0, res_row != nullptr, pe_doy, false, 0, n0 + c, o, pe_irregular, bias_sa);
        if (two)
            epilogue_cols16(p, r1, q1, res_row != nullptr, pe_doy, false, 0, n0 + c + 16, o1, pe_irregular, bias_sa);
        if (!any_res) {  // the staging buffer is free once the previous group's bulk store has read it
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
        }
        my_row[0 ^ sw] = o[0];
        my_row[1 ^ sw] = o[1];
        if (two) {
            my_row[2 ^ sw] = o1[0];
            my_row[3 ^ sw] = o1[1];
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && row_base < p.M) {  // rows past M are clipped; a block wholly past M is skipped
                tma_store_2d(tmO, stage, n0 + c, row_base);
                bulk_commit();
            }
        } else {
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int rr = i * 16 + (lane >> 1), k = lane & 1;
                const uint4 v = reinterpret_cast<const uint4 *>(stage + rr * 64)[k ^ ((rr >> 1) & 3)];
                if (row_base + rr < p.M)
                    *reinterpret_cast<uint4 *>(p.out + (size_t)(row_base + rr) * p.ldo + n0 + c + k * 8) = v;
            }
            __syncwarp();
        }
    }
    return true;
}

// Column split of a w-wide tile between the two epilogue warps of a quadrant
// (at a multiple of 32 near the middle).
__host__ __device__ constexpr int epi_split(int w) { return ((w / 2 + 16) / 32) * 32; }
template <int BN> __host__ __device__ constexpr int epi_split() { return epi_split(BN); }

// N is covered by ceil(N / BN) column tiles: all BN wide except the last,
// which is `tail` = N - (num_n - 1) * BN wide (a multiple of 16) and has its own
// tensor map (tmBt, box rows = tail) and UMMA instruction descriptor. With
// BN = 256 this keeps every MMA but the tail's at the full N = 256 issue width
// (N = 640 -> 256, 256, 128), which runs faster than equal narrower tiles:
// an M = 128, K = 16 MMA takes about as long at N = 128 or 160 as at N = 256.
// With a residual matrix, the producer also prefetches each tile's residual
// block into L2 (tmR, boxes of 128 x 128) when it starts loading the tile, so
// the epilogue's residual reads, a tile later, hit L2 instead of HBM.
template <int BN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_bf16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmBt, const __grid_constant__ CUtensorMap tmR,
                const __grid_constant__ CUtensorMap tmO, GemmArgs p) {
    using Cfg = GemmCfg<BN>;
    constexpr int S = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * Cfg::A_BYTES;
    uint8_t *staging = smem + S * Cfg::STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(staging + STAGING_BYTES);
    uint64_t *full = bars, *empty = bars + S, *tfull = bars + 2 * S, *tempty = bars + 2 * S + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * S + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_n = (p.N + BN - 1) / BN;
    const int tail = p.N - (num_n - 1) * BN;
    const int num_m = (p.M + BM - 1) / BM;
    const int ntiles = num_m * num_n;
    const int nk = p.K / BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], EPI_WARPS); }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
        if (tail != BN) prefetch_tensormap(&tmBt);
        if (p.res) prefetch_tensormap(&tmR);
    }
    if (warp == 1) { tmem_alloc(tmem_holder, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
                const int nt = t % num_n, m0 = (t / num_n) * BM, n0 = nt * BN;
                const bool last = nt == num_n - 1;
                const CUtensorMap *tb = last ? &tmBt : &tmB;
                const uint32_t bytes = (uint32_t)(Cfg::A_BYTES + (last ? tail : BN) * BK * 2);
                if (p.res)
                    for (int x = 0; x < (last ? tail : BN); x += RES_BOX) tma_prefetch_l2_2d(&tmR, n0 + x, m0);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[s], bytes);
                    tma_load_2d(sA + s * Cfg::A_BYTES, &tmA, kb * BK, m0, &full[s]);
                    tma_load_2d(sB + s * Cfg::B_BYTES, tb, kb * BK, n0, &full[s]);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
            }
            // Producer tail: wait until every stage's last fill has been released by
            // its MMA commit, so no tensor-core arrival is still in flight at exit.
            for (int i = 0; i < S; ++i) {
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) break;
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_full = umma_idesc_bf16(BM, BN);
            const uint32_t idesc_tail = umma_idesc_bf16(BM, tail);
            int s = 0;
            uint32_t ph = 0;
            int tl = 0;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tl) {
                const uint32_t idesc = t % num_n == num_n - 1 ? idesc_tail : idesc_full;
                const int buf = tl & 1;
                const uint32_t use = (uint32_t)(tl >> 1);
                if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, abort_flag, p.status, ERR_WAIT_TMEM_EMPTY)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * BN);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&full[s], ph, abort_flag, p.status, ERR_WAIT_TMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = umma_desc_sw128(smem_u32(sA + s * Cfg::A_BYTES));
                    const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + s * Cfg::B_BYTES));
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k) {
                        // +32 bytes along K inside the swizzle atom = +2 in the >>4 address field
                        umma_bf16(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                                  (kb | k) != 0 ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else {
        // epilogue warps 2..9: TMEM lane quadrant = warp % 4, column half = (warp - 2) / 4
        const int quad = warp & 3, e = warp - 2, half = e >> 2;
        uint8_t *stage = staging + e * (32 * 64);
        const uint32_t bias_sa = stage_bias(p, staging + STAGING_BYTES + BARRIER_BYTES);
        int tl = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tl) {
            const int nt = t % num_n, m0 = (t / num_n) * BM, n0 = nt * BN;
            const int w = nt == num_n - 1 ? tail : BN;
            const int c0 = half ? epi_split(w) : 0, c1 = half ? w : epi_split(w);
            const int buf = tl & 1;
            const uint32_t use = (uint32_t)(tl >> 1);
            const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN);
            if (!epilogue_tile(p, tbase, m0 + quad * 32, n0, c0, c1, stage, lane, &tfull[buf], use & 1, abort_flag,
                               bias_sa, &tmO))
                break;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
        if (lane == 0) bulk_wait0();  // this warp's output stores are complete before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512);
}

// ------------------------------------------------------------------ operand-swapped variant
// out = A W^T computed as its transpose D[feature, token] = W A^T: the weight
// rows are the UMMA's M side (128 features per tile, so N = 640 is five full
// tiles) and the activation rows its N side (256 tokens per tile). On a layer
// with N = 640 the normal tiling needs 256 + 256 + 128 columns, and its
// 128-wide tile costs as many MMA cycles as a full one once the main loop is
// long (K = 2560): this variant does no such waste. Same stages, same
// roles, same bounded waits as k_gemm_bf16; the epilogue transposes through
// the staging buffer:
//   lane f of a quadrant holds feature f of 32 tokens (tcgen05.ld 32x32b);
//   bias is one value per lane; the residual block (32 tokens x 32 features)
//   is loaded row-wise (8 rows x 64 B per instruction) into the staging
//   buffer and read back by column; the bf16 results are written by column
//   into the staging buffer, which one bulk tensor store per 32 x 32 block
//   writes to global memory row by row.
// Staging rows are 64 B with 16-byte chunks XOR-swizzled by (row >> 1) & 3,
// which keeps both the row-wise and the column-wise accesses conflict-free.
constexpr int TN_BM = 128, TN_BN = 256;  // features x tokens per tile
using TnCfg = GemmCfg<TN_BN>;            // A stage 128 x 64, B stage 256 x 64: the same bytes

__device__ __forceinline__ int stage_off(int row, int col) {  // byte offset of bf16 (row, col) in a 32 x 32 block
    return row * 64 + ((((col >> 3) ^ ((row >> 1) & 3))) << 4) + ((col & 7) << 1);
}

// The residual block of tokens t0 .. t0 + 31, features f0 .. f0 + 31, in the
// row-wise pattern: g[i] is token i * 8 + lane / 4, 16 bytes at lane % 4
// (zeros past the last token).
__device__ __forceinline__ void res_load_tn(const GemmArgs &p, int t0, int f0, int lane, uint4 (&g)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int rr = i * 8 + (lane >> 2), k = lane & 3;
        g[i] = t0 + rr < p.M ? *reinterpret_cast<const uint4 *>(p.res + (size_t)(t0 + rr) * p.ldr + f0 + k * 8)
                             : make_uint4(0, 0, 0, 0);
    }
}

// One epilogue warp of the swapped tile: features f0 .. f0 + 31 (its TMEM lane
// quadrant, one feature per lane) and token columns [c0, c1) of the tile
// whose first token is tok0. The residual loads run one 32-token group
// ahead, the first group's before the wait for the accumulator. Each group's
// 32 tokens x 32 features leave the staging buffer by one bulk tensor store
// (tmO) issued by lane 0.
__device__ __forceinline__ bool epilogue_tile_tn(const GemmArgs &p, uint32_t tbase, int f0, int tok0, int c0, int c1,
                                                 uint8_t *stage, int lane, uint64_t *tfull_bar, uint32_t parity,
                                                 volatile int *abort_flag, const CUtensorMap *tmO) {
    const int f = f0 + lane;  // this lane's output column
    const float bias = p.bias ? __ldg(p.bias + f) : 0.f;
    uint4 g[4];
    if (p.res) res_load_tn(p, tok0 + c0, f0, lane, g);
    if (!mbar_wait(tfull_bar, parity, abort_flag, p.status, ERR_WAIT_TMEM_FULL)) return false;
    tc_fence_after();
#pragma unroll 1
    for (int c = c0; c < c1; c += 32) {
        const int t0 = tok0 + c;  // first token of the group
        // the group's residual, row-wise into the staging buffer; then the next group's loads
        if (p.res) {
            // the staging buffer is free once the previous group's bulk store has read it
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int rr = i * 8 + (lane >> 2), k = lane & 3;
                *reinterpret_cast<uint4 *>(stage + rr * 64 + ((k ^ ((rr >> 1) & 3)) << 4)) = g[i];
            }
            __syncwarp();
            if (c + 32 < c1) res_load_tn(p, t0 + 32, f0, lane, g);
        }
        uint32_t r[32];
        tmem_ld16(tbase + (uint32_t)c, *reinterpret_cast<uint32_t(*)[16]>(r));
        tmem_ld16(tbase + (uint32_t)(c + 16), *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        tmem_ld_wait();
        uint16_t o[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) {
            float v = __uint_as_float(r[t]) + bias;
            if (p.relu) v = fmaxf(v, 0.f);
            if (p.res) v += __bfloat162float(*reinterpret_cast<const bf16 *>(stage + stage_off(t, lane)));
            const bf16 h = __float2bfloat16_rn(v);
            o[t] = *reinterpret_cast<const uint16_t *>(&h);
        }
        __syncwarp();  // every lane has read its residual column before the buffer is overwritten
        if (!p.res) {  // the staging buffer is free once the previous group's bulk store has read it
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
        }
#pragma unroll
        for (int t = 0; t < 32; ++t) *reinterpret_cast<uint16_t *>(stage + stage_off(t, lane)) = o[t];
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(tmO, stage, f0, t0);
            bulk_commit();
        }
    }
    return true;
}

// tmA: the weights W [N, K] (box 128 rows); tmB: the activations [M, K] (box
// 256 rows); tmR: the residual [M, N] for the L2 prefetch (box 128 x 128).
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_bf16_tn(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmR, const __grid_constant__ CUtensorMap tmO, GemmArgs p) {
    constexpr int S = TnCfg::STAGES;
    constexpr int A_BYTES = TN_BM * BK * 2, B_BYTES = TN_BN * BK * 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * A_BYTES;
    uint8_t *staging = smem + S * (A_BYTES + B_BYTES);
    uint64_t *bars = reinterpret_cast<uint64_t *>(staging + STAGING_BYTES);
    uint64_t *full = bars, *empty = bars + S, *tfull = bars + 2 * S, *tempty = bars + 2 * S + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * S + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_f = p.N / TN_BM;                      // feature tiles
    const int num_t = (p.M + TN_BN - 1) / TN_BN;        // token tiles
    const int ntiles = num_f * num_t;                   // tile t: tokens (t / num_f), features (t % num_f)
    const int nk = p.K / BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], EPI_WARPS); }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
        if (p.res) prefetch_tensormap(&tmR);
    }
    if (warp == 1) { tmem_alloc(tmem_holder, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
                const int f0 = (t % num_f) * TN_BM, tok0 = (t / num_f) * TN_BN;
                if (p.res) {
                    tma_prefetch_l2_2d(&tmR, f0, tok0);
                    tma_prefetch_l2_2d(&tmR, f0, tok0 + 128);
                }
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[s], (uint32_t)(A_BYTES + B_BYTES));
                    tma_load_2d(sA + s * A_BYTES, &tmA, kb * BK, f0, &full[s]);
                    tma_load_2d(sB + s * B_BYTES, &tmB, kb * BK, tok0, &full[s]);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
            }
            for (int i = 0; i < S; ++i) {  // every stage released before exit
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) break;
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(TN_BM, TN_BN);
            int s = 0;
            uint32_t ph = 0;
            int tl = 0;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tl) {
                const int buf = tl & 1;
                const uint32_t use = (uint32_t)(tl >> 1);
                if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, abort_flag, p.status, ERR_WAIT_TMEM_EMPTY)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * TN_BN);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&full[s], ph, abort_flag, p.status, ERR_WAIT_TMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = umma_desc_sw128(smem_u32(sA + s * A_BYTES));
                    const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + s * B_BYTES));
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k)
                        umma_bf16(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc, (kb | k) != 0 ? 1u : 0u);
                    umma_commit(&empty[s]);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else {
        // epilogue warps 2..9: TMEM lane quadrant (32 features) = warp % 4, token half = (warp - 2) / 4
        const int quad = warp & 3, e = warp - 2, half = e >> 2;
        uint8_t *stage = staging + e * (32 * 64);
        int tl = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tl) {
            const int f0 = (t % num_f) * TN_BM, tok0 = (t / num_f) * TN_BN;
            // token columns of this half that exist (the last token tile may be partial)
            const int c0 = half * (TN_BN / 2);
            const int cend = ((p.M - tok0 + 31) / 32) * 32;
            const int c1 = c0 + TN_BN / 2 < cend ? c0 + TN_BN / 2 : cend;
            const int buf = tl & 1;
            const uint32_t use = (uint32_t)(tl >> 1);
            const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * TN_BN);
            if (c0 < c1) {
                if (!epilogue_tile_tn(p, tbase, f0 + quad * 32, tok0, c0, c1, stage, lane, &tfull[buf], use & 1,
                                      abort_flag, &tmO))
                    break;
            } else if (!mbar_wait(&tfull[buf], use & 1, abort_flag, p.status, ERR_WAIT_TMEM_FULL)) {
                break;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
        if (lane == 0) bulk_wait0();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512);
}

// ------------------------------------------------------------------ CTA-pair variant
// tcgen05.mma.cta_group::2 with M = 256: a cluster of two CTAs computes a
// 256 x BN tile. Each CTA loads its own 128 rows of A and half (BN/2 rows) of
// W, so the W bytes a CTA moves per FLOP halve against the single-CTA kernel.
// The leader (cluster rank 0) waits for both CTAs' bytes on its own "full"
// barrier, issues the MMAs, and signals each CTA's "empty" and "tile full"
// barriers with one commit per CTA. Each CTA's epilogue drains its own TMEM
// (its 128 rows) and arrives on the leader's "tile empty" barrier.
// Each CTA loads only into its own shared memory (no load is shared across the pair).
template <int BN> struct Gemm2Cfg {
    static constexpr int BNH = BN / 2;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BNH * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES_RAW = (SMEM_BUDGET - 2048 - STAGING_BYTES - BIAS_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + STAGING_BYTES + BARRIER_BYTES + BIAS_BYTES;
    static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "pair UMMA N must be a multiple of 16 in [32, 256]");
    static_assert(B_BYTES % 1024 == 0, "B stage must keep 1024-byte alignment for the 128B swizzle");
};

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    k_gemm2_bf16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmO, GemmArgs p) {
    using Cfg = Gemm2Cfg<BN>;
    constexpr int S = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * Cfg::A_BYTES;
    uint8_t *staging = smem + S * Cfg::STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(staging + STAGING_BYTES);
    uint64_t *full = bars, *empty = bars + S, *tfull = bars + 2 * S, *tempty = bars + 2 * S + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * S + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int num_n = p.N / BN;
    const int num_m = (p.M + 2 * BM - 1) / (2 * BM);
    const int ntiles = num_m * num_n;
    const int nk = p.K / BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], 2 * EPI_WARPS); }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) { tmem_alloc_pair(tmem_holder, 512); tmem_relinquish_pair(); }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (int t = pair; t < ntiles; t += npairs) {
                const int m0 = (t / num_n) * (2 * BM) + (int)rank * BM;
                const int n0 = (t % num_n) * BN + (int)rank * Cfg::BNH;
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) { ok = false; break; }
                    const uint32_t fbar = mapa_shared(smem_u32(&full[s]), 0);
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
                    tma_load_2d_pair(sA + s * Cfg::A_BYTES, &tmA, kb * BK, m0, fbar);
                    tma_load_2d_pair(sB + s * Cfg::B_BYTES, &tmB, kb * BK, n0, fbar);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
            }
            for (int i = 0; i < S; ++i) {  // tail: every stage released before exit
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) break;
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(2 * BM, BN);
            int s = 0;
            uint32_t ph = 0;
            int tl = 0;
            for (int t = pair; t < ntiles; t += npairs, ++tl) {
                const int buf = tl & 1;
                const uint32_t use = (uint32_t)(tl >> 1);
                if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, abort_flag, p.status, ERR_WAIT_TMEM_EMPTY)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * BN);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&full[s], ph, abort_flag, p.status, ERR_WAIT_TMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = umma_desc_sw128(smem_u32(sA + s * Cfg::A_BYTES));
                    const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + s * Cfg::B_BYTES));
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k)
                        umma_bf16_pair(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                                       (kb | k) != 0 ? 1u : 0u);
                    umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 0));
                    umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
                umma_commit_pair(mapa_shared(smem_u32(&tfull[buf]), 0));
                umma_commit_pair(mapa_shared(smem_u32(&tfull[buf]), 1));
            }
        }
    } else {
        const int quad = warp & 3, e = warp - 2, half = e >> 2;
        const int c0 = half ? epi_split<BN>() : 0, c1 = half ? BN : epi_split<BN>();
        uint8_t *stage = staging + e * (32 * 64);
        const uint32_t bias_sa = stage_bias(p, staging + STAGING_BYTES + BARRIER_BYTES);
        int tl = 0;
        for (int t = pair; t < ntiles; t += npairs, ++tl) {
            const int buf = tl & 1;
            const uint32_t use = (uint32_t)(tl >> 1);
            const int row_base = (t / num_n) * (2 * BM) + (int)rank * BM + quad * 32;
            const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN);
            if (!epilogue_tile(p, tbase, row_base, (t % num_n) * BN, c0, c1, stage, lane, &tfull[buf], use & 1,
                               abort_flag, bias_sa, &tmO))
                break;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[buf]), 0));
        }
        if (lane == 0) bulk_wait0();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers or use its TMEM
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, 512);
}

// ------------------------------------------------------------------ operand-swapped CTA pair
// The swapped tiling on a CTA pair (tcgen05.mma.cta_group::2, M = 256): a
// cluster of two CTAs computes 256 features x 256 tokens. CTA r loads its own
// 128 weight rows (features fp * 256 + 128 r) and its half of the tile's
// tokens (tok0 + 128 r), so a CTA moves 32 KB of operands per 64-deep k-block
// for the same MMA work as the single-CTA swapped kernel's 48 KB. Barriers
// and roles are those of k_gemm2_bf16; each CTA's epilogue drains its 128
// features x 256 tokens with the swapped epilogue. When N is an odd multiple
// of 128, the last pair's second CTA has no features: its weight loads read
// the tensor map's zero fill past N, and its epilogue stores nothing.
// Layers with a residual are not run on this kernel.
using Tn2Cfg = Gemm2Cfg<256>;  // per CTA and stage: 128 weight rows and 128 tokens, 64 deep

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    k_gemm2_bf16_tn(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmO, GemmArgs p) {
    using Cfg = Tn2Cfg;
    constexpr int S = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * Cfg::A_BYTES;
    uint8_t *staging = smem + S * Cfg::STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(staging + STAGING_BYTES);
    uint64_t *full = bars, *empty = bars + S, *tfull = bars + 2 * S, *tempty = bars + 2 * S + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * S + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int num_fp = (p.N + 2 * TN_BM - 1) / (2 * TN_BM);  // feature pairs
    const int num_t = (p.M + TN_BN - 1) / TN_BN;             // token tiles
    const int ntiles = num_fp * num_t;                        // tile t: tokens t / num_fp, features t % num_fp
    const int nk = p.K / BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], 2 * EPI_WARPS); }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) { tmem_alloc_pair(tmem_holder, 512); tmem_relinquish_pair(); }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (int t = pair; t < ntiles; t += npairs) {
                const int f0 = (t % num_fp) * (2 * TN_BM) + (int)rank * TN_BM;
                const int tok0 = (t / num_fp) * TN_BN + (int)rank * (TN_BN / 2);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) { ok = false; break; }
                    const uint32_t fbar = mapa_shared(smem_u32(&full[s]), 0);
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
                    tma_load_2d_pair(sA + s * Cfg::A_BYTES, &tmA, kb * BK, f0, fbar);
                    tma_load_2d_pair(sB + s * Cfg::B_BYTES, &tmB, kb * BK, tok0, fbar);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
            }
            for (int i = 0; i < S; ++i) {  // tail: every stage released before exit
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) break;
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(2 * TN_BM, TN_BN);
            int s = 0;
            uint32_t ph = 0;
            int tl = 0;
            for (int t = pair; t < ntiles; t += npairs, ++tl) {
                const int buf = tl & 1;
                const uint32_t use = (uint32_t)(tl >> 1);
                if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, abort_flag, p.status, ERR_WAIT_TMEM_EMPTY)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * TN_BN);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&full[s], ph, abort_flag, p.status, ERR_WAIT_TMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = umma_desc_sw128(smem_u32(sA + s * Cfg::A_BYTES));
                    const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + s * Cfg::B_BYTES));
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k)
                        umma_bf16_pair(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                                       (kb | k) != 0 ? 1u : 0u);
                    umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 0));
                    umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
                umma_commit_pair(mapa_shared(smem_u32(&tfull[buf]), 0));
                umma_commit_pair(mapa_shared(smem_u32(&tfull[buf]), 1));
            }
        }
    } else {
        // epilogue warps 2..9: TMEM lane quadrant (32 features) = warp % 4, token half = (warp - 2) / 4
        const int quad = warp & 3, e = warp - 2, half = e >> 2;
        uint8_t *stage = staging + e * (32 * 64);
        int tl = 0;
        for (int t = pair; t < ntiles; t += npairs, ++tl) {
            const int f0 = (t % num_fp) * (2 * TN_BM) + (int)rank * TN_BM;  // this CTA's first feature
            const int tok0 = (t / num_fp) * TN_BN;
            const int c0 = half * (TN_BN / 2);
            const int cend = ((p.M - tok0 + 31) / 32) * 32;
            const int c1 = c0 + TN_BN / 2 < cend ? c0 + TN_BN / 2 : cend;
            const int buf = tl & 1;
            const uint32_t use = (uint32_t)(tl >> 1);
            const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * TN_BN);
            if (f0 < p.N && c0 < c1) {
                if (!epilogue_tile_tn(p, tbase, f0 + quad * 32, tok0, c0, c1, stage, lane, &tfull[buf], use & 1,
                                      abort_flag, &tmO))
                    break;
            } else if (!mbar_wait(&tfull[buf], use & 1, abort_flag, p.status, ERR_WAIT_TMEM_FULL)) {
                break;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[buf]), 0));
        }
        if (lane == 0) bulk_wait0();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers or use its TMEM
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, 512);
}

// ------------------------------------------------------------------ LayerNorm-fused variant (N = 640)
// A cluster of four CTAs owns one 128-row block of the 640-column output;
// cluster rank r computes columns [160 r, 160 r + 160) with the single-CTA
// pipeline. The epilogue never writes y:
//   pass A  y = bf16(acc + bias [+ residual]) per 32-column group; the row's
//           count / mean / M2 over the warp's columns, merged group by group
//           with Chan's parallel-variance update;
//   exchange  each of the 8 epilogue warps x 4 CTAs stores (mean, M2) of its
//           rows into every cluster CTA's shared memory (st.shared::cluster),
//           then arrives on each CTA's exchange barrier (release.cluster);
//           after its own barrier completes (acquire.cluster) a CTA merges the
//           8 partials of each row in a fixed order: mean and variance of all
//           640 values (biased, as the reference LayerNorm);
//   pass B  y recomputed from TMEM, out = bf16((y - mean) rstd g + b), staged
//           through shared memory and stored row-contiguously.
// This is LN1 fused into out-proj and LN2 into FFN2 (tessera_cpu.cpp:424-428).
constexpr int LN_N = 640, LN_BN = 160, LN_CTAS = 4;
constexpr int LN_CONTRIB = 2 * LN_CTAS;                  // epilogue warps covering one row
constexpr int XCH_BYTES = 2 * LN_CONTRIB * BM * 8;       // [tile parity][contributor][row] (mean, M2)
struct GemmLnCfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = LN_BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES_RAW = (SMEM_BUDGET - 2048 - STAGING_BYTES - XCH_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + STAGING_BYTES + XCH_BYTES + 256;
};

// y values of one 16-column group, rounded to bf16 (the value the reference
// hands to LayerNorm), as floats.
__device__ __forceinline__ void ln_y16(const GemmArgs &p, const uint32_t (&r)[16], const uint4 (&res)[2], bool has_res,
                                       int n, float (&y)[16]) {
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = __uint_as_float(r[j]);
    if (p.bias) {
        const float4 *b4 = reinterpret_cast<const float4 *>(p.bias + n);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 b = __ldg(b4 + j);
            y[4 * j] += b.x; y[4 * j + 1] += b.y; y[4 * j + 2] += b.z; y[4 * j + 3] += b.w;
        }
    }
    if (p.relu) {
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = fmaxf(y[j], 0.f);
    }
    if (has_res) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t w[4] = {res[h].x, res[h].y, res[h].z, res[h].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                y[8 * h + 2 * j] += bf16lo(w[j]);
                y[8 * h + 2 * j + 1] += bf16hi(w[j]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = bf16_round(y[j]);
}

// Chan et al. merge of (n_b, mean_b, m2_b) into (n, mean, m2).
__device__ __forceinline__ void chan_merge(float &n, float &mean, float &m2, float nb, float meanb, float m2b) {
    const float tot = n + nb;
    const float delta = meanb - mean;
    mean += delta * (nb / tot);
    m2 += m2b + delta * delta * (n * nb / tot);
    n = tot;
}

__device__ __forceinline__ bool ln_epilogue_tile(const GemmArgs &p, uint32_t tbase, int row_base, int n0, int c0,
                                                 int c1, uint8_t *stage, int lane, uint64_t *tfull_bar,
                                                 uint32_t tfull_parity, float2 *xch, uint64_t *xbar,
                                                 uint32_t xbar_parity, int contributor, int quad,
                                                 volatile int *abort_flag) {
    const int row = row_base + lane;
    const bool live = row < p.M;
    const bf16 *res_row = (live && p.res) ? p.res + (size_t)row * p.ldr : nullptr;
    auto load_group = [&](int c, uint4 (&q)[4]) {
        if (res_row) {
            const uint4 *r4 = reinterpret_cast<const uint4 *>(res_row + n0 + c);
            q[0] = r4[0];
            q[1] = r4[1];
            if (c + 32 <= c1) { q[2] = r4[2]; q[3] = r4[3]; }
        }
    };
    uint4 qn[4] = {};
    load_group(c0, qn);
    if (!mbar_wait(tfull_bar, tfull_parity, abort_flag, p.status, ERR_WAIT_TMEM_FULL)) return false;
    tc_fence_after();
    // ---- pass A: statistics of this warp's columns
    float cnt = 0.f, mean = 0.f, m2 = 0.f;
#pragma unroll 1
    for (int c = c0; c < c1; c += 32) {
        const bool two = c + 32 <= c1;
        const uint4 q0[2] = {qn[0], qn[1]}, q1[2] = {qn[2], qn[3]};
        if (c + 32 < c1) load_group(c + 32, qn);
        uint32_t r0[16], r1[16];
        tmem_ld16(tbase + (uint32_t)c, r0);
        if (two) tmem_ld16(tbase + (uint32_t)(c + 16), r1);
        tmem_ld_wait();
        float y[16];
        ln_y16(p, r0, q0, res_row != nullptr, n0 + c, y);
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) s += y[j];
        float gm = s / 16.f, g2 = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) { const float d = y[j] - gm; g2 += d * d; }
        chan_merge(cnt, mean, m2, 16.f, gm, g2);
        if (two) {
            ln_y16(p, r1, q1, res_row != nullptr, n0 + c + 16, y);
            s = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) s += y[j];
            gm = s / 16.f;
            g2 = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) { const float d = y[j] - gm; g2 += d * d; }
            chan_merge(cnt, mean, m2, 16.f, gm, g2);
        }
    }
    // ---- exchange (mean, M2) of this warp's rows with the 4 cluster CTAs
    const int rloc = quad * 32 + lane;
    const uint32_t slot = smem_u32(&xch[contributor * BM + rloc]);
#pragma unroll
    for (int dst = 0; dst < LN_CTAS; ++dst) st_cluster_f32x2(mapa_shared(slot, (uint32_t)dst), mean, m2);
    fence_acq_rel_cluster();
    __syncwarp();
    if (lane == 0) {
#pragma unroll
        for (int dst = 0; dst < LN_CTAS; ++dst) mbar_arrive_cluster(mapa_shared(smem_u32(xbar), (uint32_t)dst));
    }
    if (!mbar_wait_cluster(xbar, xbar_parity, abort_flag, p.status, ERR_WAIT_LN_EXCHANGE)) return false;
    float n_all = 0.f, mean_all = 0.f, m2_all = 0.f;
#pragma unroll
    for (int k = 0; k < LN_CONTRIB; ++k) {
        const float2 v = xch[k * BM + rloc];
        const float nk = (k & 1) ? float(LN_BN - epi_split<LN_BN>()) : float(epi_split<LN_BN>());
        chan_merge(n_all, mean_all, m2_all, nk, v.x, v.y);
    }
    const float rstd = 1.f / sqrtf(m2_all / (float)LN_N + LN_EPS);
    // ---- pass B: normalise and store
    load_group(c0, qn);
    uint4 *my_row = reinterpret_cast<uint4 *>(stage + lane * 64);
    const int sw = (lane >> 1) & 3;
#pragma unroll 1
    for (int c = c0; c < c1; c += 32) {
        const bool two = c + 32 <= c1;
        const uint4 q0[2] = {qn[0], qn[1]}, q1[2] = {qn[2], qn[3]};
        if (c + 32 < c1) load_group(c + 32, qn);
        uint32_t r0[16], r1[16];
        tmem_ld16(tbase + (uint32_t)c, r0);
        if (two) tmem_ld16(tbase + (uint32_t)(c + 16), r1);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (h == 1 && !two) break;
            float y[16];
            const int n = n0 + c + 16 * h;
            ln_y16(p, h ? r1 : r0, h ? q1 : q0, res_row != nullptr, n, y);
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = (y[j] - mean_all) * rstd * __ldg(p.ln_g + n + j) + __ldg(p.ln_b + n + j);
            my_row[(2 * h) ^ sw] = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]),
                                              pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
            my_row[(2 * h + 1) ^ sw] = make_uint4(pack_bf16x2(o[8], o[9]), pack_bf16x2(o[10], o[11]),
                                                  pack_bf16x2(o[12], o[13]), pack_bf16x2(o[14], o[15]));
        }
        __syncwarp();
        if (two) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int rr = i * 8 + (lane >> 2), k = lane & 3;
                const uint4 v = reinterpret_cast<const uint4 *>(stage + rr * 64)[k ^ ((rr >> 1) & 3)];
                if (row_base + rr < p.M)
                    *reinterpret_cast<uint4 *>(p.out + (size_t)(row_base + rr) * p.ldo + n0 + c + k * 8) = v;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int rr = i * 16 + (lane >> 1), k = lane & 1;
                const uint4 v = reinterpret_cast<const uint4 *>(stage + rr * 64)[k ^ ((rr >> 1) & 3)];
                if (row_base + rr < p.M)
                    *reinterpret_cast<uint4 *>(p.out + (size_t)(row_base + rr) * p.ldo + n0 + c + k * 8) = v;
            }
        }
        __syncwarp();
    }
    return true;
}

__global__ void __cluster_dims__(LN_CTAS, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_ln640(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs p) {
    using Cfg = GemmLnCfg;
    constexpr int S = Cfg::STAGES;
    constexpr int BN = LN_BN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * Cfg::A_BYTES;
    uint8_t *staging = smem + S * Cfg::STAGE_BYTES;
    float2 *xch = reinterpret_cast<float2 *>(staging + STAGING_BYTES);
    uint64_t *bars = reinterpret_cast<uint64_t *>(staging + STAGING_BYTES + XCH_BYTES);
    uint64_t *full = bars, *empty = bars + S, *tfull = bars + 2 * S, *tempty = bars + 2 * S + 2;
    uint64_t *xbar = bars + 2 * S + 4;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * S + 6);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int cl = blockIdx.x / LN_CTAS, ncl = gridDim.x / LN_CTAS;
    const int num_m = (p.M + BM - 1) / BM;
    const int nk = p.K / BK;
    const int n0 = (int)rank * BN;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], EPI_WARPS);
            mbar_init(&xbar[i], EPI_WARPS * LN_CTAS);
        }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) { tmem_alloc(tmem_holder, 512); tmem_relinquish(); }
    tc_fence_before();
    cluster_sync();  // every CTA's exchange barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (int mb = cl; mb < num_m; mb += ncl) {
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                    tma_load_2d(sA + s * Cfg::A_BYTES, &tmA, kb * BK, mb * BM, &full[s]);
                    tma_load_2d(sB + s * Cfg::B_BYTES, &tmB, kb * BK, n0, &full[s]);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
            }
            for (int i = 0; i < S; ++i) {
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, ERR_WAIT_SMEM_EMPTY)) break;
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(BM, BN);
            int s = 0;
            uint32_t ph = 0;
            int tl = 0;
            for (int mb = cl; mb < num_m; mb += ncl, ++tl) {
                const int buf = tl & 1;
                const uint32_t use = (uint32_t)(tl >> 1);
                if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, abort_flag, p.status, ERR_WAIT_TMEM_EMPTY)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * BN);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&full[s], ph, abort_flag, p.status, ERR_WAIT_TMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = umma_desc_sw128(smem_u32(sA + s * Cfg::A_BYTES));
                    const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + s * Cfg::B_BYTES));
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k)
                        umma_bf16(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc, (kb | k) != 0 ? 1u : 0u);
                    umma_commit(&empty[s]);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else {
        const int quad = warp & 3, e = warp - 2, half = e >> 2;
        const int c0 = half ? epi_split<BN>() : 0, c1 = half ? BN : epi_split<BN>();
        uint8_t *stage = staging + e * (32 * 64);
        const int contributor = (int)rank * 2 + half;
        int tl = 0;
        for (int mb = cl; mb < num_m; mb += ncl, ++tl) {
            const int buf = tl & 1;
            const uint32_t use = (uint32_t)(tl >> 1);
            const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN);
            if (!ln_epilogue_tile(p, tbase, mb * BM + quad * 32, n0, c0, c1, stage, lane, &tfull[buf], use & 1,
                                  xch + buf * LN_CONTRIB * BM, &xbar[buf], use & 1, contributor, quad, abort_flag))
                break;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while a peer may still write its exchange slots or barriers
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512);
}

// ------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix (cols contiguous)
// with the given box and swizzle. Rows past `rows` read as zero.
void make_tmap_box(CUtensorMap *tm, const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                   uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    auto enc = get_encode_fn();
    if (!enc) throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
    if (reinterpret_cast<uintptr_t>(ptr) % 16) throw std::runtime_error("TMA base address not 16-byte aligned");
    if ((ld_elems * 2) % 16) throw std::runtime_error("TMA row pitch not a multiple of 16 bytes");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld_elems * 2};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

// The operand maps: box = [box_rows, 64 columns] (one 128-byte swizzle atom of K).
static void make_tmap(CUtensorMap *tm, const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                      uint32_t box_rows) {
    make_tmap_box(tm, ptr, rows, cols, ld_elems, BK, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// The output map of the bulk stores: [M, N] with pitch ldo, boxes of 32 rows x
// 32 columns (64 bytes, the 64-byte swizzle of the staging buffers).
static void make_tmap_out(CUtensorMap *tm, const GemmArgs &p) {
    make_tmap_box(tm, p.out, (uint64_t)p.M, (uint64_t)p.N, (uint64_t)p.ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
}

static int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int BN> static void launch_bn(const GemmArgs &p, const bf16 *A, int lda, const bf16 *W, cudaStream_t st,
                                        int max_ctas) {
    using Cfg = GemmCfg<BN>;
    static bool attr_set[64] = {};  // per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_bf16<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) throw std::runtime_error(std::string("gemm smem attribute: ") + cudaGetErrorString(e));
        attr_set[dev & 63] = true;
    }
    const int num_n = (p.N + BN - 1) / BN;
    const int tail = p.N - (num_n - 1) * BN;
    if (tail % 16 || tail < 16) throw std::runtime_error("gemm: N must be a multiple of 16");
    CUtensorMap ta, tb, tbt, tr;
    make_tmap(&ta, A, (uint64_t)p.M, (uint64_t)p.K, (uint64_t)lda, BM);
    if (p.res) make_tmap_box(&tr, p.res, (uint64_t)p.M, (uint64_t)p.N, (uint64_t)p.ldr, (uint32_t)std::min(RES_BOX, p.N),
                             BM, CU_TENSOR_MAP_SWIZZLE_NONE);
    else tr = ta;
    // (one tile narrower than BN: both maps get the tail's box, never wider than N)
    make_tmap(&tb, W, (uint64_t)p.N, (uint64_t)p.K, (uint64_t)p.K, num_n == 1 ? (uint32_t)tail : (uint32_t)BN);
    if (tail != BN) make_tmap(&tbt, W, (uint64_t)p.N, (uint64_t)p.K, (uint64_t)p.K, (uint32_t)tail);
    else tbt = tb;
    const int ntiles = ((p.M + BM - 1) / BM) * num_n;
    int grid = std::min(ntiles, num_sms());
    if (max_ctas > 0) grid = std::min(grid, max_ctas);
    if (grid < 1) grid = 1;
    CUtensorMap to;
    make_tmap_out(&to, p);
    k_gemm_bf16<BN><<<grid, GEMM_THREADS, Cfg::SMEM_BYTES, st>>>(ta, tb, tbt, tr, to, p);
}

static void launch_tn(const GemmArgs &p, const bf16 *A, int lda, const bf16 *W, cudaStream_t st, int max_ctas) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_bf16_tn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             TnCfg::SMEM_BYTES);
        if (e != cudaSuccess) throw std::runtime_error(std::string("gemm_tn smem attribute: ") + cudaGetErrorString(e));
        attr_set[dev & 63] = true;
    }
    CUtensorMap ta, tb, tr;
    make_tmap(&ta, W, (uint64_t)p.N, (uint64_t)p.K, (uint64_t)p.K, TN_BM);
    make_tmap(&tb, A, (uint64_t)p.M, (uint64_t)p.K, (uint64_t)lda, TN_BN);
    if (p.res) make_tmap_box(&tr, p.res, (uint64_t)p.M, (uint64_t)p.N, (uint64_t)p.ldr, 128, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
    else tr = ta;
    const int ntiles = (p.N / TN_BM) * ((p.M + TN_BN - 1) / TN_BN);
    int grid = std::min(ntiles, num_sms());
    if (max_ctas > 0) grid = std::min(grid, max_ctas);
    if (grid < 1) grid = 1;
    CUtensorMap to;
    make_tmap_out(&to, p);
    k_gemm_bf16_tn<<<grid, GEMM_THREADS, TnCfg::SMEM_BYTES, st>>>(ta, tb, tr, to, p);
}

template <int BN> static void launch_pair(const GemmArgs &p, const bf16 *A, int lda, const bf16 *W, cudaStream_t st,
                                          int max_ctas) {
    using Cfg = Gemm2Cfg<BN>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        cudaError_t e =
            cudaFuncSetAttribute(k_gemm2_bf16<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) throw std::runtime_error(std::string("gemm2 smem attribute: ") + cudaGetErrorString(e));
        attr_set[dev & 63] = true;
    }
    CUtensorMap ta, tb;
    make_tmap(&ta, A, (uint64_t)p.M, (uint64_t)p.K, (uint64_t)lda, BM);
    make_tmap(&tb, W, (uint64_t)p.N, (uint64_t)p.K, (uint64_t)p.K, Cfg::BNH);
    const int ntiles = ((p.M + 2 * BM - 1) / (2 * BM)) * (p.N / BN);
    int pairs = std::min(ntiles, num_sms() / 2);
    if (max_ctas > 0) pairs = std::min(pairs, std::max(1, max_ctas / 2));
    if (pairs < 1) pairs = 1;
    CUtensorMap to;
    make_tmap_out(&to, p);
    k_gemm2_bf16<BN><<<2 * pairs, GEMM_THREADS, Cfg::SMEM_BYTES, st>>>(ta, tb, to, p);
}

static void launch_tn_pair(const GemmArgs &p, const bf16 *A, int lda, const bf16 *W, cudaStream_t st, int max_ctas) {
    using Cfg = Tn2Cfg;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        cudaError_t e =
            cudaFuncSetAttribute(k_gemm2_bf16_tn, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) throw std::runtime_error(std::string("gemm2_tn smem attribute: ") + cudaGetErrorString(e));
        attr_set[dev & 63] = true;
    }
    CUtensorMap ta, tb;
    make_tmap(&ta, W, (uint64_t)p.N, (uint64_t)p.K, (uint64_t)p.K, TN_BM);
    make_tmap(&tb, A, (uint64_t)p.M, (uint64_t)p.K, (uint64_t)lda, TN_BN / 2);
    const int ntiles = ((p.N + 2 * TN_BM - 1) / (2 * TN_BM)) * ((p.M + TN_BN - 1) / TN_BN);
    int pairs = std::min(ntiles, num_sms() / 2);
    if (max_ctas > 0) pairs = std::min(pairs, std::max(1, max_ctas / 2));
    if (pairs < 1) pairs = 1;
    CUtensorMap to;
    make_tmap_out(&to, p);
    k_gemm2_bf16_tn<<<2 * pairs, GEMM_THREADS, Cfg::SMEM_BYTES, st>>>(ta, tb, to, p);
}

static void launch_ln(const GemmArgs &p, const bf16 *A, int lda, const bf16 *W, cudaStream_t st) {
    using Cfg = GemmLnCfg;
    static int max_clusters[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!max_clusters[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_ln640, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) throw std::runtime_error(std::string("gemm_ln smem attribute: ") + cudaGetErrorString(e));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(LN_CTAS * 64);
        cfg.blockDim = dim3(GEMM_THREADS);
        cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, k_gemm_ln640, &cfg);
        if (e != cudaSuccess || n <= 0) throw std::runtime_error("gemm_ln: no cluster of 4 fits on this device");
        max_clusters[dev & 63] = n;
    }
    CUtensorMap ta, tb;
    make_tmap(&ta, A, (uint64_t)p.M, (uint64_t)p.K, (uint64_t)lda, BM);
    make_tmap(&tb, W, (uint64_t)LN_N, (uint64_t)p.K, (uint64_t)p.K, LN_BN);
    const int num_m = (p.M + BM - 1) / BM;
    const int clusters = std::max(1, std::min(num_m, max_clusters[dev & 63]));
    k_gemm_ln640<<<LN_CTAS * clusters, GEMM_THREADS, Cfg::SMEM_BYTES, st>>>(ta, tb, p);
}

// Kernel choice when launch_gemm is asked for variant 0. Unset, TC_GEMM_VARIANT
// picks per layer (gemm_auto_variant); 1 forces the single-CTA kernel, 2 the
// CTA-pair kernel, 3 the operand-swapped kernel wherever N is a multiple of 128.
int gemm_default_variant() {
    static int v = [] {
        const char *e = std::getenv("TC_GEMM_VARIANT");
        return e && *e >= '1' && *e <= '4' ? *e - '0' : 0;
    }();
    return v;
}

// The per-layer choice, from sustained timings at M = 524,288 (op_bench.py
// gemm, same call; the two kernels give bit-identical outputs): the swapped
// kernel is faster without a residual (QKV 1,334 against 1,479 us, FFN1 1,749
// against 1,869) and with one behind a long main loop (FFN2, K = 2560: 1,695
// against 1,766), and much slower for a residual behind a short one
// (out-proj, K = 640: 916 against 636), where its transposing epilogue is the
// critical path.
// TC_GEMM_TN_PAIR=1 runs the layers without a residual on the CTA-pair form of
// the swapped kernel (read once). Off by default: on the config-1 step (A/B in
// one call) FFN1 ran at 1,060 against 1,043 TFLOP/s but QKV, whose 1,920
// features leave the last pair half empty, at 999 against 1,038, and the step
// at 106.5-106.9k against 107.0-107.1k px/s.
static bool tn_pair_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("TC_GEMM_TN_PAIR");
        return e && *e == '1';
    }();
    return on;
}

static int gemm_auto_variant(const GemmArgs &p) {
    const bool swappable = p.N % TN_BM == 0 && !p.pe_doy && !p.ln_g;
    if (swappable && !p.res && tn_pair_enabled()) return 4;
    return swappable && (!p.res || p.K >= 2048) ? 3 : 1;
}

int gemm_pick_bn(int N) {
    if (N % 16 || N <= 0) return 0;
    if (N == 128) return 128;  // the smaller B stage leaves room for 6 pipeline stages
    return 256;                // 256-wide tiles, the last one narrower when 256 does not divide N
}

// The CTA-pair kernel needs BN | N (no tail tile).
static int gemm_pick_bn_pair(int N) {
    if (N % 256 == 0) return 256;
    if (N % 240 == 0) return 240;
    if (N % 160 == 0) return 160;
    if (N % 128 == 0) return 128;
    return 0;
}

void launch_gemm(const GemmArgs &p, const bf16 *A, int lda, const bf16 *W, cudaStream_t st, int bn, int max_ctas,
                 int variant) {
    if (p.M <= 0) return;
    if (p.K % BK) throw std::runtime_error("gemm: K must be a multiple of 64");
    if (variant == 0) variant = gemm_default_variant();
    if (variant == 0) variant = gemm_auto_variant(p);
    if (variant == 4 && p.res) variant = 3;  // the swapped pair takes no residual
    if (variant == 3 || variant == 4) {
        if (p.N % TN_BM || p.pe_doy || p.ln_g || p.ldo % 8 || (p.res && p.ldr % 8))
            variant = 1;  // shapes the swapped kernels do not take run on the single-CTA one
        else {
            if (variant == 4) launch_tn_pair(p, A, lda, W, st, max_ctas);
            else launch_tn(p, A, lda, W, st, max_ctas);
            return;
        }
    }
    if (bn == 0) bn = variant == 2 ? gemm_pick_bn_pair(p.N) : gemm_pick_bn(p.N);
    if (bn == 0 || p.N % 16 || (variant == 2 && p.N % bn))
        throw std::runtime_error("gemm: unsupported N " + std::to_string(p.N));
    if (p.ldo % 8 || (p.res && p.ldr % 8)) throw std::runtime_error("gemm: output/residual pitch must be 16-byte aligned");
    if (p.ln_g) {
        if (p.N != LN_N || !p.ln_b || p.pe_doy) throw std::runtime_error("gemm: LayerNorm epilogue needs N = 640");
        launch_ln(p, A, lda, W, st);
        return;
    }
    if (variant == 2) {
        switch (bn) {
        case 256: launch_pair<256>(p, A, lda, W, st, max_ctas); return;
        case 240: launch_pair<240>(p, A, lda, W, st, max_ctas); return;
        case 160: launch_pair<160>(p, A, lda, W, st, max_ctas); return;
        case 128: launch_pair<128>(p, A, lda, W, st, max_ctas); return;
        default: throw std::runtime_error("gemm: unsupported pair tile width " + std::to_string(bn));
        }
    }
    switch (bn) {
    case 256: launch_bn<256>(p, A, lda, W, st, max_ctas); break;
    case 160: launch_bn<160>(p, A, lda, W, st, max_ctas); break;
    case 128: launch_bn<128>(p, A, lda, W, st, max_ctas); break;
    default: throw std::runtime_error("gemm: unsupported tile width " + std::to_string(bn));
    }
}

}  // namespace tcb
