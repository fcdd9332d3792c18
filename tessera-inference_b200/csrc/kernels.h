// Launchers of the warp-level kernels (kernels.cu). All enqueue on `st` and
// throw std::runtime_error on invalid launch parameters.
#pragma once

#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace tcb {

// Pixel segments of a token stream: pixel i of a chunk owns tokens
// [seg(i), seg(i+1)) with seg(i) = off ? off[i] - base : i * uniform_T.
struct Segs {
    const int64_t *off = nullptr;
    int64_t base = 0;
    int64_t uniform_T = 0;
    // attention launches only: segment k of the launch is segment pix[k] of the chunk
    const int32_t *pix = nullptr;
};

// Raw tile arrays in device memory (tessera_encode.cpp:182-209 layout).
struct TileDev {
    const uint16_t *bands = nullptr;  // (T2, H, W, 10)
    const uint8_t *masks = nullptr;   // (T2, H, W)
    const uint16_t *doys = nullptr;   // (T2)
    const int16_t *asc = nullptr;     // (Ta, H, W, 2)
    const int16_t *asc_doy = nullptr; // (Ta)
    const int16_t *desc = nullptr;    // (Td, H, W, 2)
    const int16_t *desc_doy = nullptr;// (Td)
    int64_t T2 = 0, Ta = 0, Td = 0;
    int64_t N = 0;                    // pixels in the arrays (pixel stride of each time slice)
};

constexpr int MAX_STEPS = 2048;       // longest per-modality series the gather kernel accepts

// n2[p], n1[p] = valid S2 / S1 observations of pixels [p0, p0 + np) (tessera_encode.cpp:245-257).
void launch_count(const TileDev &t, int64_t p0, int64_t np, int32_t *n2, int32_t *n1, cudaStream_t st);

// Token records (bands z-scored + DOY, f32) of pixels [p0, p0 + np) of one modality,
// written at rec + (off[i] - base) * (C + 1) (tessera_encode.cpp:281-329).
// modality 0 = S2 (C = 10), 1 = S1 (C = 2). bins[i] = that pixel's token count.
void launch_gather(int modality, const TileDev &t, int64_t p0, int64_t np, const int32_t *nvalid,
                   const int32_t *bins, Segs segs, float *rec, cudaStream_t st);

// y[M, 640] = bf16(relu(bf16(rec[:, :C]) . W1^T + b1)); w1t is W1 transposed, f32 [C][640].
void launch_emb1(int C, const float *rec, int64_t M, const float *w1t, const float *b1, __nv_bfloat16 *y,
                 cudaStream_t st);

// Self-attention of pixel segments, 4 heads x 160, no mask (tessera_cpu.cpp:410-418).
// qkv holds ntok token rows of 1920 (the rows the segments index).
//
// The kernel for a pixel is chosen by that pixel's own series length T, so a
// pixel's result never depends on which other pixels share its chunk (row
// bands, devices and the tc_encode batches all give the same bytes):
//   class 0: the mma.sync kernel, for T <= 48 (every T <= 128 with TC_ATTN_TC=0);
//   class 1: the tcgen05 kernel, for 48 < T <= 128 (every T <= 128 with
//            TC_ATTN_TC=2); its bounded waits report into *status (may be null);
//   class 2: the tcgen05 kernel for 128 < T <= 256 (query halves of 128 rows,
//            S over up to 256 keys in TMEM), or the mma.sync kernel with
//            TC_ATTN_TC=0; its bounded waits report into *status.
int attention_class(int T);

// A chunk's pixels with T > 0 listed class by class (device memory), with the
// count and the longest series of each class.
struct AttnPlan {
    const int32_t *pix = nullptr;
    int64_t n[3] = {0, 0, 0};
    int tmax[3] = {0, 0, 0};
};
// Fills list[] (host, room for npix entries) and plan.n / plan.tmax from the
// segment offsets off[0..npix] (host); plan.pix is left for the caller to set
// to a device copy of list.
void attention_plan(const int64_t *off, int64_t npix, int32_t *list, AttnPlan &plan);
// Both return the number of kernels launched (one per non-empty class).
int launch_attention_plan(const __nv_bfloat16 *qkv, Segs segs, const AttnPlan &plan, int64_t ntok,
                          __nv_bfloat16 *att, int *status, cudaStream_t st);
// Every pixel with the same series length Tmax (segs describes uniform or
// offset segments): one class, one launch.
int launch_attention(const __nv_bfloat16 *qkv, Segs segs, int64_t npix, int64_t ntok, int Tmax, __nv_bfloat16 *att,
                     int *status, cudaStream_t st);

// y = bf16(LN(x) * g + b) over rows of 640 (g, b may be null for no affine).
// With pool_q set, also logits[row] = y_row . pool_q + pool_qb in f32, in the
// summation order of the pooling kernel (the last layer's LN2 feeds pooling).
void launch_layernorm640(const __nv_bfloat16 *x, int64_t M, const float *g, const float *b, __nv_bfloat16 *y,
                         cudaStream_t st, const float *pool_q = nullptr, float pool_qb = 0.f,
                         float *logits = nullptr);

// fused[i, col0:col0+640] = bf16(sum_t softmax_t(x_t . q + qb) x_t) (tessera_cpu.cpp:434-455).
// logits: the per-token logits x_t . q + qb from launch_layernorm640, or null
// to compute them here (a second read of x).
void launch_pool(const __nv_bfloat16 *x, Segs segs, int64_t npix, const float *q, float qb, __nv_bfloat16 *fused,
                 int col0, cudaStream_t st, const float *logits = nullptr);

// r = relu(bf16(LN2560(r) * g + b)) in place (tessera_cpu.cpp:568-571).
void launch_ln_relu2560(__nv_bfloat16 *r, int64_t P, const float *g, const float *b, cudaStream_t st);

// Final LN(128, no affine) rounded to bf16. Either written as f32 (out != null)
// or quantised to int8 codes + f32 scale (tessera_encode.cpp:344-361).
// Pixels with empty[i] != 0 produce the all-zero embedding.
void launch_out128(const __nv_bfloat16 *r2, int64_t P, const uint8_t *empty, float *out, int8_t *codes,
                   float *scales, cudaStream_t st);

// Bounded-wait probe: waits limit_ns on an mbarrier nothing signals, then sets *status.
void launch_wait_probe(uint64_t limit_ns, int *status, cudaStream_t st);

}  // namespace tcb
