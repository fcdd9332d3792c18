// Host interface of the tcgen05 GEMM (gemm_sm100.cu).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace tcb {

// out = round_bf16([relu](A . W^T + bias) [+ residual]) for row-major bf16 A [M, K]
// and W [N, K]. Exactly one residual source may be set: `res` (a bf16 matrix
// with pitch ldr) or `pe_doy` (per-row day of year; the residual row is the
// bf16 sinusoid of that day, from `pe_table` when the day is an integer in
// [0, 366], else computed from `pe_div`).
struct GemmArgs {
    int M = 0, N = 0, K = 0;
    const float *bias = nullptr;
    int relu = 0;
    const __nv_bfloat16 *res = nullptr;
    int ldr = 0;
    const float *pe_doy = nullptr;
    int pe_stride = 1;
    const __nv_bfloat16 *pe_table = nullptr;
    const float *pe_div = nullptr;
    __nv_bfloat16 *out = nullptr;
    int ldo = 0;
    int *status = nullptr;  // device status word (0 = ok)
    // When set (N = 640 only): out = bf16(LayerNorm(y) * ln_g + ln_b) of the
    // bf16-rounded y = [relu](A W^T + bias) + residual, eps 1e-5, fused in the
    // epilogue of a 4-CTA cluster (one 160-column tile per CTA).
    const float *ln_g = nullptr;
    const float *ln_b = nullptr;
};

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row pitch
// ld_elems, the given box and swizzle. Throws on misaligned base or pitch.
void make_tmap_box(CUtensorMap *tm, const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                   uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle);

// Tile width BN used for a given N by the single-CTA kernel (0 = unsupported):
// 256, with a narrower last tile when 256 does not divide N; 128 for N = 128.
int gemm_pick_bn(int N);

// Kernel forced by TC_GEMM_VARIANT for launch_gemm's variant 0, or 0 when the
// choice is per layer: 1 = single CTA (M = 128 token tiles), 2 = CTA pair
// (cta_group::2, M = 256 tiles), 3 = operand-swapped (the weights on the MMA's
// M side, 128 features x 256 tokens per tile), 4 = operand-swapped CTA pair
// (256 features x 256 tokens per pair; layers with a residual run on 3).
int gemm_default_variant();

// Enqueue one GEMM on `st`. bn = 0 picks the tile width; max_ctas > 0 caps the
// persistent grid; variant 0 = per layer (when N is a multiple of 128: the
// operand-swapped kernel without a residual, or its CTA-pair form there with
// TC_GEMM_TN_PAIR=1, and with a residual behind K >= 2048; else the single-CTA
// kernel), 1 = single CTA, 2 = CTA pair, 3 = operand-swapped, 4 =
// operand-swapped pair. The operand-swapped kernels give the single-CTA
// kernel's bits (tests/test_gpu_ops.py).
// Throws std::runtime_error on unsupported shapes.
void launch_gemm(const GemmArgs &p, const __nv_bfloat16 *A, int lda, const __nv_bfloat16 *W, cudaStream_t st,
                 int bn = 0, int max_ctas = 0, int variant = 0);

}  // namespace tcb
