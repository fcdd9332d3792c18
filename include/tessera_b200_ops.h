/* tessera_b200_ops.h - per-kernel entry points of libtessera_b200.so, for
 * parity tests of each stage of the forward pass against the CPU oracle.
 *
 * Every pointer is device memory of the current CUDA device; every call
 * enqueues on `stream` (a cudaStream_t, NULL = legacy default stream) and
 * returns 0, or -1 with a "tcb_op_...: message" line on stderr. bf16 arrays
 * are passed as raw 16-bit storage (void *).
 */
#ifndef TESSERA_B200_OPS_H
#define TESSERA_B200_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out[M,N] = bf16([relu](A[M,K] W[N,K]^T + bias) + residual).
 * Replaces the reference's Linear (src/tessera_cpu.cpp:215-243 make_linear,
 * src/tessera_cuda.cu:438-445 gemm). Residual: res (pitch ldr), or the DOY
 * sinusoid of pe_doy[row * pe_stride] looked up in pe_table (367 x 640 bf16,
 * src/tessera_cpu.cpp:503-509) with pe_div (320 f32) for non-table days.
 * bn = tile width (0 = automatic); variant 0 = default kernel, 1 = single-CTA
 * (M = 128 tiles), 2 = CTA pair (tcgen05 cta_group::2, M = 256 tiles). */
int tcb_op_gemm(const void *A, int lda, const void *W, const float *bias, int relu, const void *res, int ldr,
                const float *pe_doy, int pe_stride, const void *pe_table, const float *pe_div, void *out, int ldo,
                int M, int N, int K, int bn, int variant, int *status, void *stream);

/* out[M,640] = bf16(LayerNorm(y) * ln_g + ln_b), y = bf16(A[M,K] W[640,K]^T + bias + res),
 * LayerNorm eps 1e-5 over the 640 columns: the reference's out-proj + LN1 and
 * FFN2 + LN2 (src/tessera_cpu.cpp:424-428, 245-263) fused into one GEMM whose
 * epilogue exchanges row statistics across a 4-CTA cluster. */
int tcb_op_gemm_ln(const void *A, int lda, const void *W, const float *bias, const void *res, int ldr,
                   const float *ln_g, const float *ln_b, void *out, int ldo, int M, int K, int *status, void *stream);

/* Allocation-free form of tcb_op_gemm_ln, with no counterpart in the
 * reference. For callers that may not allocate device memory, such as a plugin
 * whose host framework owns the whole device-memory budget, or a hot path
 * where cudaMalloc could fail or would synchronise the device: the caller
 * passes inputs and the output only (out has pitch 640), and the intermediate
 * rows and status word live in a fixed 10 MiB static device array that every
 * GPU loading this library holds until exit. M is at most 8192 (larger M
 * returns -1 with a message). The first call on a device looks up the array's
 * address, so make it before any stream capture. Calls share the array: two
 * calls that overlap on the GPU race. Returns after the work completes. */
int tcb_op_gemm_ln_noalloc(const void *A, int lda, const void *W, const float *bias, const void *res, int ldr,
                           const float *ln_g, const float *ln_b, void *out, int M, int K, void *stream);

/* Valid-observation counts (src/tessera_encode.cpp:245-257) of pixels [p0, p0+np). */
int tcb_op_count(const uint8_t *masks, const int16_t *asc, const int16_t *desc, int64_t T2, int64_t Ta, int64_t Td,
                 int64_t N, int64_t p0, int64_t np, int32_t *n2, int32_t *n1, void *stream);

/* Gather + pad + z-score of one modality (src/tessera_encode.cpp:281-329).
 * bins[i] = rows of pixel i, off[i] = its first record (np + 1 entries);
 * rec receives (sum bins, C+1) f32 records. */
int tcb_op_gather(int modality, const uint16_t *bands, const uint8_t *masks, const uint16_t *doys,
                  const int16_t *asc, const int16_t *asc_doy, const int16_t *desc, const int16_t *desc_doy,
                  int64_t T2, int64_t Ta, int64_t Td, int64_t N, int64_t p0, int64_t np, const int32_t *bins,
                  const int64_t *off, float *rec, void *stream);

/* emb1: y = bf16(relu(bf16(rec[:, :C]) W1^T + b1)); w1t = W1^T as f32 (C x 640)
 * (src/tessera_cpu.cpp:387-404). */
int tcb_op_emb1(int C, const float *rec, int64_t M, const float *w1t, const float *b1, void *y, void *stream);

/* Self-attention per pixel segment (src/tessera_cpu.cpp:333-352,410-418).
 * off (npix+1 entries, device memory) or, when NULL, uniform segments of
 * uniform_T tokens. Each pixel's kernel follows its own length, as in the
 * tile path (tcb_attention_plan): with offsets the call reads them back,
 * lists the pixels by class, runs one launch per class and synchronizes the
 * stream before returning. Tmax must be at least every segment's length
 * (-1 otherwise) and at most 256. */
int tcb_op_attention(const void *qkv, const int64_t *off, int64_t uniform_T, int64_t npix, int Tmax, void *att,
                     void *stream);

/* LayerNorm over rows of 640 (src/tessera_cpu.cpp:245-263); g/b may be NULL. */
int tcb_op_layernorm640(const void *x, int64_t M, const float *g, const float *b, void *y, void *stream);

/* Attention pooling (src/tessera_cpu.cpp:434-455) into fused[:, col0:col0+640]. */
int tcb_op_pool(const void *x, const int64_t *off, int64_t uniform_T, int64_t npix, const float *q, float qb,
                void *fused, int col0, void *stream);

/* Head LayerNorm(2560) + ReLU in place (src/tessera_cpu.cpp:568-571). */
int tcb_op_ln_relu2560(void *r, int64_t P, const float *g, const float *b, void *stream);

/* Final LayerNorm(128, no affine) -> bf16 -> f32 out, or int8 codes + scales
 * (src/tessera_cpu.cpp:573-575, src/tessera_encode.cpp:344-361). */
int tcb_op_out128(const void *r2, int64_t P, const uint8_t *empty, float *out, int8_t *codes, float *scales,
                  void *stream);

/* Attention kernel classes of a chunk's pixels (host only, no CUDA call; no
 * reference counterpart: the reference has one attention path). off[0..npix]
 * are the segment offsets. list receives the pixels with a non-empty series,
 * class by class in pixel order: class 0 the mma.sync kernel for T <= 48,
 * class 1 the tcgen05 kernel for 48 < T <= 128, class 2 the mma.sync kernel
 * for T > 128 (TC_ATTN_TC=0 / 2 move every T <= 128 to class 0 / 1).
 * n[3] receives the pixels per class and tmax[3] the longest series per
 * class. The class of a pixel depends on its own length only. Returns 0, or
 * -1 on bad arguments (null pointers, negative npix, decreasing offsets). */
int tcb_attention_plan(const int64_t *off, int64_t npix, int32_t *list, int64_t *n, int32_t *tmax);

/* Failure-detection probe (no reference counterpart: the reference has no
 * device-side waits). One kernel waits limit_us on an mbarrier that nothing
 * signals, through the same bounded wait every pipeline kernel uses, then
 * writes its error code (6) to *status and returns; the context stays usable. */
int tcb_op_wait_probe(int64_t limit_us, int *status, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TESSERA_B200_OPS_H */
