/* tessera_b200.h - C ABI of libtessera_b200.so, the sm_100a back end of the
 * Tessera v2 Large pixel-student encoder.
 *
 * The first four functions are the reference's back-end API, with identical
 * signatures and semantics, so the reference driver links against this
 * library unchanged. The rest are additive entry points of this back end.
 * No function lets a C++ exception escape; errors are reported by return
 * value and a "tc_...: message" line on stderr, as the reference does.
 */
#ifndef TESSERA_B200_H
#define TESSERA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference back-end API -------------------------------------------- */

/* Replaces tc_create (declared src/tessera_encode.cpp:48; CPU
 * src/tessera_cpu.cpp:482-516, CUDA src/tessera_cuda.cu:598-643).
 * Loads a .tcw weight file onto the current CUDA device. block_pixels is
 * accepted for compatibility and ignored, as the CUDA back end does.
 * Returns NULL (and prints "tc_create: ...") on failure. */
void *tc_create(const char *weights_path, int block_pixels);

/* Replaces tc_encode (declared src/tessera_encode.cpp:49; CPU
 * src/tessera_cpu.cpp:518-598, CUDA src/tessera_cuda.cu:645-708).
 * s2: host f32 (G, T2, 11) = 10 z-scored bands + day of year.
 * s1: host f32 (G, T1, 3)  = VV, VH z-scored + day of year.
 * out: host f32 (G, 128), bf16-representable values.
 * 1 <= T2, T1 <= 256. Synchronous. Returns 0, or -1 on failure. */
int tc_encode(void *h, const float *s2, int64_t G, int64_t T2, const float *s1, int64_t T1, float *out);

/* Replaces tc_profile_dump (declared src/tessera_encode.cpp:50; CPU
 * src/tessera_cpu.cpp:603-637, CUDA src/tessera_cuda.cu:710-726).
 * Prints "TCPROF ..." lines to stdout. */
void tc_profile_dump(void *h);

/* Replaces tc_destroy (declared src/tessera_encode.cpp:51; CPU
 * src/tessera_cpu.cpp:639, CUDA src/tessera_cuda.cu:728). Frees all device
 * memory of the handle. */
void tc_destroy(void *h);

/* ---- additive entry points ---------------------------------------------- */

/* One handle over several GPUs: weights replicated per device. A tile is split
 * by pixel rows across the devices (no inter-GPU traffic). devices = NULL
 * means devices 0..ndev-1. Returns NULL on failure. */
void *tc_create_multi(const char *weights_path, const int *devices, int ndev);

/* Whole-tile encode from the raw staged arrays (layout of the reference
 * driver's load_tile, src/tessera_encode.cpp:182-209; dtypes checked at
 * src/tessera_encode.cpp:237-243):
 *   bands (T2,H,W,10) u16, masks (T2,H,W) u8, doys (T2) u16,
 *   asc (Ta,H,W,2) i16, asc_doy (Ta) i16, desc (Td,H,W,2) i16, desc_doy (Td) i16.
 * Does binning, padding and standardisation (src/tessera_encode.cpp:245-329),
 * the network, and the int8 quantisation (src/tessera_encode.cpp:344-361) on
 * the GPU(s). Outputs: codes (H,W,128) i8 and scales (H,W) f32, host memory.
 * Host pointers; pinned memory makes the copies faster. Ta or Td may be 0
 * (their pointers may then be NULL). Returns 0, or -1 on failure. */
int tc_encode_tile(void *h, const uint16_t *bands, const uint8_t *masks, const uint16_t *doys, const int16_t *asc,
                   const int16_t *asc_doy, const int16_t *desc, const int16_t *desc_doy, int64_t T2, int64_t Ta,
                   int64_t Td, int64_t H, int64_t W, int8_t *codes, float *scales);

/* As tc_encode_tile, for pixel rows [row0, row1) only. codes/scales still
 * point at the whole-tile outputs; only the selected rows are written. */
int tc_encode_tile_rows(void *h, const uint16_t *bands, const uint8_t *masks, const uint16_t *doys,
                        const int16_t *asc, const int16_t *asc_doy, const int16_t *desc, const int16_t *desc_doy,
                        int64_t T2, int64_t Ta, int64_t Td, int64_t H, int64_t W, int64_t row0, int64_t row1,
                        int8_t *codes, float *scales);

/* As tc_encode_tile_rows, with every array already in the memory of the
 * handle's (single) device. Enqueued on the handle's stream; returns after
 * the work completes. */
int tc_encode_tile_device(void *h, const uint16_t *bands, const uint8_t *masks, const uint16_t *doys,
                          const int16_t *asc, const int16_t *asc_doy, const int16_t *desc, const int16_t *desc_doy,
                          int64_t T2, int64_t Ta, int64_t Td, int64_t H, int64_t W, int64_t row0, int64_t row1,
                          int8_t *codes, float *scales);

/* Splits the H rows of a tile into nparts contiguous bands of near-equal
 * algorithmic FLOP (per-pixel cost from its bins), on the host.
 * row_bounds receives nparts + 1 values: band k is [row_bounds[k], row_bounds[k+1]).
 * Returns 0, or -1 on bad arguments. */
int tc_plan_rows(const uint8_t *masks, const int16_t *asc, const int16_t *desc, int64_t T2, int64_t Ta, int64_t Td,
                 int64_t H, int64_t W, int nparts, int64_t *row_bounds);

/* Page-locked host memory usable by every device (cudaHostAllocPortable), so
 * a caller's tile and output buffers are copied at full PCIe/C2C speed by the
 * tile entry points without the caller linking the CUDA runtime itself.
 * No reference counterpart. Returns NULL (and prints "tc_host_alloc: ...")
 * on failure; tc_host_free(NULL) is a no-op. */
void *tc_host_alloc(int64_t bytes);
void tc_host_free(void *p);

/* Run the handle's work on a caller-owned cudaStream_t (single-device
 * handles only); NULL restores the handle's own stream. Returns 0 or -1. */
int tc_set_stream(void *h, void *stream);

/* Profiling categories of tc_stats.ms_cat. */
enum {
    TC_CAT_H2D = 0,
    TC_CAT_PREP,      /* valid counts, gather + z-score */
    TC_CAT_EMB1,      /* K=10/2 embedding layer */
    TC_CAT_GEMM,      /* every tcgen05 GEMM launch */
    TC_CAT_ATTN,      /* per-pixel self-attention */
    TC_CAT_LN,        /* backbone LayerNorms */
    TC_CAT_POOL,      /* attention pooling */
    TC_CAT_HEAD,      /* head LayerNorms + quantisation */
    TC_CAT_D2H,
    TC_CAT_N
};

typedef struct {
    double calls;          /* encode calls since the last reset */
    double pixels;         /* pixels encoded */
    double tokens;         /* time-step tokens run through a backbone */
    double alg_flop;       /* algorithmic FLOP: dense layers on real tokens + dense attention + head */
    double gemm_flop;      /* 2*M*N*K summed over GEMM launches (real rows only) */
    double gemm_launches;  /* number of GEMM launches */
    double launches;       /* number of kernel launches of this library */
    double ms_cat[TC_CAT_N]; /* per-category device time, only while profiling is on */
    /* GEMM time and 2*M*N*K by layer (profiling on): emb2, QKV, out-proj, FFN1, FFN2, head */
    double gemm_ms_kind[6];
    double gemm_flop_kind[6];
} tc_stats;

/* Per-launch CUDA-event timing by category (adds one event per launch). */
int tc_set_profiling(void *h, int enable);
/* Cumulative counters since the last reset (summed over devices). */
int tc_get_stats(void *h, tc_stats *out);
void tc_reset_stats(void *h);

#ifdef __cplusplus
}
#endif

#endif /* TESSERA_B200_H */
